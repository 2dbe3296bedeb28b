// Backward helpers shared by the preprocess backward kernels (rtc/preprocess_backward.cu:196-403 of the
// reference): conversion of the blend sums, and the chain rule from the 2D quantities to mean, log-scale and
// quaternion.
#pragma once

#include "preprocess.cuh"

namespace fgs {

// converts the blend backward's per-primitive sums into gradients w.r.t. mean2d, conic (off-diagonal halved as
// in the reference's convention) and the opacity logit (sigmoid derivative folded in unless proper antialiasing)
__device__ inline void blend_sums_to_grads(const GradRecord& g, const Record& q, int proper_aa, float& gmx, float& gmy, float& gca,
                                           float& gcb, float& gcc, float& gop) {
    const float ca = q.q1.x, cb = q.q1.y, cc = q.q1.z, o = q.q0.z;
    gmx = ca * g.g0.x + cb * g.g0.y;
    gmy = cb * g.g0.x + cc * g.g0.y;
    gca = 0.5f * g.g0.z;
    gcb = 0.5f * g.g0.w;
    gcc = 0.5f * g.g1.x;
    gop = proper_aa ? g.g2.x : (o - o * o) * g.g2.x;
}

// store, or add with a reduction (every element receives one addition per launch, so the result is the load-add-store
// value, deterministic, and the thread does not wait for the load)
__device__ inline void put(float* p, size_t k, float v, int acc) {
    if (acc) atomicAdd(p + k, v);
    else p[k] = v;
}
__device__ inline void put3(float* p, uint32_t i, f3 v, int acc) { put(p, 3ull * i, v.x, acc); put(p, 3ull * i + 1, v.y, acc); put(p, 3ull * i + 2, v.z, acc); }

// chain rule from the 2D gradients (mean2d, conic) to mean, log-scale and quaternion
// (rtc/preprocess_backward.cu:196-403); returns the mean gradient from splatting
__device__ inline f3 geometry_backward(const Params& P, const View& v, uint32_t i, f3 m, float gmx, float gmy, float gca,
                                       float gcb, float gcc, float& g_opacity, const GradOut& O) {
    const float4 w0 = reinterpret_cast<const float4*>(v.w2c)[0];
    const float4 w1 = reinterpret_cast<const float4*>(v.w2c)[1];
    const float4 w2 = reinterpret_cast<const float4*>(v.w2c)[2];
    const float depth = w2.x * m.x + w2.y * m.y + w2.z * m.z + w2.w;
    const float x = (w0.x * m.x + w0.y * m.y + w0.z * m.z + w0.w) / depth;
    const float y = (w1.x * m.x + w1.y * m.y + w1.z * m.z + w1.w) / depth;
    const f3 s = ld3(P.scales, i);
    const float vx = det_exp(2.0f * s.x), vy = det_exp(2.0f * s.y), vz = det_exp(2.0f * s.z);
    const float4 q = reinterpret_cast<const float4*>(P.rotations)[i];
    float nsq;
    const Mat3 R = quat_to_rot(q.x, q.y, q.z, q.w, nsq);
    const Mat3 RS = {R.m11 * vx, R.m12 * vy, R.m13 * vz, R.m21 * vx, R.m22 * vy, R.m23 * vz, R.m31 * vx, R.m32 * vy, R.m33 * vz};
    const float s11 = RS.m11 * R.m11 + RS.m12 * R.m12 + RS.m13 * R.m13;
    const float s12 = RS.m11 * R.m21 + RS.m12 * R.m22 + RS.m13 * R.m23;
    const float s13 = RS.m11 * R.m31 + RS.m12 * R.m32 + RS.m13 * R.m33;
    const float s22 = RS.m21 * R.m21 + RS.m22 * R.m22 + RS.m23 * R.m23;
    const float s23 = RS.m21 * R.m31 + RS.m22 * R.m32 + RS.m23 * R.m33;
    const float s33 = RS.m31 * R.m31 + RS.m32 * R.m32 + RS.m33 * R.m33;
    const float W = static_cast<float>(v.width), H = static_cast<float>(v.height);
    const float cl = (-0.15f * W - v.cx) / v.fx, cr = (1.15f * W - v.cx) / v.fx;
    const float ct = (-0.15f * H - v.cy) / v.fy, cbm = (1.15f * H - v.cy) / v.fy;
    const float xc = clampf(x, cl, cr), yc = clampf(y, ct, cbm);
    const float j11 = v.fx / depth, j13 = -j11 * xc, j22 = v.fy / depth, j23 = -j22 * yc;
    const f3 a1 = mk3(j11 * w0.x + j13 * w2.x, j11 * w0.y + j13 * w2.y, j11 * w0.z + j13 * w2.z);
    const f3 a2 = mk3(j22 * w1.x + j23 * w2.x, j22 * w1.y + j23 * w2.y, j22 * w1.z + j23 * w2.z);
    const f3 b1 = mk3(a1.x * s11 + a1.y * s12 + a1.z * s13, a1.x * s12 + a1.y * s22 + a1.z * s23, a1.x * s13 + a1.y * s23 + a1.z * s33);
    const f3 b2 = mk3(a2.x * s11 + a2.y * s12 + a2.z * s13, a2.x * s12 + a2.y * s22 + a2.z * s23, a2.x * s13 + a2.y * s23 + a2.z * s33);
    const float a_raw = dot3(b1, a1), b = dot3(b1, a2), c_raw = dot3(b2, a2);
    const float k = v.proper_aa ? kDilationProperAA : kDilation;
    const float a = a_raw + k, c = c_raw + k;
    const float aa = a * a, bb = b * b, cc = c * c, ac = a * c, ab = a * b, bc = b * c;
    const float det = ac - bb;
    const float inv_det2 = 1.0f / (det * det);
    // d/d(cov2d); the off-diagonal entries follow the symmetric-matrix convention of the blend gradients
    const float gA = inv_det2 * (2.0f * bc * gcb - cc * gca - bb * gcc);
    const float gB = inv_det2 * (bc * gca - (ac + bb) * gcb + ab * gcc);
    const float gC = inv_det2 * (2.0f * ab * gcb - bb * gca - aa * gcc);
    if (v.proper_aa) {
        const float o = det_sigmoid(P.opacities[i]);
        const float conv = sqrtf(fmaxf((a_raw * c_raw - bb) / det, 0.0f));
        g_opacity = g_opacity * conv * o * (1.0f - o);
    }
    // d/d(cov3d) (upper triangle)
    const float d11 = a1.x * a1.x * gA + 2.0f * a1.x * a2.x * gB + a2.x * a2.x * gC;
    const float d12 = a1.x * a1.y * gA + (a1.x * a2.y + a1.y * a2.x) * gB + a2.x * a2.y * gC;
    const float d13 = a1.x * a1.z * gA + (a1.x * a2.z + a1.z * a2.x) * gB + a2.x * a2.z * gC;
    const float d22 = a1.y * a1.y * gA + 2.0f * a1.y * a2.y * gB + a2.y * a2.y * gC;
    const float d23 = a1.y * a1.z * gA + (a1.y * a2.z + a1.z * a2.y) * gB + a2.y * a2.z * gC;
    const float d33 = a1.z * a1.z * gA + 2.0f * a1.z * a2.z * gB + a2.z * a2.z * gC;
    // d/d(J W) rows
    const f3 ga1 = 2.0f * mk3(b1.x * gA + b2.x * gB, b1.y * gA + b2.y * gB, b1.z * gA + b2.z * gB);
    const f3 ga2 = 2.0f * mk3(b1.x * gB + b2.x * gC, b1.y * gB + b2.y * gC, b1.z * gB + b2.z * gC);
    const float gj11 = w0.x * ga1.x + w0.y * ga1.y + w0.z * ga1.z;
    const float gj22 = w1.x * ga2.x + w1.y * ga2.y + w1.z * ga2.z;
    const float gj13 = w2.x * ga1.x + w2.y * ga1.y + w2.z * ga1.z;
    const float gj23 = w2.x * ga2.x + w2.y * ga2.y + w2.z * ga2.z;
    if (O.densification != nullptr) {
        float* di = O.densification;
        const size_t n = P.n;
        di[i] += 1.0f;
        const float nx = 0.5f * (gmx * W), ny = 0.5f * (gmy * H);
        di[n + i] += sqrtf(nx * nx + ny * ny);
    }
    // camera-space mean from the projection and from J (with the guard-band clip masks)
    f3 gcam = mk3(j11 * gmx, j22 * gmy, -j11 * x * gmx - j22 * y * gmy);
    const bool vx_ok = x >= cl && x <= cr;
    const bool vy_ok = y >= ct && y <= cbm;
    if (vx_ok) gcam.x -= j11 * gj13 / depth;
    if (vy_ok) gcam.y -= j22 * gj23 / depth;
    const float fx_ = 1.0f + (vx_ok ? 1.0f : 0.0f), fy_ = 1.0f + (vy_ok ? 1.0f : 0.0f);
    gcam.z += (j11 * (fx_ * xc * gj13 - gj11) + j22 * (fy_ * yc * gj23 - gj22)) / depth;
    const f3 gmean = mk3(w0.x * gcam.x + w1.x * gcam.y + w2.x * gcam.z, w0.y * gcam.x + w1.y * gcam.y + w2.y * gcam.z,
                         w0.z * gcam.x + w1.z * gcam.y + w2.z * gcam.z);
    // log-scale
    const f3 gvar = mk3(R.m11 * R.m11 * d11 + R.m21 * R.m21 * d22 + R.m31 * R.m31 * d33 + 2.0f * (R.m11 * R.m21 * d12 + R.m11 * R.m31 * d13 + R.m21 * R.m31 * d23),
                        R.m12 * R.m12 * d11 + R.m22 * R.m22 * d22 + R.m32 * R.m32 * d33 + 2.0f * (R.m12 * R.m22 * d12 + R.m12 * R.m32 * d13 + R.m22 * R.m32 * d23),
                        R.m13 * R.m13 * d11 + R.m23 * R.m23 * d22 + R.m33 * R.m33 * d33 + 2.0f * (R.m13 * R.m23 * d12 + R.m13 * R.m33 * d13 + R.m23 * R.m33 * d23));
    put3(O.scales, i, 2.0f * mk3(vx, vy, vz) * gvar, O.accumulate);
    // rotation matrix, then the (unnormalised) quaternion
    const Mat3 gR = {2.0f * (RS.m11 * d11 + RS.m21 * d12 + RS.m31 * d13), 2.0f * (RS.m12 * d11 + RS.m22 * d12 + RS.m32 * d13),
                     2.0f * (RS.m13 * d11 + RS.m23 * d12 + RS.m33 * d13), 2.0f * (RS.m11 * d12 + RS.m21 * d22 + RS.m31 * d23),
                     2.0f * (RS.m12 * d12 + RS.m22 * d22 + RS.m32 * d23), 2.0f * (RS.m13 * d12 + RS.m23 * d22 + RS.m33 * d23),
                     2.0f * (RS.m11 * d13 + RS.m21 * d23 + RS.m31 * d33), 2.0f * (RS.m12 * d13 + RS.m22 * d23 + RS.m32 * d33),
                     2.0f * (RS.m13 * d13 + RS.m23 * d23 + RS.m33 * d33)};
    {
        const float r = q.x, qx = q.y, qy = q.z, qz = q.w;
        const float xx = qx * qx, yy = qy * qy, zz = qz * qz, xy = qx * qy, xz = qx * qz, yz = qy * qz;
        const float rx = r * qx, ry = r * qy, rz = r * qz;
        const float ns = r * r + xx + yy + zz;
        const float t = 2.0f * (1.0f / ns);
        const float g_xx = gR.m22 + gR.m33, g_yy = gR.m11 + gR.m33, g_zz = gR.m11 + gR.m22;
        const float g_rz = gR.m21 - gR.m12, g_xy = gR.m21 + gR.m12;
        const float g_ry = gR.m13 - gR.m31, g_xz = gR.m13 + gR.m31;
        const float g_rx = gR.m32 - gR.m23, g_yz = gR.m32 + gR.m23;
        const float h = t * (xy * g_xy + xz * g_xz + yz * g_yz + rx * g_rx + ry * g_ry + rz * g_rz - xx * g_xx - yy * g_yy - zz * g_zz);
        const float gr = t * (qx * g_rx + qy * g_ry + qz * g_rz - r * h);
        const float gx = t * (r * g_rx - 2.0f * qx * g_xx + qy * g_xy + qz * g_xz - qx * h);
        const float gy = t * (r * g_ry + qx * g_xy - 2.0f * qy * g_yy + qz * g_yz - qy * h);
        const float gz = t * (r * g_rz + qx * g_xz + qy * g_yz - 2.0f * qz * g_zz - qz * h);
        put(O.rotations, 4ull * i, gr, O.accumulate);
        put(O.rotations, 4ull * i + 1, gx, O.accumulate);
        put(O.rotations, 4ull * i + 2, gy, O.accumulate);
        put(O.rotations, 4ull * i + 3, gz, O.accumulate);
    }
    return gmean;
}

}  // namespace fgs
