// Forward and backward preprocess for the precomputed-colors path and the SH / SV / NASG / NASGabor
// appearance models, plus the order-preserving compaction of visible primitives and the depth-order
// gather that produces the packed render records.
//
// Forward: FasterGSVDACudaBackend/.../rasterization/rtc/preprocess_forward.cu:12-278 (geometry, culling,
// exact tile count, fused color). The reference compacts visible primitives with an atomic counter, so
// equal depth keys end up in scheduling order; here the compaction is a scan over fixed chunks, which
// keeps primitive order and makes the stable depth sort order ties by primitive index.
// Backward: rtc/preprocess_backward.cu:19-404.
#include "preprocess_store.cuh"
#include "appearance.cuh"
#include "launch.h"

namespace fgs {

template <int MODEL>
__device__ inline f3 fused_color(const Params& P, const AppearanceConfig& A, const View& v, uint32_t i, f3 mean) {
    if (MODEL == kPrecomputed) return ld3(P.precomputed, i);
    const f3 cam = mk3(v.cam_pos[0], v.cam_pos[1], v.cam_pos[2]);
    const f3 dv = mean - cam;
    const f3 d = rnorm3(dv) * dv;
    const int stride = residual_stride(MODEL, A.max_degree, 0);
    const float* rp = P.residual + static_cast<size_t>(i) * stride;
    const int deg = min(v.degree, A.max_degree);
    f3 res = mk3(0.0f, 0.0f, 0.0f);
    if (MODEL == kSH) res = sh_forward(rp, d, deg, A.res_act);
    if (MODEL == kSV) res = sv_forward(rp, d, deg, A.res_act);
    if (MODEL == kNASG) res = lobes_forward<false>(rp, d, deg, A.res_act);
    if (MODEL == kNASGabor) res = lobes_forward<true>(rp, d, deg, A.res_act);
    const f3 base = base_act3(A.base_act, ld3(P.base, i));
    f3 col = color_act3(A.color_act, base + res);
    if (!v.render_base) {
        const f3 bc = color_act3(A.color_act, base);
        col = mk3(fabsf(col.x - bc.x), fabsf(col.y - bc.y), fabsf(col.z - bc.z));
    }
    return col;
}

template <int MODEL>
__global__ void __launch_bounds__(kChunk) preprocess_fwd_kernel(Params P, AppearanceConfig A, View v, PrimBuffers B) {
    const uint32_t i = blockIdx.x * kChunk + threadIdx.x;
    const bool in_range = i < P.n;
    const Geometry G = project_primitive(P.means, P.scales, P.rotations, P.opacities, in_range ? i : 0, in_range, v);
    f3 color = mk3(0.0f, 0.0f, 0.0f);
    if (in_range && G.n_touched > 0) color = fused_color<MODEL>(P, A, v, i, ld3(P.means, i));
    store_primitive(B, i, in_range, G, color);
}

// exclusive scan of the per-chunk visible counts (one CTA); also totals visible primitives and instances
__global__ void __launch_bounds__(1024) chunk_scan_kernel(const uint2* __restrict__ stats, uint32_t* __restrict__ off,
                                                          unsigned long long* __restrict__ counters, uint32_t n_chunks) {
    __shared__ uint32_t warp_sums[32];
    __shared__ uint32_t carry;
    __shared__ unsigned long long inst_total;
    if (threadIdx.x == 0) { carry = 0; inst_total = 0; }
    __syncthreads();
    const uint32_t lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    unsigned long long my_inst = 0;
    for (uint32_t base = 0; base < n_chunks; base += 1024) {
        const uint32_t c = base + threadIdx.x;
        const uint2 s = c < n_chunks ? stats[c] : make_uint2(0, 0);
        my_inst += s.y;
        uint32_t x = s.x;
        for (int o = 1; o < 32; o <<= 1) {
            const uint32_t y = __shfl_up_sync(0xffffffffu, x, o);
            if (lane >= static_cast<uint32_t>(o)) x += y;
        }
        if (lane == 31) warp_sums[warp] = x;
        __syncthreads();
        if (warp == 0) {
            uint32_t w = warp_sums[lane];
            for (int o = 1; o < 32; o <<= 1) {
                const uint32_t y = __shfl_up_sync(0xffffffffu, w, o);
                if (lane >= static_cast<uint32_t>(o)) w += y;
            }
            warp_sums[lane] = w;
        }
        __syncthreads();
        const uint32_t incl = x + (warp > 0 ? warp_sums[warp - 1] : 0u) + carry;
        if (c < n_chunks) off[c] = incl - s.x;
        __syncthreads();
        if (threadIdx.x == 1023) carry = incl;
        __syncthreads();
    }
    atomicAdd(&inst_total, my_inst);
    __syncthreads();
    if (threadIdx.x == 0) { counters[0] = carry; counters[1] = inst_total; }
}

// writes (depth key, primitive index) of visible primitives in primitive order
__global__ void __launch_bounds__(kChunk) compact_kernel(const uint32_t* __restrict__ n_touched, const uint32_t* __restrict__ depth_key,
                                                         const uint32_t* __restrict__ chunk_off, uint32_t* __restrict__ keys,
                                                         uint32_t* __restrict__ idx, uint32_t n) {
    __shared__ uint32_t warp_counts[kChunk / 32];
    const uint32_t i = blockIdx.x * kChunk + threadIdx.x;
    const bool vis = i < n && n_touched[i] > 0;
    const uint32_t lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    const uint32_t ballot = __ballot_sync(0xffffffffu, vis);
    if (lane == 0) warp_counts[warp] = __popc(ballot);
    __syncthreads();
    uint32_t pos = chunk_off[blockIdx.x];
    for (uint32_t w = 0; w < warp; w++) pos += warp_counts[w];
    pos += __popc(ballot & ((1u << lane) - 1u));
    if (vis) {
        keys[pos] = depth_key[i];
        idx[pos] = i;
    }
}

// gathers records into depth order, records the rank of every visible primitive, and the tile counts
__global__ void reorder_kernel(const uint32_t* __restrict__ sorted_idx, const Record* __restrict__ rec,
                               const uint32_t* __restrict__ n_touched, Record* __restrict__ sorted_rec,
                               uint32_t* __restrict__ counts, uint32_t* __restrict__ rank_of, uint32_t n_visible) {
    const uint32_t r = blockIdx.x * blockDim.x + threadIdx.x;
    if (r >= n_visible) return;
    const uint32_t i = sorted_idx[r];
    sorted_rec[r] = rec[i];
    counts[r] = n_touched[i];
    rank_of[i] = r;
}

// ----------------------------------------------------------------------------------------------------
// backward preprocess



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

__device__ inline void put(float* p, size_t k, float v, int acc) { if (acc) p[k] += v; else p[k] = v; }
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

template <int MODEL>
__global__ void __launch_bounds__(128) preprocess_bwd_kernel(Params P, AppearanceConfig A, View v, const uint32_t* __restrict__ rank_of,
                                                             const Record* __restrict__ sorted_rec, const GradRecord* __restrict__ grads,
                                                             GradOut O) {
    const uint32_t i = blockIdx.x * blockDim.x + threadIdx.x;
    if (i >= P.n) return;
    const uint32_t r = rank_of[i];
    const int acc = O.accumulate;
    const int stride = residual_stride(MODEL, A.max_degree, 0);
    if (r == kInvalidRank) {
        if (acc) return;
        put3(O.means, i, mk3(0.0f, 0.0f, 0.0f), 0);
        put3(O.scales, i, mk3(0.0f, 0.0f, 0.0f), 0);
        for (int k = 0; k < 4; k++) O.rotations[4ull * i + k] = 0.0f;
        O.opacities[i] = 0.0f;
        if (MODEL == kPrecomputed) put3(O.precomputed, i, mk3(0.0f, 0.0f, 0.0f), 0);
        else {
            put3(O.base, i, mk3(0.0f, 0.0f, 0.0f), 0);
            for (int k = 0; k < stride; k++) O.residual[static_cast<size_t>(i) * stride + k] = 0.0f;
        }
        return;
    }
    const GradRecord g = grads[r];
    const Record rq = sorted_rec[r];
    const f3 g_color = mk3(g.g1.y, g.g1.z, g.g1.w);
    const f3 m = ld3(P.means, i);
    f3 gmean_color = mk3(0.0f, 0.0f, 0.0f);
    if (MODEL == kPrecomputed) {
        put3(O.precomputed, i, g_color, acc);
    } else {
        const f3 col = mk3(rq.q2.x, rq.q2.y, rq.q2.z);
        const f3 gpre = g_color * mk3(color_act_grad_from_y(A.color_act, col.x), color_act_grad_from_y(A.color_act, col.y),
                                      color_act_grad_from_y(A.color_act, col.z));
        const f3 base = ld3(P.base, i);
        const f3 gbase = v.render_base ? mk3(base_act_grad(A.base_act, base.x), base_act_grad(A.base_act, base.y),
                                             base_act_grad(A.base_act, base.z)) * gpre
                                       : mk3(0.0f, 0.0f, 0.0f);
        put3(O.base, i, gbase, acc);
        const f3 cam = mk3(v.cam_pos[0], v.cam_pos[1], v.cam_pos[2]);
        const f3 dv = m - cam;
        const float rn = rnorm3(dv);
        const f3 d = rn * dv;
        const int deg = min(v.degree, A.max_degree);
        const float* rp = P.residual + static_cast<size_t>(i) * stride;
        float* gr = O.residual + static_cast<size_t>(i) * stride;
        // gradients go straight to the output row; only the accumulating mode stages them (the largest supported
        // row is 10 NASGabor lobes, 90 floats)
        float local[kMaxResidualStride];
        float* out = acc ? local : gr;
        f3 gd = mk3(0.0f, 0.0f, 0.0f);
        if (MODEL == kSH) gd = sh_backward(rp, gpre, d, deg, A.res_act, out);
        if (MODEL == kSV) gd = sv_backward(rp, gpre, d, deg, A.res_act, out);
        if (MODEL == kNASG) gd = lobes_backward<false>(rp, gpre, d, deg, A.res_act, out);
        if (MODEL == kNASGabor) gd = lobes_backward<true>(rp, gpre, d, deg, A.res_act, out);
        const int active = residual_active(MODEL, deg, 0);
        if (acc) {
            for (int k = 0; k < active; k++) gr[k] += local[k];
        } else {
            for (int k = active; k < stride; k++) gr[k] = 0.0f;
        }
        gmean_color = rn * (gd - dot3(gd, d) * d);
    }
    float gmx, gmy, gca, gcb, gcc, g_opacity;
    blend_sums_to_grads(g, rq, v.proper_aa, gmx, gmy, gca, gcb, gcc, g_opacity);
    const f3 gmean = geometry_backward(P, v, i, m, gmx, gmy, gca, gcb, gcc, g_opacity, O);
    if (O.densification != nullptr && O.densification_rows == 3) {
        const float nx = 0.5f * (g.g2.y * static_cast<float>(v.width)), ny = 0.5f * (g.g2.z * static_cast<float>(v.height));
        O.densification[2ull * P.n + i] += sqrtf(nx * nx + ny * ny);
    }
    put(O.opacities, i, g_opacity, acc);
    put3(O.means, i, A.dir_grad ? gmean + gmean_color : gmean, acc);
}

// ----------------------------------------------------------------------------------------------------
// launchers

static int grid_of(uint64_t n, int block) { return static_cast<int>((n + block - 1) / block); }

cudaError_t launch_preprocess_fwd(const Params& P, const AppearanceConfig& A, const View& v, const PrimBuffers& B, bool precomputed,
                                  cudaStream_t s) {
    const int grid = grid_of(P.n, kChunk);
    if (grid == 0) return cudaSuccess;
    const int model = precomputed ? kPrecomputed : A.model;
    switch (model) {
        case kPrecomputed: preprocess_fwd_kernel<kPrecomputed><<<grid, kChunk, 0, s>>>(P, A, v, B); break;
        case kSH: preprocess_fwd_kernel<kSH><<<grid, kChunk, 0, s>>>(P, A, v, B); break;
        case kSV: preprocess_fwd_kernel<kSV><<<grid, kChunk, 0, s>>>(P, A, v, B); break;
        case kNASG: preprocess_fwd_kernel<kNASG><<<grid, kChunk, 0, s>>>(P, A, v, B); break;
        case kNASGabor: preprocess_fwd_kernel<kNASGabor><<<grid, kChunk, 0, s>>>(P, A, v, B); break;
        case kNeural: return launch_preprocess_fwd_neural(P, A, v, B, s);
        default: return cudaErrorInvalidValue;
    }
    return cudaGetLastError();
}

cudaError_t launch_compaction(const PrimBuffers& B, uint32_t n, cudaStream_t s) {
    const int chunks = grid_of(n, kChunk);
    if (chunks == 0) return cudaMemsetAsync(B.counters, 0, 2 * sizeof(unsigned long long), s);
    chunk_scan_kernel<<<1, 1024, 0, s>>>(B.chunk_stats, B.chunk_off, B.counters, chunks);
    compact_kernel<<<chunks, kChunk, 0, s>>>(B.n_touched, B.depth_key, B.chunk_off, B.keys_a, B.idx_a, n);
    return cudaGetLastError();
}

cudaError_t launch_reorder(const PrimBuffers& B, uint32_t n_visible, cudaStream_t s) {
    if (n_visible == 0) return cudaSuccess;
    reorder_kernel<<<grid_of(n_visible, 256), 256, 0, s>>>(B.sorted_idx, B.rec, B.n_touched, B.sorted_rec, B.inst_off, B.rank_of, n_visible);
    return cudaGetLastError();
}

cudaError_t launch_preprocess_bwd(const Params& P, const AppearanceConfig& A, const View& v, const uint32_t* rank_of,
                                  const Record* sorted_rec, const GradRecord* grads, const GradOut& O, bool precomputed,
                                  cudaStream_t s) {
    const int grid = grid_of(P.n, 128);
    if (grid == 0) return cudaSuccess;
    const int model = precomputed ? kPrecomputed : A.model;
    switch (model) {
        case kPrecomputed: preprocess_bwd_kernel<kPrecomputed><<<grid, 128, 0, s>>>(P, A, v, rank_of, sorted_rec, grads, O); break;
        case kSH: preprocess_bwd_kernel<kSH><<<grid, 128, 0, s>>>(P, A, v, rank_of, sorted_rec, grads, O); break;
        case kSV: preprocess_bwd_kernel<kSV><<<grid, 128, 0, s>>>(P, A, v, rank_of, sorted_rec, grads, O); break;
        case kNASG: preprocess_bwd_kernel<kNASG><<<grid, 128, 0, s>>>(P, A, v, rank_of, sorted_rec, grads, O); break;
        case kNASGabor: preprocess_bwd_kernel<kNASGabor><<<grid, 128, 0, s>>>(P, A, v, rank_of, sorted_rec, grads, O); break;
        case kNeural: return launch_preprocess_bwd_neural(P, A, v, rank_of, sorted_rec, grads, O, s);
        default: return cudaErrorInvalidValue;
    }
    return cudaGetLastError();
}

}  // namespace fgs
