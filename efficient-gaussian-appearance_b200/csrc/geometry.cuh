// Per-primitive projection, culling, EWA covariance, screen bounds and the exact tile-overlap test.
// Follows FasterGSVDACudaBackend/.../rasterization/rtc/preprocess_forward.cu:62-199 (forward geometry),
// include/tile_culling.cuh:13-65 (tile bounds and the StopThePop ellipse-vs-tile test) and
// rtc/preprocess_common.cuh:144-252 (quaternion -> rotation, exact tile count). The expressions are the reference's,
// term by term and in the same order, and the translation units that project (preprocess.cu) and emit (binning.cu)
// are compiled with -use_fast_math like the reference's kernels, so the opacity, covariance, conic, screen mean,
// power threshold, bounds and tile overlap decisions come out as the reference computes them.
#pragma once

#include "fgs_common.cuh"

namespace fgs {

// per-view constants; w2c, cam_pos and bg are device pointers read by every thread
struct View {
    const float* w2c;      // row-major 4x4 world-to-camera, rows 0..2 used
    const float* cam_pos;  // camera position in world space (3)
    const float* bg;       // background color (3)
    int width, height;
    float fx, fy, cx, cy;
    float near_plane, far_plane;
    int grid_w, grid_h;
    int proper_aa;
    int render_base;
    int degree;            // active appearance degree (0 when the residual is disabled)
};

struct Mat3 { float m11, m12, m13, m21, m22, m23, m31, m32, m33; };

// opacity activation of the forward projection (rtc/preprocess_common.cuh:70)
__device__ inline float opacity_sigmoid(float x) { return 1.0f / (1.0f + expf(-x)); }

__device__ inline Mat3 quat_to_rot(float r, float x, float y, float z, float& norm_sq) {
    const float xx = x * x, yy = y * y, zz = z * z;
    const float xy = x * y, xz = x * z, yz = y * z;
    const float rx = r * x, ry = r * y, rz = r * z;
    norm_sq = r * r + xx + yy + zz;
    const float s = 1.0f / norm_sq;
    Mat3 R;
    R.m11 = 1.0f - 2.0f * (yy + zz) * s; R.m12 = 2.0f * (xy - rz) * s;        R.m13 = 2.0f * (xz + ry) * s;
    R.m21 = 2.0f * (xy + rz) * s;        R.m22 = 1.0f - 2.0f * (xx + zz) * s; R.m23 = 2.0f * (yz - rx) * s;
    R.m31 = 2.0f * (xz - ry) * s;        R.m32 = 2.0f * (yz + rx) * s;        R.m33 = 1.0f - 2.0f * (xx + yy) * s;
    return R;
}

// screen-space bounds (x_min, x_max, y_min, y_max) in pixels -> tile bounds [tx0, tx1) x [ty0, ty1)
// t / w and t % w for w >= 1. For t < 2^21 (tile candidates of any image up to about 23k x 23k pixels) a float estimate
// from the approximate reciprocal (relative error about 2^-22, so t * (1 / w) is within t * 2^-21 < 1 / w of t / w)
// truncates to the quotient or one below it, and one correction step makes it exact; larger t divide as integers.
__device__ inline uint2 divmod_small(uint32_t t, uint32_t w) {
    if (t >= (1u << 21)) return make_uint2(t / w, t % w);
    uint32_t q = static_cast<uint32_t>(static_cast<float>(t) * __fdividef(1.0f, static_cast<float>(w)));
    uint32_t r = t - q * w;
    if (r >= w) {
        q += 1;
        r -= w;
    }
    return make_uint2(q, r);
}

__device__ inline uint4 tile_bounds_of(uint32_t xmin, uint32_t xmax, uint32_t ymin, uint32_t ymax) {
    return make_uint4(xmin / kTileW, (xmax + kTileW - 1) / kTileW, ymin / kTileH, (ymax + kTileH - 1) / kTileH);
}

// exact test whether the ellipse {power <= threshold} reaches the tile; m = mean2d - 0.5. The products and sums are
// the single-rounding operations the reference's contracting build evaluates tile_culling.cuh:47-62 with, written
// out so that the tile count (preprocess.cu) and the instance emission (binning.cu) take the same decisions whatever
// either translation unit contracts; the two divisions are the build's (fast-math) division in both.
__device__ inline bool tile_overlaps(float mx, float my, float cx, float cy, float cz, uint32_t tx, uint32_t ty, float thr) {
    const float rminx = static_cast<float>(tx * kTileW), rminy = static_cast<float>(ty * kTileH);
    const float rmaxx = static_cast<float>((tx + 1) * kTileW - 1), rmaxy = static_cast<float>((ty + 1) * kTileH - 1);
    const float xmd = __fsub_rn(rminx, mx);
    const float xl = xmd >= 0.0f ? 1.0f : 0.0f;
    const float nx = xl + (mx > rmaxx ? 1.0f : 0.0f);
    const float ymd = __fsub_rn(rminy, my);
    const float ya = ymd >= 0.0f ? 1.0f : 0.0f;
    const float ny = ya + (my > rmaxy ? 1.0f : 0.0f);
    if (ny + nx == 0.0f) return true;
    const float kx = __fmaf_rn(xl, __fsub_rn(rminx, rmaxx), rmaxx);
    const float ky = __fmaf_rn(ya, __fsub_rn(rminy, rmaxy), rmaxy);
    const float dfx = __fsub_rn(mx, kx), dfy = __fsub_rn(my, ky);
    const float dx = copysignf(static_cast<float>(kTileW - 1), xmd);
    const float dy = copysignf(static_cast<float>(kTileH - 1), ymd);
    const float dxcx = __fmul_rn(dx, cx), dycz = __fmul_rn(dy, cz);
    const float tx_ = __fmul_rn(ny, sat(__fmaf_rn(dxcx, dfx, __fmul_rn(__fmul_rn(dx, cy), dfy)) / __fmul_rn(dxcx, dx)));
    const float ty_ = __fmul_rn(nx, sat(__fmaf_rn(__fmul_rn(dy, cy), dfx, __fmul_rn(dycz, dfy)) / __fmul_rn(dycz, dy)));
    const float px = __fmaf_rn(tx_, dx, kx), py = __fmaf_rn(ty_, dy, ky);
    const float ex = __fsub_rn(mx, px), ey = __fsub_rn(my, py);
    const float inner = __fmaf_rn(__fmul_rn(cx, ex), ex, __fmul_rn(__fmul_rn(cz, ey), ey));
    const float maxp = __fmaf_rn(__fmul_rn(cy, ex), ey, __fmul_rn(0.5f, inner));
    return maxp <= thr;
}

// integer floor / ceil clamped to [0, hi]; the float is clamped first so the conversion is defined
__device__ inline uint32_t floor_clamped(float v, int hi) {
    const float c = clampf(v, -1.0f, static_cast<float>(hi) + 1.0f);
    const int i = static_cast<int>(floorf(c));
    return static_cast<uint32_t>(i < 0 ? 0 : (i > hi ? hi : i));
}
__device__ inline uint32_t ceil_clamped(float v, int hi) {
    const float c = clampf(v, -1.0f, static_cast<float>(hi) + 1.0f);
    const int i = static_cast<int>(ceilf(c));
    return static_cast<uint32_t>(i < 0 ? 0 : (i > hi ? hi : i));
}

struct Geometry {
    float depth;
    float mx, my;           // mean2d
    float ca, cb, cc;       // conic
    float opacity;
    float power_thr;        // ln(255 * opacity)
    uint32_t xmin, xmax, ymin, ymax;
    uint32_t n_touched;     // exact number of touched tiles, 0 when culled
};

// Projects primitive `idx` (which must be < n for active lanes). Must be called by all 32 lanes of a
// warp (the exact tile count of large footprints is computed warp-cooperatively).
__device__ inline Geometry project_primitive(const float* __restrict__ means, const float* __restrict__ scales,
                                             const float* __restrict__ rotations, const float* __restrict__ opacities,
                                             uint32_t idx, bool active, const View& v) {
    Geometry G;
    G.n_touched = 0;
    G.depth = 0.0f;
    const float4 w0 = reinterpret_cast<const float4*>(v.w2c)[0];
    const float4 w1 = reinterpret_cast<const float4*>(v.w2c)[1];
    const float4 w2 = reinterpret_cast<const float4*>(v.w2c)[2];
    f3 m = mk3(0.0f, 0.0f, 0.0f);
    if (active) m = ld3(means, idx);
    const float depth = w2.x * m.x + w2.y * m.y + w2.z * m.z + w2.w;
    if (depth < v.near_plane || depth > v.far_plane) active = false;
    G.depth = depth;
    float opacity = 0.0f, ca = 0.0f, cb = 0.0f, cc = 0.0f, a = 0.0f, c = 0.0f, mx = 0.0f, my = 0.0f;
    if (active) {
        opacity = opacity_sigmoid(opacities[idx]);
        if (opacity < kMinAlpha) active = false;
        const f3 s = ld3(scales, idx);
        const float vx = expf(2.0f * s.x), vy = expf(2.0f * s.y), vz = expf(2.0f * s.z);
        const float4 q = reinterpret_cast<const float4*>(rotations)[idx];
        float nsq;
        const Mat3 R = quat_to_rot(q.x, q.y, q.z, q.w, nsq);
        if (nsq < 1e-8f) active = false;
        const Mat3 RS = {R.m11 * vx, R.m12 * vy, R.m13 * vz, R.m21 * vx, R.m22 * vy, R.m23 * vz, R.m31 * vx, R.m32 * vy, R.m33 * vz};
        const float s11 = RS.m11 * R.m11 + RS.m12 * R.m12 + RS.m13 * R.m13;
        const float s12 = RS.m11 * R.m21 + RS.m12 * R.m22 + RS.m13 * R.m23;
        const float s13 = RS.m11 * R.m31 + RS.m12 * R.m32 + RS.m13 * R.m33;
        const float s22 = RS.m21 * R.m21 + RS.m22 * R.m22 + RS.m23 * R.m23;
        const float s23 = RS.m21 * R.m31 + RS.m22 * R.m32 + RS.m23 * R.m33;
        const float s33 = RS.m31 * R.m31 + RS.m32 * R.m32 + RS.m33 * R.m33;
        const float x = (w0.x * m.x + w0.y * m.y + w0.z * m.z + w0.w) / depth;
        const float y = (w1.x * m.x + w1.y * m.y + w1.z * m.z + w1.w) / depth;
        const float W = static_cast<float>(v.width), H = static_cast<float>(v.height);
        const float cl = (-0.15f * W - v.cx) / v.fx, cr = (1.15f * W - v.cx) / v.fx;
        const float ct = (-0.15f * H - v.cy) / v.fy, cbm = (1.15f * H - v.cy) / v.fy;
        const float xc = clampf(x, cl, cr), yc = clampf(y, ct, cbm);
        const float j11 = v.fx / depth, j13 = -j11 * xc, j22 = v.fy / depth, j23 = -j22 * yc;
        const f3 a1 = mk3(j11 * w0.x + j13 * w2.x, j11 * w0.y + j13 * w2.y, j11 * w0.z + j13 * w2.z);
        const f3 a2 = mk3(j22 * w1.x + j23 * w2.x, j22 * w1.y + j23 * w2.y, j22 * w1.z + j23 * w2.z);
        const f3 b1 = mk3(a1.x * s11 + a1.y * s12 + a1.z * s13, a1.x * s12 + a1.y * s22 + a1.z * s23, a1.x * s13 + a1.y * s23 + a1.z * s33);
        const f3 b2 = mk3(a2.x * s11 + a2.y * s12 + a2.z * s13, a2.x * s12 + a2.y * s22 + a2.z * s23, a2.x * s13 + a2.y * s23 + a2.z * s33);
        a = dot3(b1, a1);
        const float b = dot3(b1, a2);
        c = dot3(b2, a2);
        const float det_raw = a * c - b * b;
        const float k = v.proper_aa ? kDilationProperAA : kDilation;
        a = a + k;
        c = c + k;
        const float det = a * c - b * b;
        if (det < kMinCov2dDeterminant) active = false;
        ca = c / det;
        cb = -b / det;
        cc = a / det;
        if (v.proper_aa) {
            opacity = opacity * sqrtf(fmaxf(det_raw / det, 0.0f));
            if (opacity < kMinAlpha) active = false;
        }
        mx = x * v.fx + v.cx;
        my = y * v.fy + v.cy;
    }
    uint4 tb = make_uint4(0, 0, 0, 0);
    float thr = 0.0f;
    uint32_t n_max = 0;
    if (active) {
        thr = logf(opacity * kMinAlphaRcp);
        const float cutoff = 2.0f * thr;
        const float ex = fmaxf(sqrtf(a * cutoff) - 0.5f, 0.0f);
        const float ey = fmaxf(sqrtf(c * cutoff) - 0.5f, 0.0f);
        const int pw = v.grid_w * kTileW, ph = v.grid_h * kTileH;
        G.xmin = floor_clamped(mx - ex, pw);
        G.xmax = ceil_clamped(mx + ex, pw);
        G.ymin = floor_clamped(my - ey, ph);
        G.ymax = ceil_clamped(my + ey, ph);
        tb = tile_bounds_of(G.xmin, G.xmax, G.ymin, G.ymax);
        n_max = (tb.y - tb.x) * (tb.w - tb.z);
        if (n_max == 0) active = false;
    }
    G.mx = mx; G.my = my; G.ca = ca; G.cb = cb; G.cc = cc; G.opacity = opacity; G.power_thr = thr;
    // exact tile count: the warp lays its primitives' candidate tiles (bounds rectangles, row-major) end to end and
    // every lane tests one candidate per round (the same test and operands as the instance emission)
    const float sx = mx - 0.5f, sy = my - 0.5f;
    const uint32_t bw = tb.y - tb.x;
    const uint32_t lane = threadIdx.x & 31u;
    const uint32_t n_cand = active ? n_max : 0u;
    uint32_t incl = n_cand;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
        const uint32_t y = __shfl_up_sync(0xffffffffu, incl, o);
        if (lane >= static_cast<uint32_t>(o)) incl += y;
    }
    const uint32_t excl = incl - n_cand;
    const uint32_t total = __shfl_sync(0xffffffffu, incl, 31);
    uint32_t count = 0;
    for (uint32_t base = 0; base < total; base += 32) {
        const uint32_t c = base + lane;
        uint32_t owner = 0;  // last lane whose range starts at or before c
#pragma unroll
        for (int step = 16; step > 0; step >>= 1) {
            const uint32_t probe = owner + step;
            if (__shfl_sync(0xffffffffu, excl, probe) <= c) owner = probe;
        }
        const uint32_t o_excl = __shfl_sync(0xffffffffu, excl, owner);
        const float qx = __shfl_sync(0xffffffffu, sx, owner), qy = __shfl_sync(0xffffffffu, sy, owner);
        const float qa = __shfl_sync(0xffffffffu, ca, owner), qb = __shfl_sync(0xffffffffu, cb, owner);
        const float qc = __shfl_sync(0xffffffffu, cc, owner), qt = __shfl_sync(0xffffffffu, thr, owner);
        const uint32_t qx0 = __shfl_sync(0xffffffffu, tb.x, owner), qy0 = __shfl_sync(0xffffffffu, tb.z, owner);
        const uint32_t qw = __shfl_sync(0xffffffffu, bw, owner);
        const bool valid = c < total;  // then the owner has candidates and qw >= 1
        const uint2 qr = divmod_small(valid ? c - o_excl : 0u, valid ? qw : 1u);
        const bool hit = valid && tile_overlaps(qx, qy, qa, qb, qc, qx0 + qr.y, qy0 + qr.x, qt);
        const uint32_t hits = __ballot_sync(0xffffffffu, hit);
        const uint32_t lo = excl > base ? excl - base : 0u, hi = incl > base ? incl - base : 0u;
        if (lo < 32 && hi > lo) {
            const uint32_t top = hi >= 32 ? 0xffffffffu : ((1u << hi) - 1u);
            count += __popc(hits & top & ~((1u << lo) - 1u));
        }
    }
    G.n_touched = active ? count : 0;
    return G;
}

}  // namespace fgs
