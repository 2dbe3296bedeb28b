// Tile alpha blending: training forward (with per-32-instance checkpoints for the backward), inference
// forward, and the per-bucket backward.
//
// Forward semantics follow FasterGSVDACudaBackend/.../rasterization/include/kernels_forward.cuh:26-166
// and kernels_inference.cuh:11-126: 16x12 tiles, six warps each owning an 8x4 subtile, instances staged
// 192 at a time in shared memory, a Gaussian is skipped by a warp when its screen bounds miss the
// subtile, alpha = opacity * exp(-power), fragments below alpha 1/255 are skipped, blending stops once
// the transmittance falls below 1e-4. The acceptance test is evaluated as "exponent >= -ln(255 opacity)"
// against the per-primitive threshold stored by the preprocess (the same threshold the tile test uses),
// and exp is the deterministic polynomial of fgs_common.cuh.
// Backward: the gradients of include/kernels_backward.cuh:12-231 (the reference processes buckets of 32
// instances with the pixels pipelined through the lanes, which for small footprints spends most issue slots
// on pairs that do not overlap); here each warp walks its subtile's fragments front to back like the forward.
#include "launch.h"

namespace fgs {

struct Staged {
    float4 a;   // mean2d.x, mean2d.y, -power_threshold, opacity
    float4 h;   // -0.5 conic.x, -conic.y, -0.5 conic.z, unused
    float4 c;   // color rgb, unused
    uint2 bnd;  // bounds x (lo | hi << 16), y (lo | hi << 16)
};

__device__ inline void stage_record(const Record& q, Staged& s) {
    s.a = make_float4(q.q0.x, q.q0.y, -q.q0.w, q.q0.z);
    s.h = make_float4(-0.5f * q.q1.x, -q.q1.y, -0.5f * q.q1.z, 0.0f);
    s.c = make_float4(q.q2.x, q.q2.y, q.q2.z, 0.0f);
    s.bnd = make_uint2(__float_as_uint(q.q1.w), __float_as_uint(q.q2.w));
}

__device__ inline bool overlaps_subtile(uint2 bnd, uint32_t sx0, uint32_t sy0) {
    const uint32_t xlo = bnd.x & 0xffffu, xhi = bnd.x >> 16, ylo = bnd.y & 0xffffu, yhi = bnd.y >> 16;
    return xlo < sx0 + kSubtileW && sx0 < xhi && ylo < sy0 + kSubtileH && sy0 < yhi;
}

// exponent of the Gaussian at the pixel: dx * (h.x dx + h.y dy) + (h.z dy) dy
__device__ inline float gauss_exponent(float dx, float dy, float4 h) { return fmaf(dx, fmaf(h.x, dx, h.y * dy), (h.z * dy) * dy); }

template <bool kTrain>
__global__ void __launch_bounds__(kTilePixels) blend_kernel(BlendArgs A, float* __restrict__ image, TileBuffers T, int chw, int clamp_out) {
    __shared__ Staged st[kTilePixels];
    __shared__ uint32_t warp_max[kTilePixels / 32];
    const uint32_t t = threadIdx.x, lane = t & 31, warp = t >> 5;
    const uint32_t tile = blockIdx.y * A.grid_w + blockIdx.x;
    const uint32_t sx0 = blockIdx.x * kTileW + (warp % 2) * kSubtileW;
    const uint32_t sy0 = blockIdx.y * kTileH + (warp / 2) * kSubtileH;
    const uint32_t px = sx0 + lane % kSubtileW, py = sy0 + lane / kSubtileW;
    const uint32_t local = (py - blockIdx.y * kTileH) * kTileW + (px - blockIdx.x * kTileW);
    const bool inside = px < static_cast<uint32_t>(A.width) && py < static_cast<uint32_t>(A.height);
    const float pxf = static_cast<float>(px) + 0.5f, pyf = static_cast<float>(py) + 0.5f;
    const uint2 range = A.ranges[tile];
    const uint32_t n = range.y - range.x;
    float cr = 0.0f, cg = 0.0f, cbl = 0.0f, tr = 1.0f;
    uint32_t last = 0;
    bool done = !inside;
    for (uint32_t start = 0; start < n; start += kTilePixels) {
        if (__syncthreads_and(done)) break;
        if (start + t < n) {
            const uint32_t r = A.vals[range.x + start + t];
            stage_record(A.rec[r], st[t]);
        }
        __syncthreads();
        const uint32_t bs = min(static_cast<uint32_t>(kTilePixels), n - start);
        for (uint32_t g = 0; g < bs; g += 32) {
            const bool ov = g + lane < bs && overlaps_subtile(st[g + lane].bnd, sx0, sy0);
            uint32_t pending = __ballot_sync(0xffffffffu, ov);
            while (!done && pending) {
                const uint32_t k = g + __ffs(pending) - 1;
                pending &= pending - 1;
                const float4 a = st[k].a;
                const float dx = a.x - pxf, dy = a.y - pyf;
                const float e = gauss_exponent(dx, dy, st[k].h);
                if (e < a.z) continue;
                const float alpha = a.w * det_exp_blend(fminf(e, 0.0f));
                const float4 c = st[k].c;
                const float w = tr * alpha;
                cr = fmaf(w, c.x, cr);
                cg = fmaf(w, c.y, cg);
                cbl = fmaf(w, c.z, cbl);
                tr = tr * (1.0f - alpha);
                last = start + k + 1;
                if (tr < kTransmittanceThreshold) done = true;
            }
        }
    }
    if (inside) {
        cr = fmaf(tr, A.bg[0], cr);
        cg = fmaf(tr, A.bg[1], cg);
        cbl = fmaf(tr, A.bg[2], cbl);
        const size_t pix = static_cast<size_t>(py) * A.width + px;
        const size_t np = static_cast<size_t>(A.width) * A.height;
        if (kTrain) {
            image[pix] = cr;
            image[np + pix] = cg;
            image[2 * np + pix] = cbl;
            T.final_T[static_cast<size_t>(tile) * kTilePixels + local] = tr;
            T.n_contrib[static_cast<size_t>(tile) * kTilePixels + local] = last;
        } else {
            if (clamp_out) { cr = sat(cr); cg = sat(cg); cbl = sat(cbl); }
            if (chw) {
                image[pix] = cr;
                image[np + pix] = cg;
                image[2 * np + pix] = cbl;
            } else {
                image[3 * pix] = cr;
                image[3 * pix + 1] = cg;
                image[3 * pix + 2] = cbl;
            }
        }
    }
    if (kTrain) {
        uint32_t m = inside ? last : 0u;
        for (int o = 16; o > 0; o >>= 1) m = max(m, __shfl_xor_sync(0xffffffffu, m, o));
        if (lane == 0) warp_max[warp] = m;
        __syncthreads();
        if (t == 0) {
            uint32_t mm = 0;
            for (int w = 0; w < kTilePixels / 32; w++) mm = max(mm, warp_max[w]);
            T.tile_max[tile] = mm;
        }
    }
}

// ---------------------------------------------------------------------------------------------------
// backward: same tile / subtile walk as the forward, front to back. Each thread owns one pixel and re-derives
// its accepted fragments exactly as the forward did (the acceptance test and the transmittance updates are
// the same operations), stopping at the pixel's contributor count. The color still to be composited behind a
// fragment is the final color minus what was composited up to and including it. Per-fragment gradient terms
// are summed over the warp with a transposing butterfly (8 sums in 9 shuffles) and added to the primitive's
// gradient record with one atomic per value and warp. Stored sums (converted by the backward preprocess):
//   g0 = (sum h dx, sum h dy, sum h dx^2, sum h dx dy), g1 = (sum h dy^2, sum w g_rgb),
//   g2 = (sum G dL/dalpha, sum |dL/dmean2d.x|, sum |dL/dmean2d.y|, 0) with h = -alpha dL/dalpha.

// after the call, lane l holds the warp sum of value (l >> 2) of v[0..7]
__device__ inline float butterfly8(float v[8], uint32_t lane) {
    const bool b4 = lane & 16, b3 = lane & 8, b2 = lane & 4;
    float a[4];
#pragma unroll
    for (int j = 0; j < 4; j++) {
        const float keep = b4 ? v[j + 4] : v[j], send = b4 ? v[j] : v[j + 4];
        a[j] = keep + __shfl_xor_sync(0xffffffffu, send, 16);
    }
    float c[2];
#pragma unroll
    for (int j = 0; j < 2; j++) {
        const float keep = b3 ? a[j + 2] : a[j], send = b3 ? a[j] : a[j + 2];
        c[j] = keep + __shfl_xor_sync(0xffffffffu, send, 8);
    }
    float d = (b2 ? c[1] : c[0]) + __shfl_xor_sync(0xffffffffu, b2 ? c[0] : c[1], 4);
    d += __shfl_xor_sync(0xffffffffu, d, 2);
    d += __shfl_xor_sync(0xffffffffu, d, 1);
    return d;
}

__device__ inline float warp_sum(float x) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) x += __shfl_xor_sync(0xffffffffu, x, o);
    return x;
}

struct StagedB {
    float4 a;   // mean2d.x, mean2d.y, -power_threshold, opacity
    float4 h;   // -0.5 conic.x, -conic.y, -0.5 conic.z, bits(rank)
    float4 c;   // color rgb, unused
    uint2 bnd;
};

template <bool kAbs>
__global__ void __launch_bounds__(kTilePixels) blend_backward_kernel(BlendArgs A, const float* __restrict__ image, const float* __restrict__ grad_image,
                                                                     TileBuffers T, GradRecord* __restrict__ grads) {
    __shared__ StagedB st[kTilePixels];
    const uint32_t t = threadIdx.x, lane = t & 31, warp = t >> 5;
    const uint32_t tile = blockIdx.y * A.grid_w + blockIdx.x;
    const uint32_t sx0 = blockIdx.x * kTileW + (warp % 2) * kSubtileW;
    const uint32_t sy0 = blockIdx.y * kTileH + (warp / 2) * kSubtileH;
    const uint32_t px = sx0 + lane % kSubtileW, py = sy0 + lane / kSubtileW;
    const uint32_t local = (py - blockIdx.y * kTileH) * kTileW + (px - blockIdx.x * kTileW);
    const bool inside = px < static_cast<uint32_t>(A.width) && py < static_cast<uint32_t>(A.height);
    const float pxf = static_cast<float>(px) + 0.5f, pyf = static_cast<float>(py) + 0.5f;
    const uint2 range = A.ranges[tile];
    const uint32_t n = range.y - range.x;
    uint32_t last = 0;
    float cfr = 0.0f, cfg = 0.0f, cfb = 0.0f, gr = 0.0f, gg = 0.0f, gb = 0.0f, gac = 0.0f;
    if (inside) {
        const size_t pix = static_cast<size_t>(py) * A.width + px;
        const size_t np = static_cast<size_t>(A.width) * A.height;
        last = T.n_contrib[static_cast<size_t>(tile) * kTilePixels + local];
        const float tf = T.final_T[static_cast<size_t>(tile) * kTilePixels + local];
        const float bgr = A.bg[0], bgg = A.bg[1], bgb = A.bg[2];
        cfr = image[pix] - tf * bgr;
        cfg = image[np + pix] - tf * bgg;
        cfb = image[2 * np + pix] - tf * bgb;
        gr = grad_image[pix];
        gg = grad_image[np + pix];
        gb = grad_image[2 * np + pix];
        gac = tf * -(gr * bgr + gg * bgg + gb * bgb);
    }
    float tr = 1.0f, accr = 0.0f, accg = 0.0f, accb = 0.0f;
    bool done = last == 0;
    for (uint32_t start = 0; start < n; start += kTilePixels) {
        if (__syncthreads_and(done)) break;
        if (start + t < n) {
            const uint32_t r = A.vals[range.x + start + t];
            const Record q = A.rec[r];
            StagedB& s = st[t];
            s.a = make_float4(q.q0.x, q.q0.y, -q.q0.w, q.q0.z);
            s.h = make_float4(-0.5f * q.q1.x, -q.q1.y, -0.5f * q.q1.z, __uint_as_float(r));
            s.c = make_float4(q.q2.x, q.q2.y, q.q2.z, 0.0f);
            s.bnd = make_uint2(__float_as_uint(q.q1.w), __float_as_uint(q.q2.w));
        }
        __syncthreads();
        const uint32_t bs = min(static_cast<uint32_t>(kTilePixels), n - start);
        for (uint32_t g = 0; g < bs; g += 32) {
            const bool ov = g + lane < bs && overlaps_subtile(st[g + lane].bnd, sx0, sy0);
            uint32_t pending = __ballot_sync(0xffffffffu, ov);
            while (pending) {
                if (__all_sync(0xffffffffu, done)) break;
                const uint32_t k = g + __ffs(pending) - 1;
                pending &= pending - 1;
                const float4 a = st[k].a;
                const float4 h = st[k].h;
                const float dx = a.x - pxf, dy = a.y - pyf;
                bool acc = !done && start + k < last;
                float e = 0.0f;
                if (acc) {
                    e = gauss_exponent(dx, dy, h);
                    acc = e >= a.z;
                }
                if (!__any_sync(0xffffffffu, acc)) continue;
                float v[8] = {0.0f, 0.0f, 0.0f, 0.0f, 0.0f, 0.0f, 0.0f, 0.0f};
                float v8 = 0.0f, ax = 0.0f, ay = 0.0f;
                if (acc) {
                    const float G = det_exp_blend(fminf(e, 0.0f));
                    const float alpha = a.w * G;
                    const float4 c = st[k].c;
                    const float w = tr * alpha;
                    accr = fmaf(w, c.x, accr);
                    accg = fmaf(w, c.y, accg);
                    accb = fmaf(w, c.z, accb);
                    const float oma = 1.0f - alpha;
                    const float rcp = 1.0f / fmaxf(oma, kOneMinusAlphaEps);
                    const float afr = cfr - accr, afg = cfg - accg, afb = cfb - accb;
                    const float dl_da = (tr * c.x - afr * rcp) * gr + (tr * c.y - afg * rcp) * gg + (tr * c.z - afb * rcp) * gb + gac * rcp;
                    const float hl = -alpha * dl_da;
                    const float hx = hl * dx, hy = hl * dy;
                    v[0] = hx; v[1] = hy; v[2] = hx * dx; v[3] = hx * dy;
                    v[4] = hy * dy; v[5] = w * gr; v[6] = w * gg; v[7] = w * gb;
                    v8 = G * dl_da;
                    if (kAbs) {
                        // |dL/dmean2d| of this fragment, with the raw conic recovered exactly from the staged halves
                        const float ca = -2.0f * h.x, cb = -h.y, cc = -2.0f * h.z;
                        ax = fabsf(ca * hx + cb * hy);
                        ay = fabsf(cb * hx + cc * hy);
                    }
                    tr = tr * oma;
                    if (tr < kTransmittanceThreshold) done = true;
                }
                const float s = butterfly8(v, lane);
                const float s8 = warp_sum(v8);
                float sax = 0.0f, say = 0.0f;
                if (kAbs) { sax = warp_sum(ax); say = warp_sum(ay); }
                const uint32_t r = __float_as_uint(h.w);
                float* gp = reinterpret_cast<float*>(grads + r);
                if ((lane & 3) == 0) atomicAdd(gp + (lane >> 2), s);
                if (lane == 0) {
                    atomicAdd(gp + 8, s8);
                    if (kAbs) { atomicAdd(gp + 9, sax); atomicAdd(gp + 10, say); }
                }
            }
        }
    }
}

cudaError_t launch_blend_train(const BlendArgs& a, float* image, const TileBuffers& T, cudaStream_t s) {
    const dim3 grid(a.grid_w, a.grid_h);
    blend_kernel<true><<<grid, kTilePixels, 0, s>>>(a, image, T, 1, 0);
    return cudaGetLastError();
}

cudaError_t launch_blend_inference(const BlendArgs& a, float* image, int chw, int clamp, cudaStream_t s) {
    const dim3 grid(a.grid_w, a.grid_h);
    TileBuffers none{};
    blend_kernel<false><<<grid, kTilePixels, 0, s>>>(a, image, none, chw, clamp);
    return cudaGetLastError();
}

cudaError_t launch_blend_backward(const BlendArgs& a, const float* image, const float* grad_image, const TileBuffers& T, GradRecord* grads,
                                  int abs_grad, cudaStream_t s) {
    const dim3 grid(a.grid_w, a.grid_h);
    if (abs_grad) blend_backward_kernel<true><<<grid, kTilePixels, 0, s>>>(a, image, grad_image, T, grads);
    else blend_backward_kernel<false><<<grid, kTilePixels, 0, s>>>(a, image, grad_image, T, grads);
    return cudaGetLastError();
}

}  // namespace fgs
