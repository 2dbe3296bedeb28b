// Backward of the tile blend: for every pixel, the fragments of its tile are walked front to back again (the same
// acceptance and termination decisions as the forward: the exponent, alpha, 1 - alpha and the transmittance are
// evaluated with the forward's operations, blend_common.cuh), and the gradient terms of each accepted fragment are
// added to the primitive's gradient record: per lane with vector atomics when few lanes accept it, else summed over
// the warp first. Each warp owns an 8x12 column half of the tile and each lane three pixels of it, one per 4-row
// subtile, so a staged record's loads, the warp vote and the reduction serve all three.
//
// Semantics: FasterGSVDACudaBackend/.../rasterization/include/kernels_backward.cuh:12-231 (the reference processes
// buckets of 32 instances with the pixels pipelined through the lanes, which for small footprints spends most issue
// slots on pairs that do not overlap); here each warp walks its band's fragments front to back like the forward.
// This translation unit is compiled with -use_fast_math like the forward (its gradients are checked within a
// tolerance); the decisions above use the forward's explicit operations so they do not depend on contraction.
#include "blend_common.cuh"
#include "launch.h"

namespace fgs {

// reciprocal of x in [kOneMinusAlphaEps, 1] by the hardware approximation (only gradients use it; the acceptance and
// termination decisions that must match the forward do not)
__device__ inline float rcp_approx(float x) {
    float r;
    asm("rcp.approx.ftz.f32 %0, %1;" : "=f"(r) : "f"(x));
    return r;
}

// Visits with at most this many accepting lanes add per lane (the same addresses then take that many atomic additions
// in L2); above it the warp reduces first. Measured on the c4 step with 16x4 bands: 20 beats 12, 16 and 24, and every
// lane adding directly (32) triples the kernel's time through same-address serialisation; with the 8x12 bands 16 is
// slower and 24 the same.
constexpr int kDirectLanes = 20;

// Each warp owns a band of (8 JX) x (4 JY) pixels of the tile and each lane JX x JY pixels of it, (x + 8 jx, y + 4 jy):
// a staged record's loads, the warp's vote and the per-record reduction or atomics serve all of a lane's pixels.
// Measured on the c4 step (blend backward per step): 8x4 subtiles, one pixel per lane, 8.07 ms; 16x4 bands, two
// pixels, 7.62 ms; 8x12 column bands, three pixels, 7.25 ms; the whole 16x12 tile in one warp, six pixels, 10.6 ms.
// A lane's pixels 4 rows (8 columns) apart beat adjacent ones (three consecutive rows: 7.80 ms): a small footprint then
// spreads its accepting pixels over more lanes instead of making a few lanes walk several of them one after another.
constexpr int kBandJX = 1, kBandJY = 3;  // 8x12 column bands, two warps per tile
constexpr int kBandW = kSubtileW * kBandJX, kBandH = kSubtileH * kBandJY;
constexpr int kBandsX = kTileW / kBandW;
constexpr int kBwdWarps = kBandsX * (kTileH / kBandH);
constexpr int kBwdThreads = 32 * kBwdWarps;
constexpr int kLanePix = kBandJX * kBandJY;

__device__ inline bool overlaps_band(uint2 bnd, uint32_t bx0, uint32_t by0) {
    const uint32_t xlo = bnd.x & 0xffffu, xhi = bnd.x >> 16, ylo = bnd.y & 0xffffu, yhi = bnd.y >> 16;
    return xlo < bx0 + kBandW && bx0 < xhi && ylo < by0 + kBandH && by0 < yhi;
}

template <bool kAbs>
__global__ void __launch_bounds__(kBwdThreads) blend_backward_kernel(BlendArgs A, const float* __restrict__ image, const float* __restrict__ grad_image,
                                                                     TileBuffers T, GradRecord* __restrict__ grads) {
    __shared__ StagedB st[kTilePixels];
    const uint32_t t = threadIdx.x, lane = t & 31, warp = t >> 5;
    const uint32_t tile = blockIdx.y * A.grid_w + blockIdx.x;
    const uint32_t bx0 = blockIdx.x * kTileW + (warp % kBandsX) * kBandW, by0 = blockIdx.y * kTileH + (warp / kBandsX) * kBandH;
    const uint2 range = A.ranges[tile];
    const uint32_t n = range.y - range.x;
    // per pixel p = jy JX + jx: contributor count, dL/dcolour, (final colour without background) . dL/dcolour, the
    // background term, the transmittance and accd = (colour accumulated so far) . dL/dcolour
    uint32_t last[kLanePix];
    float pxf[kBandJX], pyf[kBandJY];
    float gcf[kLanePix], gr[kLanePix], gg[kLanePix], gb[kLanePix], gac[kLanePix], tr[kLanePix], accd[kLanePix];
    bool done[kLanePix];
#pragma unroll
    for (int jx = 0; jx < kBandJX; jx++) pxf[jx] = static_cast<float>(bx0 + lane % kSubtileW + kSubtileW * jx) + 0.5f;
#pragma unroll
    for (int jy = 0; jy < kBandJY; jy++) pyf[jy] = static_cast<float>(by0 + lane / kSubtileW + kSubtileH * jy) + 0.5f;
#pragma unroll
    for (int p = 0; p < kLanePix; p++) {
        const uint32_t px = bx0 + lane % kSubtileW + kSubtileW * (p % kBandJX), py = by0 + lane / kSubtileW + kSubtileH * (p / kBandJX);
        last[p] = 0u;
        gcf[p] = gr[p] = gg[p] = gb[p] = gac[p] = 0.0f;
        tr[p] = 1.0f;
        accd[p] = 0.0f;
        if (px < static_cast<uint32_t>(A.width) && py < static_cast<uint32_t>(A.height)) {
            const uint32_t local = (py - blockIdx.y * kTileH) * kTileW + (px - blockIdx.x * kTileW);
            const size_t pix = static_cast<size_t>(py) * A.width + px;
            const size_t np = static_cast<size_t>(A.width) * A.height;
            last[p] = T.n_contrib[static_cast<size_t>(tile) * kTilePixels + local];
            const float tf = T.final_T[static_cast<size_t>(tile) * kTilePixels + local];
            const float bgr = A.bg[0], bgg = A.bg[1], bgb = A.bg[2];
            const float cfr = image[pix] - tf * bgr;
            const float cfg = image[np + pix] - tf * bgg;
            const float cfb = image[2 * np + pix] - tf * bgb;
            gr[p] = grad_image[pix];
            gg[p] = grad_image[np + pix];
            gb[p] = grad_image[2 * np + pix];
            gac[p] = tf * -(gr[p] * bgr + gg[p] * bgg + gb[p] * bgb);
            gcf[p] = cfr * gr[p] + cfg * gg[p] + cfb * gb[p];
        }
        done[p] = last[p] == 0;
    }
    auto all_done = [&]() {
        bool d = true;
#pragma unroll
        for (int p = 0; p < kLanePix; p++) d = d && done[p];
        return d;
    };
    for (uint32_t start = 0; start < n; start += kTilePixels) {
        if (__syncthreads_and(all_done())) break;
        for (uint32_t u = t; u < kTilePixels; u += kBwdThreads) {
            if (start + u < n) {
                const uint32_t r = A.vals[range.x + start + u];
                const Record q = A.rec[r];
                StagedB& s = st[u];
                s.a = make_float4(q.q0.x, q.q0.y, 0.0f, q.q0.z);
                s.h = make_float4(kHalfConic * q.q1.x, kCrossConic * q.q1.y, kHalfConic * q.q1.z, __uint_as_float(r));
                s.c = make_float4(q.q2.x, q.q2.y, q.q2.z, 0.0f);
                s.bnd = make_uint2(__float_as_uint(q.q1.w), __float_as_uint(q.q2.w));
            }
        }
        __syncthreads();
        const uint32_t bs = min(static_cast<uint32_t>(kTilePixels), n - start);
        for (uint32_t g = 0; g < bs; g += 32) {
            const bool ov = g + lane < bs && overlaps_band(st[g + lane].bnd, bx0, by0);
            uint32_t pending = __all_sync(0xffffffffu, all_done()) ? 0u : __ballot_sync(0xffffffffu, ov);
            while (pending) {
                const uint32_t k = g + __ffs(pending) - 1;
                pending &= pending - 1;
                const float4 a = st[k].a;
                const float4 h = st[k].h;
                float v[8] = {0.0f, 0.0f, 0.0f, 0.0f, 0.0f, 0.0f, 0.0f, 0.0f};
                float v8 = 0.0f, ax = 0.0f, ay = 0.0f;
                bool any = false;
                float dxs[kBandJX], dys[kBandJY];
#pragma unroll
                for (int jx = 0; jx < kBandJX; jx++) dxs[jx] = a.x - pxf[jx];
#pragma unroll
                for (int jy = 0; jy < kBandJY; jy++) dys[jy] = a.y - pyf[jy];
#pragma unroll
                for (int p = 0; p < kLanePix; p++) {
                    const float dx = dxs[p % kBandJX], dy = dys[p / kBandJX];
                    bool acc = !done[p] && start + k < last[p];
                    float G = 0.0f, alpha = 0.0f;
                    if (acc) {
                        G = fragment_gaussian(gauss_exponent(dx, dy, h));
                        alpha = __fmul_rn(a.w, G);
                        acc = !(alpha < kMinAlpha);
                    }
                    if (acc) {
                        const float4 c = st[k].c;
                        const float w = tr[p] * alpha;
                        const float cg = c.x * gr[p] + c.y * gg[p] + c.z * gb[p];
                        accd[p] = fmaf(w, cg, accd[p]);
                        const float oma = __fsub_rn(1.0f, alpha);
                        const float rcp = rcp_approx(fmaxf(oma, kOneMinusAlphaEps));
                        const float dl_da = fmaf(tr[p], cg, rcp * (gac[p] - (gcf[p] - accd[p])));
                        const float hl = -alpha * dl_da;
                        const float hx = hl * dx, hy = hl * dy;
                        v[0] += hx; v[1] += hy; v[2] = fmaf(hx, dx, v[2]); v[3] = fmaf(hx, dy, v[3]);
                        v[4] = fmaf(hy, dy, v[4]); v[5] = fmaf(w, gr[p], v[5]); v[6] = fmaf(w, gg[p], v[6]); v[7] = fmaf(w, gb[p], v[7]);
                        v8 = fmaf(G, dl_da, v8);
                        if (kAbs) {
                            const float ca = h.x / kHalfConic, cb = h.y / kCrossConic, cc = h.z / kHalfConic;
                            ax += fabsf(ca * hx + cb * hy);
                            ay += fabsf(cb * hx + cc * hy);
                        }
                        tr[p] = __fmul_rn(tr[p], oma);
                        if (tr[p] < kTransmittanceThreshold) done[p] = true;
                        any = true;
                    }
                }
                const uint32_t accepting = __ballot_sync(0xffffffffu, any);
                if (!accepting) continue;
                const uint32_t r = __float_as_uint(h.w);
                float* gp = reinterpret_cast<float*>(grads + r);
                if (__popc(accepting) <= kDirectLanes) {
                    if (any) {
                        GradRecord* const gq = grads + r;
                        atomicAdd(&gq->g0, make_float4(v[0], v[1], v[2], v[3]));
                        atomicAdd(&gq->g1, make_float4(v[4], v[5], v[6], v[7]));
                        if (kAbs) atomicAdd(&gq->g2, make_float4(v8, ax, ay, 0.0f));
                        else atomicAdd(gp + 8, v8);
                    }
                } else {
                    const float s = butterfly8(v, lane);
                    const float s8 = warp_sum(v8);
                    float sax = 0.0f, say = 0.0f;
                    if (kAbs) { sax = warp_sum(ax); say = warp_sum(ay); }
                    if ((lane & 3) == 0) atomicAdd(gp + (lane >> 2), s);
                    if (lane == 0) {
                        atomicAdd(gp + 8, s8);
                        if (kAbs) { atomicAdd(gp + 9, sax); atomicAdd(gp + 10, say); }
                    }
                }
                if (__all_sync(0xffffffffu, all_done())) break;
            }
        }
    }
}

// Pruning scores (Speedy-Splat): the blend backward of an all-ones image gradient; every accepted fragment adds
// (opacity * dL/dalpha)^2 of its pixel to the score of its primitive. Semantics:
// FasterGSVDACudaBackend/.../rasterization/include/kernels_pruning_scores.cuh:11-173 (which re-runs the forward
// blend inside the kernel; here the training forward's final transmittance and contributor counts are reused, so
// the accepted fragments are exactly the forward's). The per-pixel terms are summed over the warp before the single
// addition per (fragment, warp).
__global__ void __launch_bounds__(kTilePixels) pruning_scores_kernel(BlendArgs A, const float* __restrict__ image, TileBuffers T,
                                                                     const uint32_t* __restrict__ rank_to_prim, float* __restrict__ scores) {
    __shared__ float4 sa[kTilePixels], sh[kTilePixels];
    __shared__ float sc[kTilePixels];  // colour sum c.r + c.g + c.b (the colour gradient is all ones)
    __shared__ uint2 sbnd[kTilePixels];
    __shared__ uint32_t sprim[kTilePixels];
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
    float gcf = 0.0f, gac = 0.0f;
    if (inside) {
        const size_t pix = static_cast<size_t>(py) * A.width + px;
        const size_t np = static_cast<size_t>(A.width) * A.height;
        last = T.n_contrib[static_cast<size_t>(tile) * kTilePixels + local];
        const float tf = T.final_T[static_cast<size_t>(tile) * kTilePixels + local];
        const float bgr = A.bg[0], bgg = A.bg[1], bgb = A.bg[2];
        gcf = (image[pix] - tf * bgr) + (image[np + pix] - tf * bgg) + (image[2 * np + pix] - tf * bgb);
        gac = tf * -(bgr + bgg + bgb);
    }
    float tr = 1.0f, accd = 0.0f;
    bool done = last == 0;
    for (uint32_t start = 0; start < n; start += kTilePixels) {
        if (__syncthreads_and(done)) break;
        if (start + t < n) {
            const uint32_t r = A.vals[range.x + start + t];
            const Record q = A.rec[r];
            sa[t] = make_float4(q.q0.x, q.q0.y, 0.0f, q.q0.z);
            sh[t] = make_float4(kHalfConic * q.q1.x, kCrossConic * q.q1.y, kHalfConic * q.q1.z, 0.0f);
            sc[t] = q.q2.x + q.q2.y + q.q2.z;
            sbnd[t] = make_uint2(__float_as_uint(q.q1.w), __float_as_uint(q.q2.w));
            sprim[t] = rank_to_prim[r];
        }
        __syncthreads();
        const uint32_t bs = min(static_cast<uint32_t>(kTilePixels), n - start);
        for (uint32_t g = 0; g < bs; g += 32) {
            const bool ov = g + lane < bs && overlaps_subtile(sbnd[g + lane], sx0, sy0);
            // `done` changes only where a fragment is accepted, so the warp votes on it once per group of 32
            // records and after each accepted fragment
            uint32_t pending = __all_sync(0xffffffffu, done) ? 0u : __ballot_sync(0xffffffffu, ov);
            while (pending) {
                const uint32_t k = g + __ffs(pending) - 1;
                pending &= pending - 1;
                const float4 a = sa[k];
                const float dx = a.x - pxf, dy = a.y - pyf;
                bool acc = !done && start + k < last;
                float alpha = 0.0f;
                if (acc) {
                    alpha = __fmul_rn(a.w, fragment_gaussian(gauss_exponent(dx, dy, sh[k])));
                    acc = !(alpha < kMinAlpha);
                }
                if (!__any_sync(0xffffffffu, acc)) continue;
                float score = 0.0f;
                if (acc) {
                    const float cg = sc[k];
                    accd = fmaf(tr * alpha, cg, accd);
                    const float oma = __fsub_rn(1.0f, alpha);
                    const float rcp = 1.0f / fmaxf(oma, kOneMinusAlphaEps);
                    const float dl_da = fmaf(tr, cg, rcp * (gac - (gcf - accd)));
                    const float dl_dg = a.w * dl_da;
                    score = dl_dg * dl_dg;
                    tr = __fmul_rn(tr, oma);
                    if (tr < kTransmittanceThreshold) done = true;
                }
                const float total = warp_sum(score);
                if (lane == 0) atomicAdd(scores + sprim[k], total);
                if (__all_sync(0xffffffffu, done)) break;
            }
        }
    }
}

cudaError_t launch_pruning_scores(const BlendArgs& a, const float* image, const TileBuffers& T, const uint32_t* rank_to_prim, float* scores,
                                  cudaStream_t s) {
    pruning_scores_kernel<<<dim3(a.grid_w, a.grid_h), kTilePixels, 0, s>>>(a, image, T, rank_to_prim, scores);
    return cudaGetLastError();
}

cudaError_t launch_blend_backward(const BlendArgs& a, const float* image, const float* grad_image, const TileBuffers& T, GradRecord* grads,
                                  int abs_grad, cudaStream_t s) {
    const dim3 grid(a.grid_w, a.grid_h);
    if (abs_grad) blend_backward_kernel<true><<<grid, kBwdThreads, 0, s>>>(a, image, grad_image, T, grads);
    else blend_backward_kernel<false><<<grid, kBwdThreads, 0, s>>>(a, image, grad_image, T, grads);
    return cudaGetLastError();
}

}  // namespace fgs
