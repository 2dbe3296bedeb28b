// Tile alpha blending: the training forward (which also stores each pixel's final transmittance and number of
// contributors, and each tile's largest contributor count, for the backward) and the inference forward.
//
// Semantics follow FasterGSVDACudaBackend/.../rasterization/include/kernels_forward.cuh:26-166 and
// kernels_inference.cuh:11-126: 16x12 tiles, six warps each owning an 8x4 subtile, instances staged 192 at a time in
// shared memory, a Gaussian is skipped by a warp when its screen bounds miss the subtile, alpha = opacity * G with the
// fragment's Gaussian G = exp2(min(exponent, 0)) (the exponent pre-scaled by log2 e through the staged conic),
// fragments with alpha below 1/255 are skipped, and blending stops once the transmittance falls below 1e-4. The
// exponent, alpha and the transmittance update are the reference's expressions written as explicit single-rounding
// operations (blend_common.cuh); this file is compiled with -use_fast_math like the reference's build, so exp2 is the
// same hardware approximation, and the accepted fragments and final transmittances equal the reference's bit for bit.
#include "blend_common.cuh"
#include "launch.h"

namespace fgs {

// The training forward is compiled for nine CTAs per SM (32 registers, 16 bytes spilled; measured on the c4 step: 3.60
// ms per step with the unconstrained 44 registers and seven CTAs, 3.40 at eight CTAs, 3.29 at nine); the inference
// forward keeps its unconstrained allocation (a minimum of 0 CTAs per SM sets no bound).
template <bool kTrain>
__global__ void __launch_bounds__(kTilePixels, kTrain ? 9 : 0) blend_kernel(BlendArgs A, float* __restrict__ image, TileBuffers T, int chw, int clamp_out) {
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
                const float alpha = __fmul_rn(a.w, fragment_gaussian(gauss_exponent(dx, dy, st[k].h)));
                if (alpha < kMinAlpha) continue;
                const float4 c = st[k].c;
                const float w = tr * alpha;
                cr = fmaf(w, c.x, cr);
                cg = fmaf(w, c.y, cg);
                cbl = fmaf(w, c.z, cbl);
                tr = __fmul_rn(tr, __fsub_rn(1.0f, alpha));
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
// backward (blend_bwd.cu): the same tile walk as the forward, front to back, with warps owning 8x12 column bands
// (three pixels per lane).
// Each thread re-derives the accepted fragments of its pixels exactly as the forward did (the acceptance test and the
// transmittance updates are the same operations), stopping at each pixel's contributor count. The colour still to be
// composited behind a fragment is the final colour minus what was composited up to and including it. Per-fragment
// gradient terms are added to the primitive's gradient record, per lane with 16-byte vector atomics when few lanes
// accept the fragment, else summed over the warp first with a transposing butterfly (8 sums in 9 shuffles) and
// added with one atomic per value and warp. Stored sums (converted by the backward preprocess):
//   g0 = (sum h dx, sum h dy, sum h dx^2, sum h dx dy), g1 = (sum h dy^2, sum w g_rgb),
//   g2 = (sum G dL/dalpha, sum |dL/dmean2d.x|, sum |dL/dmean2d.y|, 0) with h = -alpha dL/dalpha.

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

}  // namespace fgs
