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
// Backward follows include/kernels_backward.cuh:12-231 (one warp per bucket of 32 instances, pixels
// pipelined through the lanes), accumulating per-primitive gradients with 16-byte vector atomics.
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
__global__ void __launch_bounds__(kTilePixels) blend_kernel(BlendArgs A, float* __restrict__ image, TileBuffers T,
                                                            uint32_t* __restrict__ bucket_tile, float4* __restrict__ ckpt, int chw,
                                                            int clamp_out) {
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
    uint32_t bucket_base = 0;
    if (kTrain) {
        bucket_base = tile == 0 ? 0u : A.bucket_off[tile - 1];
        const uint32_t nb = (n + 31) / 32;
        for (uint32_t b = t; b < nb; b += kTilePixels) bucket_tile[bucket_base + b] = tile;
    }
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
            if (kTrain && !done) ckpt[static_cast<size_t>(bucket_base + (start + g) / 32) * kTilePixels + local] = make_float4(cr, cg, cbl, tr);
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
// backward: one warp per bucket; lane k owns instance 32*b + k, pixel state flows lane to lane
__global__ void __launch_bounds__(32) blend_backward_kernel(BlendArgs A, const float* __restrict__ image, const float* __restrict__ grad_image,
                                                            TileBuffers T, const uint32_t* __restrict__ bucket_tile,
                                                            const float4* __restrict__ ckpt, GradRecord* __restrict__ grads,
                                                            uint32_t n_tiles, int proper_aa, int abs_grad) {
    __shared__ float4 s_after[32];   // color still to be added after this bucket (rgb), transmittance at bucket start
    __shared__ float4 s_grad[32];    // dL/dpixel (rgb), -T_final <dL/dpixel, bg>
    __shared__ uint32_t s_last[32];
    const uint32_t b = blockIdx.x;
    const uint32_t lane = threadIdx.x;
    if (b >= A.bucket_off[n_tiles - 1]) return;
    const uint32_t tile = bucket_tile[b];
    const uint2 range = A.ranges[tile];
    const uint32_t n = range.y - range.x;
    const uint32_t tb = b - (tile == 0 ? 0u : A.bucket_off[tile - 1]);
    if (tb * 32 >= T.tile_max[tile]) return;
    const uint32_t k = tb * 32 + lane;
    const bool valid = k < n;
    const uint32_t tx = tile % A.grid_w, ty = tile / A.grid_w;
    const uint32_t px0 = tx * kTileW, py0 = ty * kTileH;
    uint32_t r = 0;
    float mx = 0.0f, my = 0.0f, negthr = 0.0f, o = 0.0f, ca = 0.0f, cb = 0.0f, cc = 0.0f;
    float4 h = make_float4(0.0f, 0.0f, 0.0f, 0.0f);
    float colr = 0.0f, colg = 0.0f, colb = 0.0f;
    uint32_t submask = 0;  // subtiles (2 x 3 per tile) whose rectangle the screen bounds overlap
    if (valid) {
        r = A.vals[range.x + k];
        const Record q = A.rec[r];
        mx = q.q0.x; my = q.q0.y; o = q.q0.z; negthr = -q.q0.w;
        ca = q.q1.x; cb = q.q1.y; cc = q.q1.z;
        h = make_float4(-0.5f * ca, -cb, -0.5f * cc, 0.0f);
        colr = q.q2.x; colg = q.q2.y; colb = q.q2.z;
        const uint2 bnd = make_uint2(__float_as_uint(q.q1.w), __float_as_uint(q.q2.w));
        for (uint32_t w = 0; w < kTilePixels / 32; w++)
            if (overlaps_subtile(bnd, px0 + (w % 2) * kSubtileW, py0 + (w / 2) * kSubtileH)) submask |= 1u << w;
    }
    const float bgr = A.bg[0], bgg = A.bg[1], bgb = A.bg[2];
    const size_t np = static_cast<size_t>(A.width) * A.height;
    const float4* ck = ckpt + static_cast<size_t>(b) * kTilePixels;
    float gmx = 0.0f, gmy = 0.0f, gca = 0.0f, gcb = 0.0f, gcc = 0.0f, gop = 0.0f, gr = 0.0f, gg = 0.0f, gbb = 0.0f, ax = 0.0f, ay = 0.0f;
    uint32_t last = 0;
    float afr = 0.0f, afg = 0.0f, afb = 0.0f, tr = 0.0f, pgr = 0.0f, pgg = 0.0f, pgb = 0.0f, gac = 0.0f;
    for (int i = 0; i < kTilePixels + 31; i++) {
        if ((i & 31) == 0) {
            const uint32_t lp = static_cast<uint32_t>(i) + lane;  // tile-local pixel (row-major, 16 wide)
            uint32_t lc = 0;
            float4 sa = make_float4(0.0f, 0.0f, 0.0f, 0.0f), sg = make_float4(0.0f, 0.0f, 0.0f, 0.0f);
            if (lp < static_cast<uint32_t>(kTilePixels)) {
                const uint32_t ppx = px0 + lp % kTileW, ppy = py0 + lp / kTileW;
                if (ppx < static_cast<uint32_t>(A.width) && ppy < static_cast<uint32_t>(A.height)) {
                    const size_t pix = static_cast<size_t>(ppy) * A.width + ppx;
                    const float tf = T.final_T[static_cast<size_t>(tile) * kTilePixels + lp];
                    lc = T.n_contrib[static_cast<size_t>(tile) * kTilePixels + lp];
                    if (lc > tb * 32) {  // the checkpoint of this bucket was written for this pixel
                        const float4 c0 = ck[lp];
                        sa = make_float4(image[pix] - tf * bgr - c0.x, image[np + pix] - tf * bgg - c0.y,
                                         image[2 * np + pix] - tf * bgb - c0.z, c0.w);
                        const float g0 = grad_image[pix], g1 = grad_image[np + pix], g2 = grad_image[2 * np + pix];
                        sg = make_float4(g0, g1, g2, tf * -(g0 * bgr + g1 * bgg + g2 * bgb));
                    } else {
                        lc = 0;
                    }
                }
            }
            s_after[lane] = sa;
            s_grad[lane] = sg;
            s_last[lane] = lc;
            __syncwarp();
        }
        if (i > 0) {
            last = __shfl_up_sync(0xffffffffu, last, 1);
            afr = __shfl_up_sync(0xffffffffu, afr, 1);
            afg = __shfl_up_sync(0xffffffffu, afg, 1);
            afb = __shfl_up_sync(0xffffffffu, afb, 1);
            tr = __shfl_up_sync(0xffffffffu, tr, 1);
            pgr = __shfl_up_sync(0xffffffffu, pgr, 1);
            pgg = __shfl_up_sync(0xffffffffu, pgg, 1);
            pgb = __shfl_up_sync(0xffffffffu, pgb, 1);
            gac = __shfl_up_sync(0xffffffffu, gac, 1);
        }
        const int pix = i - static_cast<int>(lane);
        if (lane == 0 && pix < kTilePixels) {
            const int slot = i & 31;
            last = s_last[slot];
            const float4 sa = s_after[slot], sg = s_grad[slot];
            afr = sa.x; afg = sa.y; afb = sa.z; tr = sa.w;
            pgr = sg.x; pgg = sg.y; pgb = sg.z; gac = sg.w;
        }
        if ((i & 31) == 31) __syncwarp();  // the chunk in shared memory is replaced at the next multiple of 32
        if (!valid || pix < 0 || pix >= kTilePixels || k >= last) continue;
        const uint32_t lx = static_cast<uint32_t>(pix) % kTileW, ly = static_cast<uint32_t>(pix) / kTileW;
        if (!((submask >> ((ly / kSubtileH) * 2 + lx / kSubtileW)) & 1u)) continue;
        const float dx = mx - (static_cast<float>(px0 + lx) + 0.5f), dy = my - (static_cast<float>(py0 + ly) + 0.5f);
        const float e = gauss_exponent(dx, dy, h);
        if (e < negthr) continue;
        const float G = det_exp_blend(fminf(e, 0.0f));
        const float alpha = o * G;
        const float w = tr * alpha;
        gr += w * pgr; gg += w * pgg; gbb += w * pgb;
        afr -= w * colr; afg -= w * colg; afb -= w * colb;
        const float oma = 1.0f - alpha;
        const float rcp = 1.0f / fmaxf(oma, kOneMinusAlphaEps);
        const float dl_da = (tr * colr - afr * rcp) * pgr + (tr * colg - afg * rcp) * pgg + (tr * colb - afb * rcp) * pgb + gac * rcp;
        gop += G * dl_da;
        const float hlp = -alpha * dl_da;
        gca += 0.5f * hlp * (dx * dx);
        gcb += 0.5f * hlp * (dx * dy);
        gcc += 0.5f * hlp * (dy * dy);
        const float dmx = hlp * (ca * dx + cb * dy), dmy = hlp * (cb * dx + cc * dy);
        gmx += dmx; gmy += dmy;
        ax += fabsf(dmx); ay += fabsf(dmy);
        tr = tr * oma;
    }
    if (valid) {
        const float go = proper_aa ? gop : (o - o * o) * gop;
        atomicAdd(&grads[r].g0, make_float4(gmx, gmy, gca, gcb));
        atomicAdd(&grads[r].g1, make_float4(gcc, gr, gg, gbb));
        atomicAdd(&grads[r].g2, make_float4(go, abs_grad ? ax : 0.0f, abs_grad ? ay : 0.0f, 0.0f));
    }
}

cudaError_t launch_blend_train(const BlendArgs& a, float* image, const TileBuffers& T, uint32_t* bucket_tile, float4* ckpt, cudaStream_t s) {
    const dim3 grid(a.grid_w, a.grid_h);
    blend_kernel<true><<<grid, kTilePixels, 0, s>>>(a, image, T, bucket_tile, ckpt, 1, 0);
    return cudaGetLastError();
}

cudaError_t launch_blend_inference(const BlendArgs& a, float* image, int chw, int clamp, cudaStream_t s) {
    const dim3 grid(a.grid_w, a.grid_h);
    TileBuffers none{};
    blend_kernel<false><<<grid, kTilePixels, 0, s>>>(a, image, none, nullptr, nullptr, chw, clamp);
    return cudaGetLastError();
}

cudaError_t launch_blend_backward(const BlendArgs& a, const float* image, const float* grad_image, const TileBuffers& T,
                                  const uint32_t* bucket_tile, const float4* ckpt, uint32_t n_buckets_max, GradRecord* grads, int proper_aa,
                                  int abs_grad, cudaStream_t s) {
    if (n_buckets_max == 0) return cudaSuccess;
    blend_backward_kernel<<<n_buckets_max, 32, 0, s>>>(a, image, grad_image, T, bucket_tile, ckpt, grads,
                                                        static_cast<uint32_t>(a.grid_w * a.grid_h), proper_aa, abs_grad);
    return cudaGetLastError();
}

}  // namespace fgs
