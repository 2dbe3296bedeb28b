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
#include "preprocess_bwd.cuh"
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
    // kNeural: the residual comes from the colour pass over the visible primitives, which overwrites this colour
    const f3 base = base_act3(A.base_act, ld3(P.base, i));
    f3 col = color_act3(A.color_act, base + res);
    if (!v.render_base) {
        const f3 bc = color_act3(A.color_act, base);
        col = mk3(fabsf(col.x - bc.x), fabsf(col.y - bc.y), fabsf(col.z - bc.z));
    }
    return col;
}

// The Neural preprocess (geometry only: the colour pass evaluates the appearance) is compiled for eight CTAs per SM
// (32 registers, a few bytes spilled; measured on the c4 step: 1.53 -> 1.46 ms per step against 47 registers and five
// CTAs); the other models keep their unconstrained allocation (a minimum of 0 CTAs per SM sets no bound).
template <int MODEL>
__global__ void __launch_bounds__(kChunk, MODEL == kNeural ? 8 : 0) preprocess_fwd_kernel(Params P, AppearanceConfig A, View v, PrimBuffers B) {
    const uint32_t i = blockIdx.x * kChunk + threadIdx.x;
    const bool in_range = i < P.n;
    const Geometry G = project_primitive(P.means, P.scales, P.rotations, P.opacities, in_range ? i : 0, in_range, v);
    f3 color = mk3(0.0f, 0.0f, 0.0f);
    if (in_range && G.n_touched > 0) color = fused_color<MODEL>(P, A, v, i, ld3(P.means, i));
    store_primitive(B, i, in_range, G, color, blockIdx.x);
}

// Compaction offsets in three parallel phases: per group of 1024 chunks the visible and instance sums; one CTA scans
// the group sums (and writes the totals); per group the exclusive scan of the chunks' visible counts.
constexpr int kScanGroup = 1024;

__device__ inline uint32_t block1024_exclusive_scan(uint32_t x, uint32_t* warp_sums, uint32_t* total) {
    const uint32_t lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    uint32_t incl = x;
    for (int o = 1; o < 32; o <<= 1) {
        const uint32_t y = __shfl_up_sync(0xffffffffu, incl, o);
        if (lane >= static_cast<uint32_t>(o)) incl += y;
    }
    if (lane == 31) warp_sums[warp] = incl;
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
    const uint32_t r = incl - x + (warp > 0 ? warp_sums[warp - 1] : 0u);
    if (total) *total = warp_sums[31];
    __syncthreads();
    return r;
}

__global__ void __launch_bounds__(kScanGroup) chunk_group_sums(const uint2* __restrict__ stats, uint32_t n_chunks, uint32_t* __restrict__ g_vis,
                                                              unsigned long long* __restrict__ g_inst) {
    __shared__ uint32_t warp_sums[32];
    __shared__ unsigned long long inst;
    if (threadIdx.x == 0) inst = 0;
    const uint32_t c = blockIdx.x * kScanGroup + threadIdx.x;
    const uint2 st = c < n_chunks ? stats[c] : make_uint2(0, 0);
    uint32_t tot = 0;
    block1024_exclusive_scan(st.x, warp_sums, &tot);
    unsigned long long y = st.y;
    for (int o = 16; o > 0; o >>= 1) y += __shfl_down_sync(0xffffffffu, y, o);
    if ((threadIdx.x & 31) == 0) atomicAdd(&inst, y);
    __syncthreads();
    if (threadIdx.x == 0) {
        g_vis[blockIdx.x] = tot;
        g_inst[blockIdx.x] = inst;
    }
}

__global__ void __launch_bounds__(kScanGroup) chunk_group_scan(uint32_t* __restrict__ g_vis, const unsigned long long* __restrict__ g_inst,
                                                              uint32_t n_groups, unsigned long long* __restrict__ counters) {
    __shared__ uint32_t warp_sums[32];
    __shared__ unsigned long long inst;
    if (threadIdx.x == 0) inst = 0;
    uint32_t carry = 0;
    unsigned long long my_inst = 0;
    for (uint32_t base = 0; base < n_groups; base += kScanGroup) {
        const uint32_t g = base + threadIdx.x;
        const uint32_t x = g < n_groups ? g_vis[g] : 0u;
        if (g < n_groups) my_inst += g_inst[g];
        uint32_t tot = 0;
        const uint32_t ex = block1024_exclusive_scan(x, warp_sums, &tot);
        if (g < n_groups) g_vis[g] = carry + ex;
        carry += tot;
    }
    atomicAdd(&inst, my_inst);
    __syncthreads();
    if (threadIdx.x == 0) {
        counters[0] = carry;
        counters[1] = inst;
    }
}

__global__ void __launch_bounds__(kScanGroup) chunk_offsets(const uint2* __restrict__ stats, uint32_t n_chunks, const uint32_t* __restrict__ g_vis,
                                                           uint32_t* __restrict__ off) {
    __shared__ uint32_t warp_sums[32];
    const uint32_t c = blockIdx.x * kScanGroup + threadIdx.x;
    const uint32_t x = c < n_chunks ? stats[c].x : 0u;
    const uint32_t ex = block1024_exclusive_scan(x, warp_sums, nullptr);
    if (c < n_chunks) off[c] = g_vis[blockIdx.x] + ex;
}

// writes (depth key, primitive index) of visible primitives in primitive order
__global__ void __launch_bounds__(kChunk) compact_kernel(const uint32_t* __restrict__ n_touched, const uint32_t* __restrict__ depth_key,
                                                         const uint32_t* __restrict__ chunk_off, uint32_t* __restrict__ keys,
                                                         uint32_t* __restrict__ idx, uint32_t* __restrict__ vis_idx, uint32_t n) {
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
        vis_idx[pos] = i;
    }
}

// gathers records into depth order, records the rank of every visible primitive, and the tile counts. A block takes
// 256 consecutive ranks; the records are copied as 16-byte thirds with three consecutive lanes on one record, so a
// warp instruction reads whole 48-byte records and the depth-ordered output is written contiguously.
constexpr int kReorderRanks = 256;
__global__ void __launch_bounds__(kReorderRanks) reorder_kernel(const uint32_t* __restrict__ sorted_idx, const Record* __restrict__ rec,
                                                                const uint32_t* __restrict__ n_touched, Record* __restrict__ sorted_rec,
                                                                uint32_t* __restrict__ counts, uint32_t* __restrict__ rank_of, uint32_t n_visible) {
    __shared__ uint32_t prim[kReorderRanks];
    const uint32_t r0 = blockIdx.x * kReorderRanks, t = threadIdx.x;
    const uint32_t m = min(static_cast<uint32_t>(kReorderRanks), n_visible - r0);
    if (t < m) {
        const uint32_t i = sorted_idx[r0 + t];
        prim[t] = i;
        counts[r0 + t] = n_touched[i];
        rank_of[i] = r0 + t;
    }
    __syncthreads();
    const float4* src = reinterpret_cast<const float4*>(rec);
    float4* dst = reinterpret_cast<float4*>(sorted_rec + r0);
    for (uint32_t c = t; c < 3 * m; c += kReorderRanks) {
        const uint32_t k = c / 3, part = c - 3 * k;
        dst[c] = src[3ull * prim[k] + part];
    }
}

// ----------------------------------------------------------------------------------------------------
// backward preprocess



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
        case kNeural: preprocess_fwd_kernel<kNeural><<<grid, kChunk, 0, s>>>(P, A, v, B); break;
        default: return cudaErrorInvalidValue;
    }
    return cudaGetLastError();
}

cudaError_t launch_compaction(const PrimBuffers& B, uint32_t n, cudaStream_t s) {
    const int chunks = grid_of(n, kChunk);
    if (chunks == 0) return cudaMemsetAsync(B.counters, 0, 2 * sizeof(unsigned long long), s);
    const int groups = (chunks + kScanGroup - 1) / kScanGroup;
    chunk_group_sums<<<groups, kScanGroup, 0, s>>>(B.chunk_stats, chunks, B.group_vis, B.group_inst);
    chunk_group_scan<<<1, kScanGroup, 0, s>>>(B.group_vis, B.group_inst, groups, B.counters);
    chunk_offsets<<<groups, kScanGroup, 0, s>>>(B.chunk_stats, chunks, B.group_vis, B.chunk_off);
    compact_kernel<<<chunks, kChunk, 0, s>>>(B.n_touched, B.depth_key, B.chunk_off, B.keys_a, B.idx_a, B.vis_idx, n);
    return cudaGetLastError();
}

cudaError_t launch_reorder(const PrimBuffers& B, uint32_t n_visible, cudaStream_t s) {
    if (n_visible == 0) return cudaSuccess;
    reorder_kernel<<<grid_of(n_visible, kReorderRanks), kReorderRanks, 0, s>>>(B.sorted_idx, B.rec, B.n_touched, B.sorted_rec, B.inst_off,
                                                                              B.rank_of, n_visible);
    return cudaGetLastError();
}

cudaError_t launch_preprocess_bwd(const Params& P, const AppearanceConfig& A, const View& v, const uint32_t* rank_of,
                                  const Record* sorted_rec, const GradRecord* grads, const GradOut& O, bool precomputed,
                                  const uint32_t* vis_idx, uint32_t n_visible, cudaStream_t s) {
    const int grid = grid_of(P.n, 128);
    if (grid == 0) return cudaSuccess;
    const int model = precomputed ? kPrecomputed : A.model;
    switch (model) {
        case kPrecomputed: preprocess_bwd_kernel<kPrecomputed><<<grid, 128, 0, s>>>(P, A, v, rank_of, sorted_rec, grads, O); break;
        case kSH: preprocess_bwd_kernel<kSH><<<grid, 128, 0, s>>>(P, A, v, rank_of, sorted_rec, grads, O); break;
        case kSV: preprocess_bwd_kernel<kSV><<<grid, 128, 0, s>>>(P, A, v, rank_of, sorted_rec, grads, O); break;
        case kNASG: preprocess_bwd_kernel<kNASG><<<grid, 128, 0, s>>>(P, A, v, rank_of, sorted_rec, grads, O); break;
        case kNASGabor: preprocess_bwd_kernel<kNASGabor><<<grid, 128, 0, s>>>(P, A, v, rank_of, sorted_rec, grads, O); break;
        case kNeural: return launch_preprocess_bwd_neural(P, A, v, rank_of, sorted_rec, grads, O, vis_idx, n_visible, s);
        default: return cudaErrorInvalidValue;
    }
    return cudaGetLastError();
}

}  // namespace fgs
