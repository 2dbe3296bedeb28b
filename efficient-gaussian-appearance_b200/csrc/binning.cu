// Instance emission (one (tile, depth rank) pair per touched tile, in depth order and, within a
// primitive, in row-major tile order), per-tile instance ranges and per-tile bucket offsets.
// Follows FasterGSVDACudaBackend/.../rasterization/include/kernels_common.cuh:33-157 and
// include/kernels_forward.cuh:14-24 with src/forward.cu:204-221.
#include "launch.h"

namespace fgs {

// One warp emits the instances of its 32 primitives together: their candidate tiles (the bounds rectangles,
// row-major) are laid end to end and every lane tests one candidate per round, so a warp spends
// ceil(sum of candidates / 32) rounds whatever the mix of footprint sizes. A hit of primitive L goes to
// inst_off[L] + (hits of L before it), which keeps depth order across primitives and row-major tile order within one;
// consecutive hits of one primitive are consecutive lanes and consecutive addresses. A primitive never writes past
// the instances its tile count reserved (inst_off of the next rank, or n_instances for the last): the count and the
// emission evaluate the same tile test on the same record values, and the bound keeps the buffers safe regardless.
template <typename K>
__global__ void __launch_bounds__(256) emit_kernel(const Record* __restrict__ rec, const uint32_t* __restrict__ inst_off,
                                                   K* __restrict__ keys, uint32_t* __restrict__ vals, uint32_t n_visible,
                                                   uint32_t grid_w, uint32_t n_instances) {
    const uint32_t r = blockIdx.x * blockDim.x + threadIdx.x;
    const uint32_t lane = threadIdx.x & 31;
    const bool active = r < n_visible;
    if (__ballot_sync(0xffffffffu, active) == 0) return;
    float sx = 0.0f, sy = 0.0f, ca = 0.0f, cb = 0.0f, cc = 0.0f, thr = 0.0f;
    uint4 tb = make_uint4(0, 0, 0, 0);
    uint32_t n_max = 0, w = 0, lim = 0;
    if (active) {
        const Record q = rec[r];
        sx = q.q0.x - 0.5f;
        sy = q.q0.y - 0.5f;
        thr = q.q0.w;
        ca = q.q1.x; cb = q.q1.y; cc = q.q1.z;
        const uint32_t bx = __float_as_uint(q.q1.w), by = __float_as_uint(q.q2.w);
        tb = tile_bounds_of(bx & 0xffffu, bx >> 16, by & 0xffffu, by >> 16);
        n_max = (tb.y - tb.x) * (tb.w - tb.z);
        w = inst_off[r];
        lim = r + 1 < n_visible ? inst_off[r + 1] : n_instances;
    }
    const uint32_t bw = tb.y - tb.x;
    // candidate ranges [excl, incl) of the lanes' primitives in the warp's flattened list
    uint32_t incl = n_max;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
        const uint32_t y = __shfl_up_sync(0xffffffffu, incl, o);
        if (lane >= static_cast<uint32_t>(o)) incl += y;
    }
    const uint32_t excl = incl - n_max;
    const uint32_t total = __shfl_sync(0xffffffffu, incl, 31);
    uint32_t emitted = 0;  // hits of this lane's primitive in earlier rounds
    for (uint32_t base = 0; base < total; base += 32) {
        const uint32_t c = base + lane;
        // owner: the lane whose range holds candidate c (the last lane with excl <= c; empty ranges are skipped
        // because a later lane with the same excl exists only when the earlier range is empty)
        uint32_t owner = 0;
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
        const uint32_t qpos = __shfl_sync(0xffffffffu, w, owner) + __shfl_sync(0xffffffffu, emitted, owner);
        const uint32_t qlim = __shfl_sync(0xffffffffu, lim, owner);
        const bool valid = c < total;  // then the owner has candidates and qw >= 1
        const uint2 qr = divmod_small(valid ? c - o_excl : 0u, valid ? qw : 1u);
        const uint32_t tx = qx0 + qr.y, ty = qy0 + qr.x;
        const bool hit = valid && tile_overlaps(qx, qy, qa, qb, qc, tx, ty, qt);
        const uint32_t hits = __ballot_sync(0xffffffffu, hit);
        // lanes of this round that belong to the owner: from the owner's first candidate in the round up to this lane
        const uint32_t first = o_excl > base ? o_excl - base : 0u;
        const uint32_t before = hits & ((1u << lane) - 1u) & ~((1u << first) - 1u);
        const uint32_t o = qpos + __popc(before);
        if (hit && o < qlim) {
            keys[o] = static_cast<K>(ty * grid_w + tx);
            vals[o] = (r & ~31u) + owner;  // the owner's depth rank
        }
        // this lane's primitive: its candidates in this round are lanes [excl - base, incl - base) clipped to the round
        const uint32_t lo = excl > base ? excl - base : 0u, hi = incl > base ? incl - base : 0u;
        if (lo < 32 && hi > lo) {
            const uint32_t top = hi >= 32 ? 0xffffffffu : ((1u << hi) - 1u);
            emitted += __popc(hits & top & ~((1u << lo) - 1u));
        }
    }
    // reserved slots left unwritten (only if the count had found more tiles than the emission) get the primitive's
    // first candidate tile, so no stale key or rank reaches the range extraction or the blend
    if (active)
        for (uint32_t o = w + emitted; o < lim; o++) {
            keys[o] = static_cast<K>(tb.z * grid_w + tb.x);
            vals[o] = r;
        }
}

template <typename K>
__global__ void ranges_kernel(const K* __restrict__ keys, uint2* __restrict__ ranges, uint64_t n) {
    const uint64_t j = static_cast<uint64_t>(blockIdx.x) * blockDim.x + threadIdx.x;
    if (j >= n) return;
    const uint32_t k = keys[j];
    if (j == 0 || static_cast<uint32_t>(keys[j - 1]) != k) ranges[k].x = static_cast<uint32_t>(j);
    if (j == n - 1 || static_cast<uint32_t>(keys[j + 1]) != k) ranges[k].y = static_cast<uint32_t>(j + 1);
}

// the same with 8 consecutive keys per thread read as 16-byte vectors (keys 16-byte aligned)
template <typename K>
__global__ void __launch_bounds__(256) ranges8_kernel(const K* __restrict__ keys, uint2* __restrict__ ranges, uint64_t n) {
    constexpr int kVec = 16 / sizeof(K);  // keys per 16-byte vector
    const uint64_t j0 = (static_cast<uint64_t>(blockIdx.x) * blockDim.x + threadIdx.x) * 8;
    if (j0 >= n) return;
    uint32_t k[8];
    if (j0 + 8 <= n) {
#pragma unroll
        for (int v = 0; v < 8 / kVec; v++) {
            const uint4 q = reinterpret_cast<const uint4*>(keys + j0)[v];
            const K* e = reinterpret_cast<const K*>(&q);
#pragma unroll
            for (int i = 0; i < kVec; i++) k[v * kVec + i] = e[i];
        }
    } else {
#pragma unroll
        for (int i = 0; i < 8; i++) k[i] = j0 + i < n ? static_cast<uint32_t>(keys[j0 + i]) : 0u;
    }
    uint32_t prev = j0 > 0 ? static_cast<uint32_t>(keys[j0 - 1]) : 0u;
    const uint32_t after = j0 + 8 < n ? static_cast<uint32_t>(keys[j0 + 8]) : 0u;
#pragma unroll
    for (int i = 0; i < 8; i++) {
        const uint64_t j = j0 + i;
        if (j >= n) break;
        const uint32_t cur = k[i];
        if (j == 0 || prev != cur) ranges[cur].x = static_cast<uint32_t>(j);
        const uint32_t next = i < 7 ? k[i + 1] : after;
        if (j == n - 1 || next != cur) ranges[cur].y = static_cast<uint32_t>(j + 1);
        prev = cur;
    }
}

// buckets of 32 instances per tile, inclusive scan (one CTA; a thread scans 8 consecutive tiles per round, so a
// 1080p grid takes one round)
__global__ void __launch_bounds__(1024) bucket_scan_kernel(const uint2* __restrict__ ranges, uint32_t* __restrict__ off, uint32_t n_tiles) {
    constexpr int kPer = 8;
    __shared__ uint32_t warp_sums[32];
    const uint32_t lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    uint32_t carry = 0;
    for (uint32_t base = 0; base < n_tiles; base += 1024 * kPer) {
        const uint32_t first = base + threadIdx.x * kPer;
        uint32_t cnt[kPer], sum = 0;
#pragma unroll
        for (int j = 0; j < kPer; j++) {
            cnt[j] = 0;
            if (first + j < n_tiles) {
                const uint2 rg = ranges[first + j];
                cnt[j] = (rg.y - rg.x + 31) / 32;
            }
            sum += cnt[j];
        }
        uint32_t x = sum;
#pragma unroll
        for (int o = 1; o < 32; o <<= 1) {
            const uint32_t y = __shfl_up_sync(0xffffffffu, x, o);
            if (lane >= static_cast<uint32_t>(o)) x += y;
        }
        if (lane == 31) warp_sums[warp] = x;
        __syncthreads();
        if (warp == 0) {
            uint32_t v = warp_sums[lane];
#pragma unroll
            for (int o = 1; o < 32; o <<= 1) {
                const uint32_t y = __shfl_up_sync(0xffffffffu, v, o);
                if (lane >= static_cast<uint32_t>(o)) v += y;
            }
            warp_sums[lane] = v;
        }
        __syncthreads();
        uint32_t run = carry + x - sum + (warp > 0 ? warp_sums[warp - 1] : 0u);
#pragma unroll
        for (int j = 0; j < kPer; j++) {
            run += cnt[j];
            if (first + j < n_tiles) off[first + j] = run;
        }
        carry += warp_sums[31];
        __syncthreads();
    }
}

cudaError_t launch_emit(const Record* sorted_rec, const uint32_t* inst_off, void* keys, uint32_t* vals, uint32_t n_visible, int grid_w,
                        bool wide, uint64_t n_instances, cudaStream_t s) {
    if (n_visible == 0) return cudaSuccess;
    const int grid = static_cast<int>((n_visible + 255) / 256);
    const uint32_t ni = static_cast<uint32_t>(n_instances);
    if (wide) emit_kernel<uint32_t><<<grid, 256, 0, s>>>(sorted_rec, inst_off, static_cast<uint32_t*>(keys), vals, n_visible, grid_w, ni);
    else emit_kernel<uint16_t><<<grid, 256, 0, s>>>(sorted_rec, inst_off, static_cast<uint16_t*>(keys), vals, n_visible, grid_w, ni);
    return cudaGetLastError();
}

cudaError_t launch_ranges(const void* keys, uint64_t n, bool wide, const TileBuffers& T, int n_tiles, cudaStream_t s) {
    cudaError_t e = cudaMemsetAsync(T.ranges, 0, sizeof(uint2) * n_tiles, s);
    if (e != cudaSuccess) return e;
    if (n > 0) {
        if ((reinterpret_cast<uintptr_t>(keys) & 15u) == 0) {
            const unsigned grid = static_cast<unsigned>((n + 8 * 256 - 1) / (8 * 256));
            if (wide) ranges8_kernel<uint32_t><<<grid, 256, 0, s>>>(static_cast<const uint32_t*>(keys), T.ranges, n);
            else ranges8_kernel<uint16_t><<<grid, 256, 0, s>>>(static_cast<const uint16_t*>(keys), T.ranges, n);
        } else {
            const unsigned grid = static_cast<unsigned>((n + 255) / 256);
            if (wide) ranges_kernel<uint32_t><<<grid, 256, 0, s>>>(static_cast<const uint32_t*>(keys), T.ranges, n);
            else ranges_kernel<uint16_t><<<grid, 256, 0, s>>>(static_cast<const uint16_t*>(keys), T.ranges, n);
        }
    }
    bucket_scan_kernel<<<1, 1024, 0, s>>>(T.ranges, T.bucket_off, static_cast<uint32_t>(n_tiles));
    return cudaGetLastError();
}

}  // namespace fgs
