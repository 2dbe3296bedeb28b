// Instance emission (one (tile, depth rank) pair per touched tile, in depth order and, within a
// primitive, in row-major tile order), per-tile instance ranges and per-tile bucket offsets.
// Follows FasterGSVDACudaBackend/.../rasterization/include/kernels_common.cuh:33-157 and
// include/kernels_forward.cuh:14-24 with src/forward.cu:204-221.
#include "launch.h"

namespace fgs {

template <typename K>
__global__ void __launch_bounds__(256) emit_kernel(const Record* __restrict__ rec, const uint32_t* __restrict__ inst_off,
                                                   K* __restrict__ keys, uint32_t* __restrict__ vals, uint32_t n_visible,
                                                   uint32_t grid_w) {
    const uint32_t r = blockIdx.x * blockDim.x + threadIdx.x;
    const uint32_t lane = threadIdx.x & 31;
    const bool active = r < n_visible;
    if (__ballot_sync(0xffffffffu, active) == 0) return;
    float sx = 0.0f, sy = 0.0f, ca = 0.0f, cb = 0.0f, cc = 0.0f, thr = 0.0f;
    uint4 tb = make_uint4(0, 0, 0, 0);
    uint32_t n_max = 0, w = 0;
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
    }
    const uint32_t bw = tb.y - tb.x;
    if (active && n_max <= kSequentialTiles) {
        for (uint32_t t = 0; t < n_max; t++) {
            const uint32_t tx = tb.x + t % bw, ty = tb.z + t / bw;
            if (tile_overlaps(sx, sy, ca, cb, cc, tx, ty, thr)) {
                keys[w] = static_cast<K>(ty * grid_w + tx);
                vals[w] = r;
                w++;
            }
        }
    }
    uint32_t big = __ballot_sync(0xffffffffu, active && n_max > kSequentialTiles);
    while (big) {
        const uint32_t src = __ffs(big) - 1;
        big &= big - 1;
        const float qx = __shfl_sync(0xffffffffu, sx, src), qy = __shfl_sync(0xffffffffu, sy, src);
        const float qa = __shfl_sync(0xffffffffu, ca, src), qb = __shfl_sync(0xffffffffu, cb, src);
        const float qc = __shfl_sync(0xffffffffu, cc, src), qt = __shfl_sync(0xffffffffu, thr, src);
        const uint32_t qx0 = __shfl_sync(0xffffffffu, tb.x, src), qy0 = __shfl_sync(0xffffffffu, tb.z, src);
        const uint32_t qw = __shfl_sync(0xffffffffu, bw, src), qn = __shfl_sync(0xffffffffu, n_max, src);
        const uint32_t qr = __shfl_sync(0xffffffffu, r, src);
        uint32_t pos = __shfl_sync(0xffffffffu, w, src);
        for (uint32_t base = 0; base < qn; base += 32) {
            const uint32_t t = base + lane;
            const uint32_t tx = qx0 + t % qw, ty = qy0 + t / qw;
            const bool hit = t < qn && tile_overlaps(qx, qy, qa, qb, qc, tx, ty, qt);
            const uint32_t ballot = __ballot_sync(0xffffffffu, hit);
            if (hit) {
                const uint32_t o = pos + __popc(ballot & ((1u << lane) - 1u));
                keys[o] = static_cast<K>(ty * grid_w + tx);
                vals[o] = qr;
            }
            pos += __popc(ballot);
        }
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

// buckets of 32 instances per tile, inclusive scan (one CTA)
__global__ void __launch_bounds__(1024) bucket_scan_kernel(const uint2* __restrict__ ranges, uint32_t* __restrict__ off, uint32_t n_tiles) {
    __shared__ uint32_t warp_sums[32];
    __shared__ uint32_t carry;
    if (threadIdx.x == 0) carry = 0;
    __syncthreads();
    const uint32_t lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    for (uint32_t base = 0; base < n_tiles; base += 1024) {
        const uint32_t t = base + threadIdx.x;
        uint32_t cnt = 0;
        if (t < n_tiles) {
            const uint2 rg = ranges[t];
            cnt = (rg.y - rg.x + 31) / 32;
        }
        uint32_t x = cnt;
        for (int o = 1; o < 32; o <<= 1) {
            const uint32_t y = __shfl_up_sync(0xffffffffu, x, o);
            if (lane >= static_cast<uint32_t>(o)) x += y;
        }
        if (lane == 31) warp_sums[warp] = x;
        __syncthreads();
        if (warp == 0) {
            uint32_t v = warp_sums[lane];
            for (int o = 1; o < 32; o <<= 1) {
                const uint32_t y = __shfl_up_sync(0xffffffffu, v, o);
                if (lane >= static_cast<uint32_t>(o)) v += y;
            }
            warp_sums[lane] = v;
        }
        __syncthreads();
        const uint32_t incl = x + (warp > 0 ? warp_sums[warp - 1] : 0u) + carry;
        if (t < n_tiles) off[t] = incl;
        __syncthreads();
        if (threadIdx.x == 1023) carry = incl;
        __syncthreads();
    }
}

cudaError_t launch_emit(const Record* sorted_rec, const uint32_t* inst_off, void* keys, uint32_t* vals, uint32_t n_visible, int grid_w,
                        bool wide, cudaStream_t s) {
    if (n_visible == 0) return cudaSuccess;
    const int grid = static_cast<int>((n_visible + 255) / 256);
    if (wide) emit_kernel<uint32_t><<<grid, 256, 0, s>>>(sorted_rec, inst_off, static_cast<uint32_t*>(keys), vals, n_visible, grid_w);
    else emit_kernel<uint16_t><<<grid, 256, 0, s>>>(sorted_rec, inst_off, static_cast<uint16_t*>(keys), vals, n_visible, grid_w);
    return cudaGetLastError();
}

cudaError_t launch_ranges(const void* keys, uint64_t n, bool wide, const TileBuffers& T, int n_tiles, cudaStream_t s) {
    cudaError_t e = cudaMemsetAsync(T.ranges, 0, sizeof(uint2) * n_tiles, s);
    if (e != cudaSuccess) return e;
    if (n > 0) {
        const unsigned grid = static_cast<unsigned>((n + 255) / 256);
        if (wide) ranges_kernel<uint32_t><<<grid, 256, 0, s>>>(static_cast<const uint32_t*>(keys), T.ranges, n);
        else ranges_kernel<uint16_t><<<grid, 256, 0, s>>>(static_cast<const uint16_t*>(keys), T.ranges, n);
    }
    bucket_scan_kernel<<<1, 1024, 0, s>>>(T.ranges, T.bucket_off, static_cast<uint32_t>(n_tiles));
    return cudaGetLastError();
}

}  // namespace fgs
