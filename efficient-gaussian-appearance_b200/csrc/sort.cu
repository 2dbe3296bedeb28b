// Stable key/value radix sorts and the exclusive scan of the binning stage, written for this library.
// Depth sort: 32-bit depth keys of the visible primitives with their primitive indices
// (FasterGSVDACudaBackend/.../rasterization/src/forward.cu:88-97); tile sort: 16- or 32-bit tile keys over
// [0, end_bit) with the depth ranks (forward.cu:182-191, key width rule forward.cu:139-140). Both sorts are stable,
// so tile lists keep depth order and equal depth keys keep primitive order.
//
// Least-significant-digit radix sort, at most 8 bits per pass (the key bits are split into equal passes). Each pass:
//  1. upsweep: every CTA counts the digits of its 4096-key tile (shared-memory histogram) -> hist[digit][tile];
//  2. row scan: one CTA per digit turns its row into exclusive offsets across tiles and records the digit total;
//  3. downsweep: every CTA ranks its tile stably (8 warps own consecutive 512-key chunks; within a warp, one ballot
//     per digit bit finds the lanes with the same digit, their order gives the rank, and per-warp running counts
//     carry across the 16 rounds), stages keys and values in shared memory in digit order and writes each digit's
//     run contiguously to its global offset (digit base from the scanned totals + the tile's row offset).
// Positions are 32-bit: a sort takes fewer than 2^32 - 4096 keys.
// Traffic per pass: keys read twice, keys and values read and written once.
#include "launch.h"

namespace fgs {

namespace {

constexpr int kSortThreads = 256;
constexpr int kSortWarps = kSortThreads / 32;
constexpr int kSortItems = 16;                          // keys per thread
constexpr int kSortTile = kSortThreads * kSortItems;    // 4096 keys per tile
constexpr int kRadix = 256;

uint32_t n_tiles_of(uint64_t n) { return static_cast<uint32_t>((n + kSortTile - 1) / kSortTile); }

// exclusive scan of one value per thread over a 256-thread block; returns the block total in *total
__device__ inline uint32_t block_exclusive_scan(uint32_t x, uint32_t* warp_tot, uint32_t* total) {
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    uint32_t incl = x;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
        const uint32_t y = __shfl_up_sync(0xffffffffu, incl, o);
        if (lane >= o) incl += y;
    }
    if (lane == 31) warp_tot[warp] = incl;
    __syncthreads();
    if (warp == 0) {
        uint32_t w = lane < kSortWarps ? warp_tot[lane] : 0u;
#pragma unroll
        for (int o = 1; o < 32; o <<= 1) {
            const uint32_t y = __shfl_up_sync(0xffffffffu, w, o);
            if (lane >= o) w += y;
        }
        if (lane < kSortWarps) warp_tot[lane] = w;  // inclusive
    }
    __syncthreads();
    const uint32_t before = warp > 0 ? warp_tot[warp - 1] : 0u;
    if (total) *total = warp_tot[kSortWarps - 1];
    const uint32_t r = before + incl - x;
    __syncthreads();
    return r;
}

template <typename K>
__global__ void __launch_bounds__(kSortThreads) radix_upsweep(const K* __restrict__ keys, uint32_t n, int shift, uint32_t mask,
                                                              uint32_t* __restrict__ hist, uint32_t n_tiles) {
    __shared__ uint32_t cnt[kRadix];
    cnt[threadIdx.x] = 0;
    const uint32_t base = blockIdx.x * kSortTile + threadIdx.x;
    // all loads first (the shared atomics below would otherwise keep each load waiting behind the previous one)
    uint32_t d[kSortItems];
#pragma unroll
    for (int j = 0; j < kSortItems; j++) {
        const uint32_t i = base + j * kSortThreads;
        d[j] = i < n ? (static_cast<uint32_t>(keys[i]) >> shift) & mask : kRadix;
    }
    __syncthreads();
#pragma unroll
    for (int j = 0; j < kSortItems; j++)
        if (d[j] < kRadix) atomicAdd(&cnt[d[j]], 1u);
    __syncthreads();
    hist[threadIdx.x * n_tiles + blockIdx.x] = cnt[threadIdx.x];
}

// row d of hist: exclusive offsets over the tiles; totals[d] = the row sum
__global__ void __launch_bounds__(kSortThreads) radix_row_scan(uint32_t* __restrict__ hist, uint32_t n_tiles, uint32_t* __restrict__ totals) {
    __shared__ uint32_t warp_tot[kSortWarps];
    uint32_t* row = hist + static_cast<uint64_t>(blockIdx.x) * n_tiles;
    uint32_t carry = 0;
    for (uint32_t c0 = 0; c0 < n_tiles; c0 += kSortThreads) {
        const uint32_t c = c0 + threadIdx.x;
        const uint32_t x = c < n_tiles ? row[c] : 0u;
        uint32_t tot = 0;
        const uint32_t ex = block_exclusive_scan(x, warp_tot, &tot);
        if (c < n_tiles) row[c] = carry + ex;
        carry += tot;
    }
    if (threadIdx.x == 0) totals[blockIdx.x] = carry;
}

// lanes of the warp whose (valid) digit equals this lane's, from one ballot per digit bit (fixed cost, unlike a
// match instruction whose cost grows with the number of distinct values)
__device__ inline uint32_t digit_peers(uint32_t d, int bits, bool valid) {
    uint32_t m = __ballot_sync(0xffffffffu, valid);
#pragma unroll
    for (int b = 0; b < 8; b++) {
        if (b >= bits) break;
        const bool set = (d >> b) & 1u;
        const uint32_t bb = __ballot_sync(0xffffffffu, set);
        m &= set ? bb : ~bb;
    }
    return m;
}

template <typename K>
__global__ void __launch_bounds__(kSortThreads, 3) radix_downsweep(const K* __restrict__ kin, K* __restrict__ kout, const uint32_t* __restrict__ vin,
                                                                uint32_t* __restrict__ vout, uint32_t n, int shift, int bits, uint32_t mask,
                                                                const uint32_t* __restrict__ hist, const uint32_t* __restrict__ totals,
                                                                uint32_t n_tiles) {
    __shared__ uint32_t run[kSortWarps][kRadix];  // per-warp digit counts (then exclusive offsets within the tile)
    __shared__ uint32_t tile_off[kRadix];         // first tile-local position of each digit
    __shared__ uint32_t glob_off[kRadix];         // first global position of each digit for this tile
    __shared__ uint32_t warp_tot[kSortWarps];
    __shared__ K skey[kSortTile];
    __shared__ uint32_t sval[kSortTile];
    const int t = threadIdx.x, lane = t & 31, warp = t >> 5;
#pragma unroll
    for (int w = 0; w < kSortWarps; w++) run[w][t] = 0;
    // global base of every digit: exclusive scan of the digit totals, plus this tile's row offset
    {
        const uint32_t base = block_exclusive_scan(totals[t], warp_tot, nullptr);
        glob_off[t] = base + hist[t * n_tiles + blockIdx.x];
    }
    __syncthreads();
    // warp chunk: keys [tile + warp * 512, + 512), 16 rounds of 32 consecutive keys
    const uint32_t chunk = blockIdx.x * kSortTile + warp * (kSortItems * 32);
    const uint32_t left = n > chunk ? n - chunk : 0u;  // keys of this warp's chunk that exist
    const K* kc = kin + chunk;
    const uint32_t* vc = vin + chunk;
    K key[kSortItems];
    uint32_t val[kSortItems], rank[kSortItems];
    uint32_t valid_bits = 0;
    const uint32_t lt = (1u << lane) - 1u;
    // all loads first: the ranking rounds below are serialised through the shared counters and must not wait on
    // one global load each
#pragma unroll
    for (int j = 0; j < kSortItems; j++) {
        const uint32_t i = j * 32 + lane;
        const bool valid = i < left;
        key[j] = valid ? kc[i] : K(0);
        valid_bits |= valid ? (1u << j) : 0u;
    }
#pragma unroll
    for (int j = 0; j < kSortItems; j++) {
        const bool valid = (valid_bits >> j) & 1u;
        const uint32_t d = valid ? (static_cast<uint32_t>(key[j]) >> shift) & mask : kRadix;  // kRadix: no digit
        const uint32_t peers = digit_peers(d, bits, valid);
        const uint32_t prior = d < kRadix ? run[warp][d] : 0u;
        rank[j] = prior + __popc(peers & lt);
        __syncwarp();
        if (d < kRadix && (peers & lt) == 0) run[warp][d] = prior + __popc(peers);
        __syncwarp();
    }
    // values are only needed for the scatter: their loads overlap the offset scan
#pragma unroll
    for (int j = 0; j < kSortItems; j++) val[j] = (valid_bits >> j) & 1u ? vc[j * 32 + lane] : 0u;
    __syncthreads();
    // tile-local offsets: digit-major, warps in order within a digit (the chunks are consecutive in the input)
    {
        uint32_t cnt = 0;
#pragma unroll
        for (int w = 0; w < kSortWarps; w++) {
            const uint32_t c = run[w][t];
            run[w][t] = cnt;
            cnt += c;
        }
        tile_off[t] = block_exclusive_scan(cnt, warp_tot, nullptr);
    }
    __syncthreads();
#pragma unroll
    for (int j = 0; j < kSortItems; j++) {
        if (!((valid_bits >> j) & 1u)) continue;
        const uint32_t d = (static_cast<uint32_t>(key[j]) >> shift) & mask;
        const uint32_t p = tile_off[d] + run[warp][d] + rank[j];
        skey[p] = key[j];
        sval[p] = val[j];
    }
    __syncthreads();
    // write out in tile-local order: consecutive positions of a digit go to consecutive global positions
    const uint32_t tile_base = blockIdx.x * kSortTile;
    const uint32_t count = n - tile_base < static_cast<uint32_t>(kSortTile) ? n - tile_base : kSortTile;
    for (uint32_t p = t; p < count; p += kSortThreads) {
        const K k = skey[p];
        const uint32_t d = (static_cast<uint32_t>(k) >> shift) & mask;
        const uint32_t g = glob_off[d] + (p - tile_off[d]);
        kout[g] = k;
        vout[g] = sval[p];
    }
}

struct SortTemp {
    uint32_t* hist;    // [kRadix][n_tiles]
    uint32_t* totals;  // [kRadix]
};

SortTemp carve_sort_temp(void* temp, uint64_t n) {
    SortTemp T;
    T.hist = static_cast<uint32_t*>(temp);
    T.totals = T.hist + static_cast<uint64_t>(kRadix) * n_tiles_of(n);
    return T;
}

size_t sort_temp_bytes(uint64_t n) { return (static_cast<uint64_t>(kRadix) * n_tiles_of(n) + kRadix) * sizeof(uint32_t); }

// sorts bits [0, end_bit) of the keys; the result ends in (ka, va) or (kb, vb), reported through *kout / *vout
template <typename K>
cudaError_t radix_sort_pairs(K* ka, K* kb, uint32_t* va, uint32_t* vb, uint64_t n, int end_bit, void* temp, size_t temp_bytes, K** kout,
                             uint32_t** vout, cudaStream_t s) {
    *kout = ka;
    *vout = va;
    if (n == 0 || end_bit <= 0) return cudaSuccess;
    if (temp_bytes < sort_temp_bytes(n)) return cudaErrorInvalidValue;
    if (n > 0xFFFFFFFFull - kSortTile) return cudaErrorInvalidValue;  // positions are 32-bit
    const SortTemp T = carve_sort_temp(temp, n);
    const uint32_t tiles = n_tiles_of(n);
    const int passes = (end_bit + 7) / 8;
    const int bits = (end_bit + passes - 1) / passes;
    const uint32_t mask = (1u << bits) - 1u;
    K* kin = ka;
    K* kx = kb;
    uint32_t* vin = va;
    uint32_t* vx = vb;
    for (int p = 0; p < passes; p++) {
        const int shift = p * bits;
        radix_upsweep<K><<<tiles, kSortThreads, 0, s>>>(kin, static_cast<uint32_t>(n), shift, mask, T.hist, tiles);
        radix_row_scan<<<kRadix, kSortThreads, 0, s>>>(T.hist, tiles, T.totals);
        radix_downsweep<K><<<tiles, kSortThreads, 0, s>>>(kin, kx, vin, vx, static_cast<uint32_t>(n), shift, bits, mask, T.hist, T.totals, tiles);
        cudaError_t e = cudaGetLastError();
        if (e != cudaSuccess) return e;
        K* tk = kin; kin = kx; kx = tk;
        uint32_t* tv = vin; vin = vx; vx = tv;
    }
    *kout = kin;
    *vout = vin;
    return cudaSuccess;
}

// ---------------------------------------------------------------------------------------------------
// exclusive scan (in place): per-tile sums, a scan of the tile sums, per-tile scans with the tile's offset

__global__ void __launch_bounds__(kSortThreads) scan_tile_sums(const uint32_t* __restrict__ data, uint32_t n, uint32_t* __restrict__ sums) {
    __shared__ uint32_t warp_tot[kSortWarps];
    const uint64_t base = static_cast<uint64_t>(blockIdx.x) * kSortTile;
    uint32_t x = 0;
#pragma unroll 4
    for (int j = 0; j < kSortItems; j++) {
        const uint64_t i = base + static_cast<uint64_t>(j) * kSortThreads + threadIdx.x;
        if (i < n) x += data[i];
    }
    uint32_t tot = 0;
    block_exclusive_scan(x, warp_tot, &tot);
    if (threadIdx.x == 0) sums[blockIdx.x] = tot;
}

__global__ void __launch_bounds__(kSortThreads) scan_sums(uint32_t* __restrict__ sums, uint32_t n_tiles) {
    __shared__ uint32_t warp_tot[kSortWarps];
    uint32_t carry = 0;
    for (uint32_t c0 = 0; c0 < n_tiles; c0 += kSortThreads) {
        const uint32_t c = c0 + threadIdx.x;
        const uint32_t x = c < n_tiles ? sums[c] : 0u;
        uint32_t tot = 0;
        const uint32_t ex = block_exclusive_scan(x, warp_tot, &tot);
        if (c < n_tiles) sums[c] = carry + ex;
        carry += tot;
    }
}

// each thread scans 16 consecutive values of the tile; the thread offsets come from a block scan of their sums
__global__ void __launch_bounds__(kSortThreads) scan_tiles(uint32_t* __restrict__ data, uint32_t n, const uint32_t* __restrict__ sums) {
    __shared__ uint32_t warp_tot[kSortWarps];
    const uint64_t first = static_cast<uint64_t>(blockIdx.x) * kSortTile + static_cast<uint64_t>(threadIdx.x) * kSortItems;
    uint32_t v[kSortItems];
    uint32_t s = 0;
#pragma unroll
    for (int j = 0; j < kSortItems; j++) {
        const uint64_t i = first + j;
        v[j] = i < n ? data[i] : 0u;
        s += v[j];
    }
    uint32_t run = sums[blockIdx.x] + block_exclusive_scan(s, warp_tot, nullptr);
#pragma unroll
    for (int j = 0; j < kSortItems; j++) {
        const uint64_t i = first + j;
        if (i < n) data[i] = run;
        run += v[j];
    }
}

}  // namespace

size_t depth_sort_temp_bytes(uint32_t n) { return sort_temp_bytes(n); }

cudaError_t depth_sort(PrimBuffers& B, uint32_t n_visible, cudaStream_t s) {
    uint32_t* kout = nullptr;
    uint32_t* vout = nullptr;
    const cudaError_t e = radix_sort_pairs<uint32_t>(B.keys_a, B.keys_b, B.idx_a, B.idx_b, n_visible, 32, B.sort_temp, B.sort_temp_bytes, &kout, &vout, s);
    B.sorted_idx = vout;
    return e;
}

size_t exclusive_scan_temp_bytes(uint32_t n) { return (static_cast<size_t>(n_tiles_of(n)) + 1) * sizeof(uint32_t); }

cudaError_t exclusive_scan_u32(uint32_t* data, uint32_t n, void* temp, size_t temp_bytes, cudaStream_t s) {
    if (n == 0) return cudaSuccess;
    if (temp_bytes < exclusive_scan_temp_bytes(n)) return cudaErrorInvalidValue;
    const uint32_t tiles = n_tiles_of(n);
    uint32_t* sums = static_cast<uint32_t*>(temp);
    scan_tile_sums<<<tiles, kSortThreads, 0, s>>>(data, n, sums);
    scan_sums<<<1, kSortThreads, 0, s>>>(sums, tiles);
    scan_tiles<<<tiles, kSortThreads, 0, s>>>(data, n, sums);
    return cudaGetLastError();
}

size_t tile_sort_temp_bytes(uint64_t n, int end_bit, bool wide) {
    (void)end_bit;
    (void)wide;
    return sort_temp_bytes(n);
}

cudaError_t tile_sort(void* keys_a, void* keys_b, uint32_t* vals_a, uint32_t* vals_b, uint64_t n, int end_bit, bool wide, void* temp,
                      size_t temp_bytes, const void** keys_out, const uint32_t** vals_out, cudaStream_t s) {
    uint32_t* vout = nullptr;
    cudaError_t e;
    if (wide) {
        uint32_t* kout = nullptr;
        e = radix_sort_pairs<uint32_t>(static_cast<uint32_t*>(keys_a), static_cast<uint32_t*>(keys_b), vals_a, vals_b, n, end_bit, temp, temp_bytes,
                                       &kout, &vout, s);
        *keys_out = kout;
    } else {
        uint16_t* kout = nullptr;
        e = radix_sort_pairs<uint16_t>(static_cast<uint16_t*>(keys_a), static_cast<uint16_t*>(keys_b), vals_a, vals_b, n, end_bit, temp, temp_bytes,
                                       &kout, &vout, s);
        *keys_out = kout;
    }
    *vals_out = vout;
    return e;
}

}  // namespace fgs
