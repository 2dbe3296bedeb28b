// Output stage shared by all forward preprocess kernels: writes the per-primitive record, the depth key
// and the chunk statistics used by the order-preserving compaction of visible primitives.
#pragma once

#include "preprocess.cuh"

namespace fgs {

__device__ inline float bits_of_bounds(uint32_t lo, uint32_t hi) { return __uint_as_float(lo | (hi << 16)); }

// Stores primitive `idx` of chunk `chunk`; must be reached by every thread of the CTA (kChunk threads).
__device__ inline void store_primitive(const PrimBuffers& B, uint32_t idx, bool in_range, const Geometry& G, f3 color, uint32_t chunk) {
    const bool visible = in_range && G.n_touched > 0;
    if (in_range) {
        B.n_touched[idx] = G.n_touched;
        B.rank_of[idx] = kInvalidRank;
        if (visible) {
            B.depth_key[idx] = __float_as_uint(G.depth);
            Record r;
            r.q0 = make_float4(G.mx, G.my, G.opacity, G.power_thr);
            r.q1 = make_float4(G.ca, G.cb, G.cc, bits_of_bounds(G.xmin, G.xmax));
            r.q2 = make_float4(color.x, color.y, color.z, bits_of_bounds(G.ymin, G.ymax));
            B.rec[idx] = r;
        }
    }
    // chunk statistics: visible count and instance sum
    __shared__ uint32_t warp_inst[kChunk / 32];
    uint32_t inst = visible ? G.n_touched : 0u;
    for (int o = 16; o > 0; o >>= 1) inst += __shfl_down_sync(0xffffffffu, inst, o);
    const int nvis = __syncthreads_count(visible);
    if ((threadIdx.x & 31) == 0) warp_inst[threadIdx.x >> 5] = inst;
    __syncthreads();
    if (threadIdx.x == 0) {
        uint32_t s = 0;
        for (int w = 0; w < kChunk / 32; w++) s += warp_inst[w];
        B.chunk_stats[chunk] = make_uint2(static_cast<uint32_t>(nvis), s);
    }
}

}  // namespace fgs
