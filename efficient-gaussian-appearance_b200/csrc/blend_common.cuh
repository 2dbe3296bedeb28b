// Pieces shared by the forward blend (blend.cu) and the backward blend (blend_bwd.cu): staged record layouts,
// the subtile bounds test, the Gaussian exponent at a pixel, and the warp reductions of the backward.
#pragma once

#include "launch.h"

namespace fgs {

// -0.5 log2(e) and -log2(e): folded into the conic so that a fragment's Gaussian is one exp2 of the exponent
// (rasterization/include/kernels_common.cuh:13-17)
constexpr float kLog2eBlend = 1.44269504089f;
constexpr float kHalfConic = -0.5f * kLog2eBlend;
constexpr float kCrossConic = -kLog2eBlend;

struct Staged {
    float4 a;   // mean2d.x, mean2d.y, unused, opacity
    float4 h;   // conic scaled for exp2: kHalfConic conic.x, kCrossConic conic.y, kHalfConic conic.z, unused
    float4 c;   // color rgb, unused
    uint2 bnd;  // bounds x (lo | hi << 16), y (lo | hi << 16)
};

__device__ inline void stage_record(const Record& q, Staged& s) {
    s.a = make_float4(q.q0.x, q.q0.y, 0.0f, q.q0.z);
    s.h = make_float4(kHalfConic * q.q1.x, kCrossConic * q.q1.y, kHalfConic * q.q1.z, 0.0f);
    s.c = make_float4(q.q2.x, q.q2.y, q.q2.z, 0.0f);
    s.bnd = make_uint2(__float_as_uint(q.q1.w), __float_as_uint(q.q2.w));
}

__device__ inline bool overlaps_subtile(uint2 bnd, uint32_t sx0, uint32_t sy0) {
    const uint32_t xlo = bnd.x & 0xffffu, xhi = bnd.x >> 16, ylo = bnd.y & 0xffffu, yhi = bnd.y >> 16;
    return xlo < sx0 + kSubtileW && sx0 < xhi && ylo < sy0 + kSubtileH && sy0 < yhi;
}

// base-2 exponent of the Gaussian at the pixel, dx (h.x dx + h.y dy) + h.z dy dy with the scaled conic h
// (kernels_forward.cuh:119-121), in the single-rounding operations the reference's contracting build evaluates it
// with inside its blend (measured against the reference kernels' transmittance), spelled out so that the forward and
// the backward blend take identical decisions
__device__ inline float gauss_exponent(float dx, float dy, float4 h) {
    return fmaf(__fmul_rn(h.z, dy), dy, __fmul_rn(dx, fmaf(h.x, dx, __fmul_rn(h.y, dy))));
}

// the Gaussian of a fragment from its base-2 exponent; alpha = opacity * Gaussian (one rounding), and the reference
// skips the fragment when alpha is below 1/255 (kernels_forward.cuh:122-127, original opacity interpretation)
__device__ inline float fragment_gaussian(float e) { return exp2f(fminf(e, 0.0f)); }



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
    float4 a;   // mean2d.x, mean2d.y, unused, opacity
    float4 h;   // conic scaled for exp2 (as Staged), bits(rank)
    float4 c;   // color rgb, unused
    uint2 bnd;
};

}  // namespace fgs
