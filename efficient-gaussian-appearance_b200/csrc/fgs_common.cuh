// Shared constants, small vector helpers and the deterministic functions used by the kernels of the rasterizer.
//
// Arithmetic contract. The translation units whose results decide integer outcomes (preprocess.cu, binning.cu,
// blend.cu, blend_bwd.cu: culling, screen bounds, tile overlap, fragment acceptance, early termination) are compiled
// with -use_fast_math, like the reference's own build, and write the expressions whose rounding matters as explicit
// single-rounding operations (__fmul_rn, __fadd_rn, fmaf) in the reference's order, so that the decisions, tile lists
// and transmittances equal the reference's kernels bit for bit. The Neural MLP units (neural.cu, neural_tc.cu) keep
// the compiler's default contraction and use the deterministic sine and cosine below, so their fp16 MLP inputs are
// reproducible by a C restatement. det_exp / det_sigmoid serve gradient terms of the backward preprocess only.
#pragma once

#include <cstdint>
#include <cuda_runtime.h>
#include <cuda_fp16.h>

namespace fgs {

// ---- rasterizer constants (FasterGSVDACudaBackend/.../rasterization/include/rasterization_config.h:10-60) ----
constexpr float kDilation = 0.3f;
constexpr float kDilationProperAA = 0.1f;
constexpr float kMinCov2dDeterminant = 1e-6f;
constexpr float kOneMinusAlphaEps = 1e-6f;
constexpr float kTransmittanceThreshold = 1e-4f;
constexpr float kMinAlphaRcp = 255.0f;
constexpr float kMinAlpha = 1.0f / 255.0f;
constexpr float kMlpLossScale = 128.0f;
constexpr int kTileW = 16;
constexpr int kTileH = 12;
constexpr int kTilePixels = kTileW * kTileH;  // 192
constexpr int kSubtileW = 8;
constexpr int kSubtileH = 4;
constexpr uint32_t kInvalidRank = 0xffffffffu;

enum Model : int { kPrecomputed = 0, kSH = 1, kSV = 2, kNASG = 3, kNASGabor = 4, kNeural = 5 };

// ---- small vector helpers ----
struct f3 { float x, y, z; };
__host__ __device__ inline f3 mk3(float x, float y, float z) { return f3{x, y, z}; }
__host__ __device__ inline f3 operator+(f3 a, f3 b) { return mk3(a.x + b.x, a.y + b.y, a.z + b.z); }
__host__ __device__ inline f3 operator-(f3 a, f3 b) { return mk3(a.x - b.x, a.y - b.y, a.z - b.z); }
__host__ __device__ inline f3 operator*(float s, f3 a) { return mk3(s * a.x, s * a.y, s * a.z); }
__host__ __device__ inline f3 operator*(f3 a, float s) { return mk3(a.x * s, a.y * s, a.z * s); }
__host__ __device__ inline f3 operator*(f3 a, f3 b) { return mk3(a.x * b.x, a.y * b.y, a.z * b.z); }
__host__ __device__ inline float dot3(f3 a, f3 b) { return a.x * b.x + a.y * b.y + a.z * b.z; }
__device__ inline f3 ld3(const float* p, uint32_t i) { return mk3(p[3 * i], p[3 * i + 1], p[3 * i + 2]); }
__device__ inline void st3(float* p, uint32_t i, f3 v) { p[3 * i] = v.x; p[3 * i + 1] = v.y; p[3 * i + 2] = v.z; }

__device__ inline float clampf(float x, float lo, float hi) { return fminf(fmaxf(x, lo), hi); }
// [0,1] clamp with NaN -> 0, written with comparisons so that every implementation agrees
__device__ inline float sat(float x) { return x > 0.0f ? (x < 1.0f ? x : 1.0f) : 0.0f; }

// ---- deterministic exp ----
// Cody-Waite reduction x = n*ln2 + r (ln2 split into a high part with trailing zero bits and a low
// correction), e^r from its Taylor series through r^7 (|r| <= ln2/2, truncation < 6e-9 relative),
// and the 2^n scale applied through the exponent field. Inputs below -87 return 0, above 88 inf.
constexpr float kLn2Hi = 0.693145751953125f;      // ln2 rounded to 16 significant bits
constexpr float kLn2Lo = 1.428606765330187e-06f;  // ln2 - kLn2Hi
constexpr float kLog2e = 1.44269504088896341f;

__device__ inline float det_exp(float x) {
    if (x != x) return x;
    if (x < -87.0f) return 0.0f;
    if (x > 88.0f) return __int_as_float(0x7f800000);
    const float n = rintf(x * kLog2e);
    float r = fmaf(-n, kLn2Hi, x);
    r = fmaf(-n, kLn2Lo, r);
    float p = 1.0f / 5040.0f;
    p = fmaf(p, r, 1.0f / 720.0f);
    p = fmaf(p, r, 1.0f / 120.0f);
    p = fmaf(p, r, 1.0f / 24.0f);
    p = fmaf(p, r, 1.0f / 6.0f);
    p = fmaf(p, r, 0.5f);
    p = fmaf(p, r, 1.0f);
    p = fmaf(p, r, 1.0f);
    const int e = static_cast<int>(n) + 127;   // in [1, 254] for the accepted range
    return p * __int_as_float(e << 23);
}

// sine and cosine of the Neural frequency encoding, deterministic: Cody-Waite reduction x = k (pi/2) + r with pi/2
// split into three floats (P1 = float(pi/2), P2 = float(pi/2 - P1), P3 = float(pi/2 - P1 - P2); fused multiply-adds),
// |r| <= pi/4, then the Taylor series of sin r through r^9 and of cos r through r^10 (truncation below 2e-9), rotated by
// the quadrant k mod 4. Every operation is an explicit single-rounding operation, so the oracle's C restatement gives
// the same bits, and the fp16 inputs of the MLP are identical on both sides. Arguments with |x| <= 0.78 (the latent
// features, which stay small) have k = 0 and r = x + 0, so they skip the reduction. Arguments are clamped to
// |x| <= 8192, where the three-part reduction stays accurate (the latent features never come near it); the function
// is inline arithmetic only, with no call in the MLP kernels' hot loops.
constexpr float kTwoOverPi = 0.636619746685028076171875f;
constexpr float kPio2P1 = 1.57079637050628662109375f;
constexpr float kPio2P2 = -4.371138828673792886547744274139404296875e-08f;
constexpr float kPio2P3 = -1.7151245100058819e-15f;
__device__ inline void enc_sincos(float x, float* sp, float* cp) {
    float k = 0.0f, r;
    if (fabsf(x) <= 0.78f) {
        r = __fadd_rn(x, 0.0f);
    } else {
        x = fminf(fmaxf(x, -8192.0f), 8192.0f);
        k = rintf(__fmul_rn(x, kTwoOverPi));
        r = fmaf(-k, kPio2P1, x);
        r = fmaf(-k, kPio2P2, r);
        r = fmaf(-k, kPio2P3, r);
    }
    const float r2 = __fmul_rn(r, r);
    float ps = 1.0f / 362880.0f;
    ps = fmaf(ps, r2, -1.0f / 5040.0f);
    ps = fmaf(ps, r2, 1.0f / 120.0f);
    ps = fmaf(ps, r2, -1.0f / 6.0f);
    const float sn = fmaf(ps, __fmul_rn(r2, r), r);
    float pc = -1.0f / 3628800.0f;
    pc = fmaf(pc, r2, 1.0f / 40320.0f);
    pc = fmaf(pc, r2, -1.0f / 720.0f);
    pc = fmaf(pc, r2, 1.0f / 24.0f);
    pc = fmaf(pc, r2, -0.5f);
    const float cs = fmaf(pc, r2, 1.0f);
    // quadrant q = k mod 4: (sin, cos) = (s, c), (c, -s), (-s, -c), (-c, s)
    const int q = static_cast<int>(k);
    const float so = (q & 1) ? cs : sn, co = (q & 1) ? sn : cs;
    *sp = (q & 2) ? -so : so;
    *cp = ((q + 1) & 2) ? -co : co;
}

__device__ inline float det_sigmoid(float x) { return 1.0f / (1.0f + det_exp(-x)); }

__device__ inline float rnorm3(f3 v) { return 1.0f / sqrtf(fmaxf(dot3(v, v), 1e-24f)); }

// ---- activations (rasterization/rtc/preprocess_common.cuh:51-142; Appearance/utils.py:366-417) ----
// ids: base {0 none, 1 exp(3x)}, residual {0 none, 1 tanh, 2 softplus beta 10},
// color {0 x+.5, 1 relu(x+.5), 2 softplus10(x+.5), 3 sigmoid(4x), 4 clamp(x+.5,0,1), 5 1-e^-x}
__device__ inline float softplus10(float x) { return (fmaxf(10.0f * x, 0.0f) + log1pf(expf(-fabsf(10.0f * x)))) / 10.0f; }
__device__ inline float softplus10_grad_from_y(float y) { return -expm1f(-10.0f * y); }

__device__ inline float base_act(int id, float x) { return id == 1 ? det_exp(3.0f * x) : x; }
__device__ inline float base_act_grad(int id, float x) { return id == 1 ? 3.0f * det_exp(3.0f * x) : 1.0f; }
__device__ inline float residual_act(int id, float x) {
    return id == 1 ? tanhf(x) : (id == 2 ? softplus10(x) : x);
}
__device__ inline float residual_act_grad_from_y(int id, float y) {
    return id == 1 ? 1.0f - y * y : (id == 2 ? softplus10_grad_from_y(y) : 1.0f);
}
__device__ inline float color_act(int id, float x) {
    switch (id) {
        case 1: return fmaxf(x + 0.5f, 0.0f);
        case 2: return softplus10(x + 0.5f);
        case 3: return 1.0f / (1.0f + det_exp(-4.0f * x));
        case 4: return clampf(x + 0.5f, 0.0f, 1.0f);
        case 5: return -expm1f(-x);
        default: return x + 0.5f;
    }
}
__device__ inline float color_act_grad_from_y(int id, float y) {
    switch (id) {
        case 1: return y > 0.0f ? 1.0f : 0.0f;
        case 2: return softplus10_grad_from_y(y);
        case 3: return 4.0f * (y - y * y);
        case 4: return (y > 0.0f && y < 1.0f) ? 1.0f : 0.0f;
        case 5: return 1.0f - y;
        default: return 1.0f;
    }
}
__device__ inline f3 base_act3(int id, f3 v) { return mk3(base_act(id, v.x), base_act(id, v.y), base_act(id, v.z)); }
__device__ inline f3 residual_act3(int id, f3 v) { return mk3(residual_act(id, v.x), residual_act(id, v.y), residual_act(id, v.z)); }
__device__ inline f3 color_act3(int id, f3 v) { return mk3(color_act(id, v.x), color_act(id, v.y), color_act(id, v.z)); }

// packed per-visible-primitive render record, 48 bytes (three float4):
//   q0 = (mean2d.x, mean2d.y, opacity, power_threshold = ln(255 * opacity))
//   q1 = (conic.x, conic.y, conic.z, bits(x_min | x_max << 16))
//   q2 = (color.r, color.g, color.b, bits(y_min | y_max << 16))
struct __align__(16) Record { float4 q0, q1, q2; };

// per-visible-primitive gradient accumulator filled by the backward blend, 48 bytes:
//   g0 = (d mean2d.x, d mean2d.y, d conic.x, d conic.y), g1 = (d conic.z, d color.rgb),
//   g2 = (d opacity (sigmoid derivative folded in unless proper antialiasing), |d mean2d|.x, |d mean2d|.y, 0)
struct __align__(16) GradRecord { float4 g0, g1, g2; };

}  // namespace fgs
