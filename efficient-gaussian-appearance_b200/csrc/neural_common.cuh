// Pieces of the neural appearance shared by the mma.sync kernels (neural.cu) and the tcgen05 kernels
// (neural_tc.cu): MLP shape, frequency-encoding octave, SH band inputs of the view direction and their gradient.
// Semantics: FasterGSVDACudaBackend/.../rasterization/rtc/appearance_neural.cuh:10-160 (encoding, SH degrees with
// gating of the bands beyond the active degree) and Appearance/Neural.py:40-53 (network layout).
#pragma once

#include "appearance.cuh"
#include "preprocess.cuh"

namespace fgs {

constexpr float kLossScale = kMlpLossScale;
constexpr float kShC0 = 0.28209479177387814f;

// value * 2^f: the octave scaling of the frequency encoding (exact, so equal to scalbnf for every input)
__device__ inline float octave(float value, int f) { return f == 0 ? value : value * static_cast<float>(1 << f); }

// MLP geometry of one configuration (all widths multiples of 16)
struct MlpShape {
    int kin;        // padded input width
    int nn;         // hidden width
    int layers;     // n_hidden + 1 matmuls
    int w_off[10];  // offset of each layer in the flat weight vector
    int w_rows[10]; // output rows of each layer (nn, ..., 16)
    int w_cols[10]; // input columns of each layer (kin, nn, ...)
    int n_params;
};

__host__ __device__ inline MlpShape mlp_shape(const AppearanceConfig& A) {
    MlpShape s;
    s.kin = A.n_input_pad;
    s.nn = A.n_neurons;
    s.layers = A.n_hidden + 1;
    int off = 0;
    for (int l = 0; l < s.layers; l++) {
        s.w_off[l] = off;
        s.w_cols[l] = l == 0 ? s.kin : s.nn;
        s.w_rows[l] = l == s.layers - 1 ? 16 : s.nn;
        off += s.w_rows[l] * s.w_cols[l];
    }
    s.n_params = off;
    return s;
}

// SH band values of the MLP's direction input (bands 0..3 selected by mask; band l >= 1 is zero unless it is among
// the first `deg` selected bands), passed to out(k, value) in input order; returns the number written. Every product
// and sum is an explicit single-rounding operation (this file is compiled with contraction), so the values, and the
// fp16 inputs rounded from them, are the oracle's bit for bit.
template <typename Out>
__device__ inline int sh_band_values(int mask, int deg, f3 d, Out&& out) {
    const float x = d.x, y = d.y, z = d.z;
    const float xx = __fmul_rn(x, x), yy = __fmul_rn(y, y), zz = __fmul_rn(z, z);
    const float xy = __fmul_rn(x, y), xz = __fmul_rn(x, z), yz = __fmul_rn(y, z);
    int o = 0, rank = 0;
    if (mask & 1) out(o++, kShC0);
    if (mask & 2) {
        const float m = rank++ < deg ? 1.0f : 0.0f;
        out(o++, __fmul_rn(m, __fmul_rn(-kShC1, y)));
        out(o++, __fmul_rn(m, __fmul_rn(kShC1, z)));
        out(o++, __fmul_rn(m, __fmul_rn(-kShC1, x)));
    }
    if (mask & 4) {
        const float m = rank++ < deg ? 1.0f : 0.0f;
        out(o++, __fmul_rn(m, __fmul_rn(kShC2a, xy)));
        out(o++, __fmul_rn(m, __fmul_rn(-kShC2a, yz)));
        out(o++, __fmul_rn(m, __fsub_rn(__fmul_rn(kShC2b, zz), kShC2c)));
        out(o++, __fmul_rn(m, __fmul_rn(-kShC2a, xz)));
        out(o++, __fmul_rn(m, __fsub_rn(__fmul_rn(kShC2d, xx), __fmul_rn(kShC2d, yy))));
    }
    if (mask & 8) {
        const float m = rank++ < deg ? 1.0f : 0.0f;
        const float A = 0.59004358992664352f, B = 2.8906114426405538f, C = 0.45704579946446572f;
        const float D = 0.3731763325901154f, E = 1.4453057213202769f;
        const float one_5zz = __fsub_rn(1.0f, __fmul_rn(5.0f, zz));
        out(o++, __fmul_rn(m, __fmul_rn(__fmul_rn(A, y), __fadd_rn(__fmul_rn(-3.0f, xx), yy))));
        out(o++, __fmul_rn(m, __fmul_rn(__fmul_rn(B, xy), z)));
        out(o++, __fmul_rn(m, __fmul_rn(__fmul_rn(C, y), one_5zz)));
        out(o++, __fmul_rn(m, __fmul_rn(__fmul_rn(D, z), __fsub_rn(__fmul_rn(5.0f, zz), 3.0f))));
        out(o++, __fmul_rn(m, __fmul_rn(__fmul_rn(C, x), one_5zz)));
        out(o++, __fmul_rn(m, __fmul_rn(__fmul_rn(E, z), __fsub_rn(xx, yy))));
        out(o++, __fmul_rn(m, __fmul_rn(__fmul_rn(A, x), __fadd_rn(-xx, __fmul_rn(3.0f, yy)))));
    }
    return o;
}

// gradient of sum_k g[k] * band_k(d) with respect to the unit direction
__device__ inline f3 sh_band_grad(int mask, int deg, f3 d, const float* g) {
    const float x = d.x, y = d.y, z = d.z;
    const float xx = x * x, yy = y * y, zz = z * z;
    f3 r = mk3(0.0f, 0.0f, 0.0f);
    int o = 0, rank = 0;
    if (mask & 1) o++;
    if (mask & 2) {
        if (rank++ < deg) {
            r.y += -kShC1 * g[o];
            r.z += kShC1 * g[o + 1];
            r.x += -kShC1 * g[o + 2];
        }
        o += 3;
    }
    if (mask & 4) {
        if (rank++ < deg) {
            r = r + g[o] * mk3(kShC2a * y, kShC2a * x, 0.0f);
            r = r + g[o + 1] * mk3(0.0f, -kShC2a * z, -kShC2a * y);
            r = r + g[o + 2] * mk3(0.0f, 0.0f, 2.0f * kShC2b * z);
            r = r + g[o + 3] * mk3(-kShC2a * z, 0.0f, -kShC2a * x);
            r = r + g[o + 4] * mk3(2.0f * kShC2d * x, -2.0f * kShC2d * y, 0.0f);
        }
        o += 5;
    }
    if (mask & 8) {
        if (rank++ < deg) {
            const float A = 0.59004358992664352f, B = 2.8906114426405538f, C = 0.45704579946446572f;
            const float D = 0.3731763325901154f, E = 1.4453057213202769f;
            r = r + g[o] * mk3(-6.0f * A * x * y, A * (3.0f * yy - 3.0f * xx), 0.0f);
            r = r + g[o + 1] * mk3(B * y * z, B * x * z, B * x * y);
            r = r + g[o + 2] * mk3(0.0f, C * (1.0f - 5.0f * zz), -10.0f * C * y * z);
            r = r + g[o + 3] * mk3(0.0f, 0.0f, D * (15.0f * zz - 3.0f));
            r = r + g[o + 4] * mk3(C * (1.0f - 5.0f * zz), 0.0f, -10.0f * C * x * z);
            r = r + g[o + 5] * mk3(2.0f * E * x * z, -2.0f * E * y * z, E * (xx - yy));
            r = r + g[o + 6] * mk3(A * (3.0f * yy - 3.0f * xx), 6.0f * A * x * y, 0.0f);
        }
        o += 7;
    }
    return r;
}

// unit view direction from the camera to m (and 1 / distance), in explicit single-rounding IEEE operations: the MLP's
// SH inputs depend on it bit for bit
__device__ inline f3 view_dir(const View& v, f3 m, float* rn_out) {
    const f3 dv = mk3(__fsub_rn(m.x, v.cam_pos[0]), __fsub_rn(m.y, v.cam_pos[1]), __fsub_rn(m.z, v.cam_pos[2]));
    const float d2 = __fadd_rn(__fadd_rn(__fmul_rn(dv.x, dv.x), __fmul_rn(dv.y, dv.y)), __fmul_rn(dv.z, dv.z));
    const float rn = __fdiv_rn(1.0f, __fsqrt_rn(fmaxf(d2, 1e-24f)));
    if (rn_out) *rn_out = rn;
    return mk3(__fmul_rn(rn, dv.x), __fmul_rn(rn, dv.y), __fmul_rn(rn, dv.z));
}

// store, or add with a reduction (one addition per element and launch: deterministic, no load on the critical path)
__device__ inline void put1(float* p, size_t k, float v, int acc) {
    if (acc) atomicAdd(p + k, v);
    else p[k] = v;
}
__device__ inline void put3n(float* p, uint32_t i, f3 v, int acc) { put1(p, 3ull * i, v.x, acc); put1(p, 3ull * i + 1, v.y, acc); put1(p, 3ull * i + 2, v.z, acc); }

}  // namespace fgs
