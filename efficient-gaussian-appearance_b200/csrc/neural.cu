// Neural appearance: per-Gaussian latent features -> (optional) frequency encoding, concatenated with the SH
// band values of the view direction -> fully connected fp16 MLP (no biases, ReLU or identity hidden activation,
// linear output padded to 16 rows) -> residual activation on the first three outputs.
//
// Semantics: FasterGSVDACudaBackend/.../rasterization/rtc/appearance_neural.cuh:10-407 (encoding, SH bands,
// gating, loss-scaled fp16 backward) with the MLP of tiny-cuda-nn's FullyFusedMLP as configured by
// Appearance/Neural.py:40-53. Inputs padded to a multiple of 16 carry the value 1. The flat weight vector holds
// the input layer [n_neurons, n_input_pad], the hidden layers [n_neurons, n_neurons] and the output layer
// [16, n_neurons], each row-major.
//
// Design: persistent CTAs stage the weights once as fp16 in shared memory; each warp evaluates the MLP for its
// own 32 primitives with mma.sync m16n8k16 (fp16 operands, fp32 accumulation), layer outputs rounded to fp16.
// The backward recomputes the forward activations (no forward context is stored), scales the output gradient
// by 128 before rounding it to fp16 (as the reference does), and accumulates the weight gradient in fp32 in
// shared memory across all primitives a CTA processes, flushing it with one atomic add per weight and CTA.
#include <cuda_fp16.h>
#include "preprocess_store.cuh"
#include "preprocess_bwd.cuh"
#include "appearance.cuh"
#include "launch.h"

namespace fgs {

namespace {

constexpr int kFwdRows = kChunk;  // 256 primitives per forward CTA iteration (the compaction granule)
constexpr int kBwdRows = 128;     // 128 primitives per backward CTA iteration
constexpr float kLossScale = kMlpLossScale;
constexpr float kShC0 = 0.28209479177387814f;

__device__ inline uint32_t smem_u32(const void* p) { return static_cast<uint32_t>(__cvta_generic_to_shared(p)); }

__device__ inline void ldsm_x4(uint32_t r[4], const void* p) {
    asm volatile("ldmatrix.sync.aligned.m8n8.x4.shared.b16 {%0, %1, %2, %3}, [%4];\n"
                 : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3])
                 : "r"(smem_u32(p)));
}
__device__ inline void ldsm_x4_t(uint32_t r[4], const void* p) {
    asm volatile("ldmatrix.sync.aligned.m8n8.x4.trans.shared.b16 {%0, %1, %2, %3}, [%4];\n"
                 : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3])
                 : "r"(smem_u32(p)));
}
__device__ inline void mma16816(float c[4], const uint32_t a[4], uint32_t b0, uint32_t b1) {
    asm volatile("mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32 {%0, %1, %2, %3}, {%4, %5, %6, %7}, {%8, %9}, {%0, %1, %2, %3};\n"
                 : "+f"(c[0]), "+f"(c[1]), "+f"(c[2]), "+f"(c[3])
                 : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
}

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

// half-precision weight matrices in shared memory: layer l at offset sw_off[l] (halves), row stride cols + 8
__host__ __device__ inline int smem_weights_halves(const MlpShape& s, int* offs) {
    int off = 0;
    for (int l = 0; l < s.layers; l++) {
        if (offs) offs[l] = off;
        off += s.w_rows[l] * (s.w_cols[l] + 8);
    }
    return off;
}

__device__ inline void load_weights(const MlpShape& s, const float* __restrict__ w, __half* sw, const int* soff) {
    for (int l = 0; l < s.layers; l++) {
        const int rows = s.w_rows[l], cols = s.w_cols[l], ld = cols + 8;
        for (int e = threadIdx.x; e < rows * cols; e += blockDim.x) {
            const int r = e / cols, c = e - r * cols;
            sw[soff[l] + r * ld + c] = __float2half_rn(w[s.w_off[l] + e]);
        }
    }
}

// one layer for the warp's 32 rows: out[row][0..NOUT) = act(in[row][0..K) . W^T), rounded to fp16
template <int NOUT>
__device__ inline void layer_forward(const __half* in, int ld_in, int K, const __half* W, int ld_w, __half* out, int ld_out, int row0, bool relu) {
    const int lane = threadIdx.x & 31;
    float acc[2][NOUT / 8][4];
#pragma unroll
    for (int m = 0; m < 2; m++)
#pragma unroll
        for (int n = 0; n < NOUT / 8; n++)
#pragma unroll
            for (int q = 0; q < 4; q++) acc[m][n][q] = 0.0f;
    for (int k0 = 0; k0 < K; k0 += 16) {
        uint32_t a[2][4];
#pragma unroll
        for (int m = 0; m < 2; m++) ldsm_x4(a[m], in + (row0 + m * 16 + (lane & 15)) * ld_in + k0 + (lane >> 4) * 8);
#pragma unroll
        for (int n = 0; n < NOUT / 8; n += 2) {
            uint32_t b[4];
            ldsm_x4(b, W + (n * 8 + (lane & 7) + (lane >> 4) * 8) * ld_w + k0 + ((lane >> 3) & 1) * 8);
#pragma unroll
            for (int m = 0; m < 2; m++) {
                mma16816(acc[m][n], a[m], b[0], b[1]);
                mma16816(acc[m][n + 1], a[m], b[2], b[3]);
            }
        }
    }
    const int g = lane >> 2, tq = lane & 3;
#pragma unroll
    for (int m = 0; m < 2; m++)
#pragma unroll
        for (int n = 0; n < NOUT / 8; n++) {
            float v0 = acc[m][n][0], v1 = acc[m][n][1], v2 = acc[m][n][2], v3 = acc[m][n][3];
            if (relu) { v0 = fmaxf(v0, 0.0f); v1 = fmaxf(v1, 0.0f); v2 = fmaxf(v2, 0.0f); v3 = fmaxf(v3, 0.0f); }
            const int r = row0 + m * 16 + g, c = n * 8 + tq * 2;
            *reinterpret_cast<__half2*>(out + r * ld_out + c) = __floats2half2_rn(v0, v1);
            *reinterpret_cast<__half2*>(out + (r + 8) * ld_out + c) = __floats2half2_rn(v2, v3);
        }
}

// SH band values of the MLP's direction input (bands 0..3 selected by mask; band l >= 1 is zero unless it is among
// the first `deg` selected bands); returns the number written
__device__ inline int sh_band_values(int mask, int deg, f3 d, float* out) {
    const float x = d.x, y = d.y, z = d.z;
    const float xx = x * x, yy = y * y, zz = z * z, xy = x * y, xz = x * z, yz = y * z;
    int o = 0, rank = 0;
    if (mask & 1) out[o++] = kShC0;
    if (mask & 2) {
        const float m = rank++ < deg ? 1.0f : 0.0f;
        out[o++] = m * (-kShC1 * y);
        out[o++] = m * (kShC1 * z);
        out[o++] = m * (-kShC1 * x);
    }
    if (mask & 4) {
        const float m = rank++ < deg ? 1.0f : 0.0f;
        out[o++] = m * (kShC2a * xy);
        out[o++] = m * (-kShC2a * yz);
        out[o++] = m * (kShC2b * zz - kShC2c);
        out[o++] = m * (-kShC2a * xz);
        out[o++] = m * (kShC2d * xx - kShC2d * yy);
    }
    if (mask & 8) {
        const float m = rank++ < deg ? 1.0f : 0.0f;
        out[o++] = m * (0.59004358992664352f * y * (-3.0f * xx + yy));
        out[o++] = m * (2.8906114426405538f * xy * z);
        out[o++] = m * (0.45704579946446572f * y * (1.0f - 5.0f * zz));
        out[o++] = m * (0.3731763325901154f * z * (5.0f * zz - 3.0f));
        out[o++] = m * (0.45704579946446572f * x * (1.0f - 5.0f * zz));
        out[o++] = m * (1.4453057213202769f * z * (xx - yy));
        out[o++] = m * (0.59004358992664352f * x * (-xx + 3.0f * yy));
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

// writes this thread's MLP input row (fp16): encoded features, SH band values, padding ones
__device__ inline void assemble_inputs(const Params& P, const AppearanceConfig& A, uint32_t i, bool valid, f3 d, int deg, __half* row) {
    const int F = A.feature_dim, nraw = F + (A.base_input ? 3 : 0), nf = A.n_freq;
    int o = 0;
    for (int j = 0; j < nraw; j++) {
        float val = 0.0f;
        if (valid) val = j < F ? P.residual[static_cast<size_t>(i) * F + j] : P.base[3ull * i + (j - F)];
        if (nf == 0) {
            row[o++] = __float2half_rn(val);
        } else {
            for (int f = 0; f < nf; f++) {
                float s, c;
                sincosf(scalbnf(val, f), &s, &c);
                row[o++] = __float2half_rn(s);
                row[o++] = __float2half_rn(c);
            }
        }
    }
    float sh[16];
    const int nsh = sh_band_values(A.sh_mask, deg, d, sh);
    for (int k = 0; k < nsh; k++) row[o++] = __float2half_rn(sh[k]);
    for (; o < A.n_input_pad; o++) row[o] = __float2half_rn(1.0f);
}

__device__ inline f3 view_dir(const View& v, f3 m, float* rn_out) {
    const f3 cam = mk3(v.cam_pos[0], v.cam_pos[1], v.cam_pos[2]);
    const f3 dv = m - cam;
    const float rn = rnorm3(dv);
    if (rn_out) *rn_out = rn;
    return rn * dv;
}

// runs the MLP for the warp's rows [row0, row0 + 32); buffers: bufA holds the input on entry; returns the buffer
// (and its stride) that holds the 16 outputs
template <int NN>
__device__ inline const __half* mlp_forward_warp(const MlpShape& s, const __half* sw, const int* soff, __half* bufA, int ldA, __half* bufB,
                                                 int ldB, int row0, int hidden_act, int* ld_out) {
    __half* in = bufA;
    int ld_in = ldA;
    __half* out = bufB;
    int ld_o = ldB;
    for (int l = 0; l < s.layers; l++) {
        const bool last = l == s.layers - 1;
        if (last) layer_forward<16>(in, ld_in, s.w_cols[l], sw + soff[l], s.w_cols[l] + 8, out, ld_o, row0, false);
        else layer_forward<NN>(in, ld_in, s.w_cols[l], sw + soff[l], s.w_cols[l] + 8, out, ld_o, row0, hidden_act == 1);
        __syncwarp();
        __half* t = in; in = out; out = t;
        const int tl = ld_in; ld_in = ld_o; ld_o = tl;
    }
    *ld_out = ld_in;
    return in;
}

// ---------------------------------------------------------------------------------------------------
// forward preprocess with the fused MLP
template <int NN>
__global__ void __launch_bounds__(kFwdRows) neural_fwd_kernel(Params P, AppearanceConfig A, View v, PrimBuffers B, uint32_t n_chunks) {
    extern __shared__ __align__(16) unsigned char smem[];
    const MlpShape s = mlp_shape(A);
    int soff[10];
    const int wh = smem_weights_halves(s, soff);
    __half* sw = reinterpret_cast<__half*>(smem);
    const int ldA = (s.kin > NN ? s.kin : NN) + 8, ldB = NN + 8;
    __half* bufA = sw + ((wh + 7) & ~7);
    __half* bufB = bufA + kFwdRows * ldA;
    load_weights(s, P.mlp, sw, soff);
    __syncthreads();
    const int deg = min(v.degree, A.max_degree);
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    for (uint32_t chunk = blockIdx.x; chunk < n_chunks; chunk += gridDim.x) {
        const uint32_t i = chunk * kFwdRows + threadIdx.x;
        const bool in_range = i < P.n;
        const Geometry G = project_primitive(P.means, P.scales, P.rotations, P.opacities, in_range ? i : 0, in_range, v);
        const bool visible = in_range && G.n_touched > 0;
        f3 res = mk3(0.0f, 0.0f, 0.0f);
        if (deg > 0 && __any_sync(0xffffffffu, visible)) {
            const f3 d = view_dir(v, visible ? ld3(P.means, i) : mk3(0.0f, 0.0f, 1.0f), nullptr);
            assemble_inputs(P, A, i, visible, d, deg, bufA + threadIdx.x * ldA);
            __syncwarp();
            int ldo;
            const __half* y = mlp_forward_warp<NN>(s, sw, soff, bufA, ldA, bufB, ldB, warp * 32, A.hidden_act, &ldo);
            const __half* yr = y + threadIdx.x * ldo;
            res = residual_act3(A.res_act, mk3(__half2float(yr[0]), __half2float(yr[1]), __half2float(yr[2])));
            __syncwarp();
        }
        (void)lane;
        f3 color = mk3(0.0f, 0.0f, 0.0f);
        if (visible) {
            const f3 base = base_act3(A.base_act, ld3(P.base, i));
            color = color_act3(A.color_act, base + res);
            if (!v.render_base) {
                const f3 bc = color_act3(A.color_act, base);
                color = mk3(fabsf(color.x - bc.x), fabsf(color.y - bc.y), fabsf(color.z - bc.z));
            }
        }
        store_primitive(B, i, in_range, G, color, chunk);
    }
}

// ---------------------------------------------------------------------------------------------------
// backward

// dIn[row][0..K) = dOut[row][0..NOUT) . W (W: [NOUT][K]) for the warp's rows, 32 output columns at a time;
// masked by (act_in > 0) when relu, rounded to fp16 into `out` or stored as fp32 into `out32`
template <int NOUT>
__device__ inline void layer_backward_data(const __half* dout, int ld_dout, const __half* W, int ld_w, int K, const __half* act_in, int ld_act,
                                           bool relu, __half* out, int ld_out, float* out32, int ld_out32, int row0) {
    const int lane = threadIdx.x & 31, g = lane >> 2, tq = lane & 3;
    for (int c0 = 0; c0 < K; c0 += 32) {
        const int ncols = min(32, K - c0);
        float acc[2][4][4];
#pragma unroll
        for (int m = 0; m < 2; m++)
#pragma unroll
            for (int n = 0; n < 4; n++)
#pragma unroll
                for (int q = 0; q < 4; q++) acc[m][n][q] = 0.0f;
#pragma unroll
        for (int kk = 0; kk < NOUT; kk += 16) {
            uint32_t a[2][4];
#pragma unroll
            for (int m = 0; m < 2; m++) ldsm_x4(a[m], dout + (row0 + m * 16 + (lane & 15)) * ld_dout + kk + (lane >> 4) * 8);
#pragma unroll
            for (int n = 0; n < 4; n += 2) {
                if (n * 8 >= ncols) break;
                uint32_t b[4];
                ldsm_x4_t(b, W + (kk + ((lane >> 3) & 1) * 8 + (lane & 7)) * ld_w + c0 + n * 8 + (lane >> 4) * 8);
#pragma unroll
                for (int m = 0; m < 2; m++) {
                    mma16816(acc[m][n], a[m], b[0], b[1]);
                    mma16816(acc[m][n + 1], a[m], b[2], b[3]);
                }
            }
        }
#pragma unroll
        for (int m = 0; m < 2; m++)
#pragma unroll
            for (int n = 0; n < 4; n++) {
                if (n * 8 >= ncols) break;
                const int r = row0 + m * 16 + g, c = c0 + n * 8 + tq * 2;
                float v0 = acc[m][n][0], v1 = acc[m][n][1], v2 = acc[m][n][2], v3 = acc[m][n][3];
                if (relu) {
                    const __half2 h01 = *reinterpret_cast<const __half2*>(act_in + r * ld_act + c);
                    const __half2 h23 = *reinterpret_cast<const __half2*>(act_in + (r + 8) * ld_act + c);
                    if (!(__low2float(h01) > 0.0f)) v0 = 0.0f;
                    if (!(__high2float(h01) > 0.0f)) v1 = 0.0f;
                    if (!(__low2float(h23) > 0.0f)) v2 = 0.0f;
                    if (!(__high2float(h23) > 0.0f)) v3 = 0.0f;
                }
                if (out) {
                    *reinterpret_cast<__half2*>(out + r * ld_out + c) = __floats2half2_rn(v0, v1);
                    *reinterpret_cast<__half2*>(out + (r + 8) * ld_out + c) = __floats2half2_rn(v2, v3);
                } else {
                    out32[r * ld_out32 + c] = v0;
                    out32[r * ld_out32 + c + 1] = v1;
                    out32[(r + 8) * ld_out32 + c] = v2;
                    out32[(r + 8) * ld_out32 + c + 1] = v3;
                }
            }
    }
}

// dW[M][K] += dOut^T[M][rows] . In[rows][K] over all kBwdRows rows; 16x16 output tiles distributed over the warps
__device__ inline void layer_backward_weights(const __half* dout, int ld_dout, int M, const __half* in, int ld_in, int K, float* dW) {
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5, nwarps = blockDim.x >> 5;
    const int g = lane >> 2, tq = lane & 3;
    const int tiles_m = M / 16, tiles_k = K / 16;
    for (int t = warp; t < tiles_m * tiles_k; t += nwarps) {
        const int m0 = (t / tiles_k) * 16, n0 = (t % tiles_k) * 16;
        float acc[2][4] = {{0.0f, 0.0f, 0.0f, 0.0f}, {0.0f, 0.0f, 0.0f, 0.0f}};
        for (int k0 = 0; k0 < kBwdRows; k0 += 16) {
            uint32_t a[4], b[4];
            ldsm_x4_t(a, dout + (k0 + (lane >> 4) * 8 + (lane & 7)) * ld_dout + m0 + ((lane >> 3) & 1) * 8);
            ldsm_x4_t(b, in + (k0 + ((lane >> 3) & 1) * 8 + (lane & 7)) * ld_in + n0 + (lane >> 4) * 8);
            mma16816(acc[0], a, b[0], b[1]);
            mma16816(acc[1], a, b[2], b[3]);
        }
#pragma unroll
        for (int n = 0; n < 2; n++) {
            const int r = m0 + g, c = n0 + n * 8 + tq * 2;
            dW[r * K + c] += acc[n][0];
            dW[r * K + c + 1] += acc[n][1];
            dW[(r + 8) * K + c] += acc[n][2];
            dW[(r + 8) * K + c + 1] += acc[n][3];
        }
    }
}

__device__ inline void put1(float* p, size_t k, float v, int acc) { if (acc) p[k] += v; else p[k] = v; }
__device__ inline void put3n(float* p, uint32_t i, f3 v, int acc) { put1(p, 3ull * i, v.x, acc); put1(p, 3ull * i + 1, v.y, acc); put1(p, 3ull * i + 2, v.z, acc); }

struct NeuralBwdSmem {
    int soff[10];
    int wh;
    int ldX, ldH, ldY, ldD, ldG;
    size_t off_dw, off_x, off_h, off_y, off_d, off_g, total;
};

__host__ __device__ inline NeuralBwdSmem neural_bwd_layout(const MlpShape& s) {
    NeuralBwdSmem L;
    L.wh = smem_weights_halves(s, L.soff);
    L.ldX = s.kin + 8;
    L.ldH = s.nn + 8;
    L.ldY = 16 + 8;
    L.ldD = s.nn + 8;
    L.ldG = s.kin + 4;
    size_t off = (static_cast<size_t>(L.wh) * 2 + 15) & ~static_cast<size_t>(15);
    L.off_dw = off;
    off += static_cast<size_t>(s.n_params) * 4;
    L.off_x = off;
    off += static_cast<size_t>(kBwdRows) * L.ldX * 2;
    L.off_h = off;
    off += static_cast<size_t>(kBwdRows) * L.ldH * 2 * (s.layers - 1 > 0 ? s.layers - 1 : 1);
    L.off_y = off;
    off += static_cast<size_t>(kBwdRows) * L.ldY * 2;
    L.off_d = off;
    off += static_cast<size_t>(kBwdRows) * L.ldD * 2 * 2;
    L.off_g = off;
    off += static_cast<size_t>(kBwdRows) * L.ldG * 4;
    L.total = off;
    return L;
}

template <int NN>
__global__ void __launch_bounds__(kBwdRows) neural_bwd_kernel(Params P, AppearanceConfig A, View v, const uint32_t* __restrict__ rank_of,
                                                              const Record* __restrict__ sorted_rec, const GradRecord* __restrict__ grads,
                                                              GradOut O, uint32_t n_chunks) {
    extern __shared__ __align__(16) unsigned char smem[];
    const MlpShape s = mlp_shape(A);
    const NeuralBwdSmem L = neural_bwd_layout(s);
    __half* sw = reinterpret_cast<__half*>(smem);
    float* dW = reinterpret_cast<float*>(smem + L.off_dw);
    __half* X = reinterpret_cast<__half*>(smem + L.off_x);
    __half* H = reinterpret_cast<__half*>(smem + L.off_h);   // layer inputs 1..layers-1
    __half* Y = reinterpret_cast<__half*>(smem + L.off_y);   // outputs, then the scaled output gradient
    __half* D0 = reinterpret_cast<__half*>(smem + L.off_d);  // ping-pong hidden gradients
    __half* D1 = D0 + kBwdRows * L.ldD;
    float* GX = reinterpret_cast<float*>(smem + L.off_g);    // input gradient (fp32, scaled)
    load_weights(s, P.mlp, sw, L.soff);
    for (int e = threadIdx.x; e < s.n_params; e += blockDim.x) dW[e] = 0.0f;
    __syncthreads();
    const int deg = min(v.degree, A.max_degree);
    const int warp = threadIdx.x >> 5, t = threadIdx.x;
    const int acc_mode = O.accumulate;
    const int F = A.feature_dim;
    const int nraw = F + (A.base_input ? 3 : 0), per = A.n_freq > 0 ? 2 * A.n_freq : 1;
    for (uint32_t chunk = blockIdx.x; chunk < n_chunks; chunk += gridDim.x) {
        const uint32_t i = chunk * kBwdRows + t;
        const bool in_range = i < P.n;
        const uint32_t r = in_range ? rank_of[i] : kInvalidRank;
        const bool visible = r != kInvalidRank;
        GradRecord g;
        Record rq;
        f3 gpre = mk3(0.0f, 0.0f, 0.0f), m = mk3(0.0f, 0.0f, 1.0f);
        if (visible) {
            g = grads[r];
            rq = sorted_rec[r];
            m = ld3(P.means, i);
            const f3 col = mk3(rq.q2.x, rq.q2.y, rq.q2.z);
            gpre = mk3(g.g1.y, g.g1.z, g.g1.w) * mk3(color_act_grad_from_y(A.color_act, col.x), color_act_grad_from_y(A.color_act, col.y),
                                                     color_act_grad_from_y(A.color_act, col.z));
        }
        float rn = 1.0f;
        const f3 d = view_dir(v, m, &rn);
        f3 gbase = mk3(0.0f, 0.0f, 0.0f);
        if (visible && v.render_base) {
            const f3 b = ld3(P.base, i);
            gbase = mk3(base_act_grad(A.base_act, b.x), base_act_grad(A.base_act, b.y), base_act_grad(A.base_act, b.z)) * gpre;
        }
        f3 gmean_color = mk3(0.0f, 0.0f, 0.0f);
        const bool any_visible = __syncthreads_or(visible);
        if (deg > 0 && any_visible) {
            assemble_inputs(P, A, i, visible, d, deg, X + t * L.ldX);
            __syncwarp();
            // forward, keeping every layer's input
            const int row0 = warp * 32;
            for (int l = 0; l < s.layers; l++) {
                const __half* in = l == 0 ? X : H + (l - 1) * kBwdRows * L.ldH;
                const int ldi = l == 0 ? L.ldX : L.ldH;
                if (l == s.layers - 1) layer_forward<16>(in, ldi, s.w_cols[l], sw + L.soff[l], s.w_cols[l] + 8, Y, L.ldY, row0, false);
                else layer_forward<NN>(in, ldi, s.w_cols[l], sw + L.soff[l], s.w_cols[l] + 8, H + l * kBwdRows * L.ldH, L.ldH, row0, A.hidden_act == 1);
                __syncwarp();
            }
            // scaled output gradient
            {
                __half* yr = Y + t * L.ldY;
                float dy[3] = {0.0f, 0.0f, 0.0f};
                if (visible) {
                    const float gv[3] = {gpre.x, gpre.y, gpre.z};
                    for (int c = 0; c < 3; c++) {
                        const float y = __half2float(yr[c]);
                        dy[c] = gv[c] * residual_act_grad_from_y(A.res_act, residual_act(A.res_act, y));
                    }
                }
                for (int c = 0; c < 16; c++) yr[c] = __float2half_rn(c < 3 ? kLossScale * dy[c] : 0.0f);
            }
            __syncthreads();
            // output layer and hidden layers, last to first
            const __half* dcur = Y;
            int ld_cur = L.ldY;
            __half* dbuf[2] = {D0, D1};
            int pp = 0;
            for (int l = s.layers - 1; l >= 0; l--) {
                const __half* in = l == 0 ? X : H + (l - 1) * kBwdRows * L.ldH;
                const int ldi = l == 0 ? L.ldX : L.ldH;
                float* dWl = dW + s.w_off[l];
                layer_backward_weights(dcur, ld_cur, s.w_rows[l], in, ldi, s.w_cols[l], dWl);
                if (l > 0) {
                    __half* dnext = dbuf[pp];
                    if (s.w_rows[l] == 16) layer_backward_data<16>(dcur, ld_cur, sw + L.soff[l], s.w_cols[l] + 8, s.w_cols[l], in, ldi, A.hidden_act == 1, dnext, L.ldD, nullptr, 0, row0);
                    else layer_backward_data<NN>(dcur, ld_cur, sw + L.soff[l], s.w_cols[l] + 8, s.w_cols[l], in, ldi, A.hidden_act == 1, dnext, L.ldD, nullptr, 0, row0);
                    dcur = dnext;
                    ld_cur = L.ldD;
                    pp ^= 1;
                } else {
                    if (s.w_rows[0] == 16) layer_backward_data<16>(dcur, ld_cur, sw + L.soff[0], s.w_cols[0] + 8, s.w_cols[0], nullptr, 0, false, nullptr, 0, GX, L.ldG, row0);
                    else layer_backward_data<NN>(dcur, ld_cur, sw + L.soff[0], s.w_cols[0] + 8, s.w_cols[0], nullptr, 0, false, nullptr, 0, GX, L.ldG, row0);
                }
                __syncthreads();
            }
            // feature, base-input and direction gradients from the (scaled) input gradient
            if (visible) {
                const float* gx = GX + t * L.ldG;
                const float inv = 1.0f / kLossScale;
                float* gres = O.residual + static_cast<size_t>(i) * F;
                for (int j = 0; j < nraw; j++) {
                    const float val = j < F ? P.residual[static_cast<size_t>(i) * F + j] : P.base[3ull * i + (j - F)];
                    float gv = 0.0f;
                    if (A.n_freq == 0) gv = gx[j];
                    else
                        for (int f = 0; f < A.n_freq; f++) {
                            float sn, cs;
                            sincosf(scalbnf(val, f), &sn, &cs);
                            gv += static_cast<float>(1 << f) * (cs * gx[j * per + 2 * f] - sn * gx[j * per + 2 * f + 1]);
                        }
                    gv *= inv;
                    if (j < F) put1(gres, j, gv, acc_mode);
                    else if (j == F) gbase.x += gv;
                    else if (j == F + 1) gbase.y += gv;
                    else gbase.z += gv;
                }
                float gsh[16];
                int nsh = 0;
                for (int l = 0; l <= 3; l++)
                    if (A.sh_mask & (1 << l)) nsh += 2 * l + 1;
                for (int k = 0; k < nsh; k++) gsh[k] = gx[nraw * per + k] * inv;
                const f3 gd = sh_band_grad(A.sh_mask, deg, d, gsh);
                gmean_color = rn * (gd - dot3(gd, d) * d);
            }
            __syncthreads();
        } else if (visible) {
            float* gres = O.residual + static_cast<size_t>(i) * F;
            for (int j = 0; j < F; j++) put1(gres, j, 0.0f, acc_mode);
        }
        if (!in_range) continue;
        if (!visible) {
            if (acc_mode) continue;
            put3n(O.means, i, mk3(0.0f, 0.0f, 0.0f), 0);
            put3n(O.scales, i, mk3(0.0f, 0.0f, 0.0f), 0);
            for (int k = 0; k < 4; k++) O.rotations[4ull * i + k] = 0.0f;
            O.opacities[i] = 0.0f;
            put3n(O.base, i, mk3(0.0f, 0.0f, 0.0f), 0);
            for (int j = 0; j < F; j++) O.residual[static_cast<size_t>(i) * F + j] = 0.0f;
            continue;
        }
        put3n(O.base, i, gbase, acc_mode);
        float gmx, gmy, gca, gcb, gcc, g_opacity;
        blend_sums_to_grads(g, rq, v.proper_aa, gmx, gmy, gca, gcb, gcc, g_opacity);
        const f3 gmean = geometry_backward(P, v, i, m, gmx, gmy, gca, gcb, gcc, g_opacity, O);
        if (O.densification != nullptr && O.densification_rows == 3) {
            const float nx = 0.5f * (g.g2.y * static_cast<float>(v.width)), ny = 0.5f * (g.g2.z * static_cast<float>(v.height));
            O.densification[2ull * P.n + i] += sqrtf(nx * nx + ny * ny);
        }
        put1(O.opacities, i, g_opacity, acc_mode);
        put3n(O.means, i, A.dir_grad ? gmean + gmean_color : gmean, acc_mode);
    }
    __syncthreads();
    const float inv = 1.0f / kLossScale;
    for (int e = threadIdx.x; e < s.n_params; e += blockDim.x) atomicAdd(O.mlp + e, dW[e] * inv);
}

int sm_count() {
    int dev = 0, sms = 148;
    cudaGetDevice(&dev);
    cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
    return sms;
}

size_t fwd_smem_bytes(const AppearanceConfig& A) {
    const MlpShape s = mlp_shape(A);
    const int wh = smem_weights_halves(s, nullptr);
    const int ldA = (s.kin > s.nn ? s.kin : s.nn) + 8, ldB = s.nn + 8;
    return static_cast<size_t>((wh + 7) & ~7) * 2 + static_cast<size_t>(kFwdRows) * (ldA + ldB) * 2;
}

template <typename K>
cudaError_t launch_persistent(K kernel, size_t smem, int threads, uint32_t n_chunks, int* grid_out) {
    cudaError_t e = cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, static_cast<int>(smem));
    if (e != cudaSuccess) return e;
    int per_sm = 0;
    e = cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, kernel, threads, smem);
    if (e != cudaSuccess) return e;
    if (per_sm < 1) return cudaErrorInvalidConfiguration;
    const uint32_t cap = static_cast<uint32_t>(per_sm) * static_cast<uint32_t>(sm_count());
    *grid_out = static_cast<int>(n_chunks < cap ? n_chunks : cap);
    return cudaSuccess;
}

}  // namespace

cudaError_t launch_preprocess_fwd_neural(const Params& P, const AppearanceConfig& A, const View& v, const PrimBuffers& B, cudaStream_t st) {
    const uint32_t n_chunks = (P.n + kFwdRows - 1) / kFwdRows;
    if (n_chunks == 0) return cudaSuccess;
    const size_t smem = fwd_smem_bytes(A);
    int grid = 0;
    cudaError_t e = cudaSuccess;
    switch (A.n_neurons) {
        case 16: e = launch_persistent(neural_fwd_kernel<16>, smem, kFwdRows, n_chunks, &grid); if (!e) neural_fwd_kernel<16><<<grid, kFwdRows, smem, st>>>(P, A, v, B, n_chunks); break;
        case 32: e = launch_persistent(neural_fwd_kernel<32>, smem, kFwdRows, n_chunks, &grid); if (!e) neural_fwd_kernel<32><<<grid, kFwdRows, smem, st>>>(P, A, v, B, n_chunks); break;
        case 64: e = launch_persistent(neural_fwd_kernel<64>, smem, kFwdRows, n_chunks, &grid); if (!e) neural_fwd_kernel<64><<<grid, kFwdRows, smem, st>>>(P, A, v, B, n_chunks); break;
        default: return cudaErrorInvalidValue;
    }
    if (e != cudaSuccess) return e;
    return cudaGetLastError();
}

cudaError_t launch_preprocess_bwd_neural(const Params& P, const AppearanceConfig& A, const View& v, const uint32_t* rank_of,
                                         const Record* sorted_rec, const GradRecord* grads, const GradOut& O, cudaStream_t st) {
    const uint32_t n_chunks = (P.n + kBwdRows - 1) / kBwdRows;
    if (n_chunks == 0) return cudaSuccess;
    if (!O.accumulate) {
        cudaError_t e = cudaMemsetAsync(O.mlp, 0, static_cast<size_t>(A.n_params) * sizeof(float), st);
        if (e != cudaSuccess) return e;
    }
    const MlpShape s = mlp_shape(A);
    const size_t smem = neural_bwd_layout(s).total;
    int grid = 0;
    cudaError_t e = cudaSuccess;
    switch (A.n_neurons) {
        case 16: e = launch_persistent(neural_bwd_kernel<16>, smem, kBwdRows, n_chunks, &grid); if (!e) neural_bwd_kernel<16><<<grid, kBwdRows, smem, st>>>(P, A, v, rank_of, sorted_rec, grads, O, n_chunks); break;
        case 32: e = launch_persistent(neural_bwd_kernel<32>, smem, kBwdRows, n_chunks, &grid); if (!e) neural_bwd_kernel<32><<<grid, kBwdRows, smem, st>>>(P, A, v, rank_of, sorted_rec, grads, O, n_chunks); break;
        case 64: e = launch_persistent(neural_bwd_kernel<64>, smem, kBwdRows, n_chunks, &grid); if (!e) neural_bwd_kernel<64><<<grid, kBwdRows, smem, st>>>(P, A, v, rank_of, sorted_rec, grads, O, n_chunks); break;
        default: return cudaErrorInvalidValue;
    }
    if (e != cudaSuccess) return e;
    return cudaGetLastError();
}

size_t neural_grad_scratch_floats(const AppearanceConfig& A) { return static_cast<size_t>(A.n_params); }

size_t neural_smem_bytes(const AppearanceConfig& A) {
    const size_t b = neural_bwd_layout(mlp_shape(A)).total, f = fwd_smem_bytes(A);
    return b > f ? b : f;
}

}  // namespace fgs
