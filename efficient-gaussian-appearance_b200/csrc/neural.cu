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
// Design (rows = visible primitives, taken from the order-preserving compaction list, so no MLP work is spent on
// culled primitives):
//  - forward: after the geometry pass, a colour pass evaluates the MLP for 32 rows per warp with mma.sync m16n8k16
//    (fp16 operands, fp32 accumulation, layer outputs rounded to fp16) and writes the colour into the record;
//    features are loaded and encoded one lane per feature (coalesced 128-byte rows), SH inputs one lane per row;
//  - backward: 8 warps x 16 rows per CTA batch of 128 rows; the forward activations are recomputed, the output
//    gradient is scaled by 128 before rounding to fp16 (as the reference does); the hidden-layer gradients
//    overwrite their activations in place and the input gradient (fp32) reuses the dead buffers, so two CTAs fit
//    on an SM; the weight gradient is accumulated in registers over every batch a CTA processes, each warp owning
//    fixed 16x16 tiles, and flushed with one atomic add per weight and CTA at the end.
//  Configurations whose weight-gradient tiles exceed the register budget (or degree-0 views) use a general
//  backward over all primitives that keeps the weight gradient in shared memory.
#include <cuda_fp16.h>

#include <algorithm>
#include "preprocess_bwd.cuh"
#include "neural_common.cuh"
#include "launch.h"

namespace fgs {

namespace {

constexpr int kBwdRows = 128;  // rows per backward CTA batch

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

// one layer for the warp's 16 * MT rows: out[row][0..NOUT) = act(in[row][0..K) . W^T), rounded to fp16
template <int NOUT, int MT>
__device__ inline void layer_forward(const __half* in, int ld_in, int K, const __half* W, int ld_w, __half* out, int ld_out, int row0, bool relu) {
    const int lane = threadIdx.x & 31;
    float acc[MT][NOUT / 8][4];
#pragma unroll
    for (int m = 0; m < MT; m++)
#pragma unroll
        for (int n = 0; n < NOUT / 8; n++)
#pragma unroll
            for (int q = 0; q < 4; q++) acc[m][n][q] = 0.0f;
    for (int k0 = 0; k0 < K; k0 += 16) {
        uint32_t a[MT][4];
#pragma unroll
        for (int m = 0; m < MT; m++) ldsm_x4(a[m], in + (row0 + m * 16 + (lane & 15)) * ld_in + k0 + (lane >> 4) * 8);
#pragma unroll
        for (int n = 0; n < NOUT / 8; n += 2) {
            uint32_t b[4];
            ldsm_x4(b, W + (n * 8 + (lane & 7) + (lane >> 4) * 8) * ld_w + k0 + ((lane >> 3) & 1) * 8);
#pragma unroll
            for (int m = 0; m < MT; m++) {
                mma16816(acc[m][n], a[m], b[0], b[1]);
                mma16816(acc[m][n + 1], a[m], b[2], b[3]);
            }
        }
    }
    const int g = lane >> 2, tq = lane & 3;
#pragma unroll
    for (int m = 0; m < MT; m++)
#pragma unroll
        for (int n = 0; n < NOUT / 8; n++) {
            float v0 = acc[m][n][0], v1 = acc[m][n][1], v2 = acc[m][n][2], v3 = acc[m][n][3];
            if (relu) { v0 = fmaxf(v0, 0.0f); v1 = fmaxf(v1, 0.0f); v2 = fmaxf(v2, 0.0f); v3 = fmaxf(v3, 0.0f); }
            const int r = row0 + m * 16 + g, c = n * 8 + tq * 2;
            *reinterpret_cast<__half2*>(out + r * ld_out + c) = __floats2half2_rn(v0, v1);
            *reinterpret_cast<__half2*>(out + (r + 8) * ld_out + c) = __floats2half2_rn(v2, v3);
        }
}

// writes this thread's MLP input row (fp16): encoded features, SH band values, padding ones
__device__ inline void assemble_inputs(const Params& P, const AppearanceConfig& A, uint32_t i, bool valid, f3 d, int deg, __half* row) {
    if (!valid) {  // all-zero row: finite activations, no contribution to the weight gradient
        for (int o = 0; o < A.n_input_pad; o++) row[o] = __float2half_rn(0.0f);
        return;
    }
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
                enc_sincos(octave(val, f), &s, &c);
                row[o++] = __float2half_rn(s);
                row[o++] = __float2half_rn(c);
            }
        }
    }
    const int o0 = o;
    o += sh_band_values(A.sh_mask, deg, d, [&](int k, float val) { row[o0 + k] = __float2half_rn(val); });
    for (; o < A.n_input_pad; o++) row[o] = __float2half_rn(1.0f);
}


// runs the MLP for the warp's rows [row0, row0 + 16 * MT); buffers: bufA holds the input on entry; returns the
// buffer (and its stride) that holds the 16 outputs
template <int NN, int MT>
__device__ inline const __half* mlp_forward_warp(const MlpShape& s, const __half* sw, const int* soff, __half* bufA, int ldA, __half* bufB,
                                                 int ldB, int row0, int hidden_act, int* ld_out) {
    __half* in = bufA;
    int ld_in = ldA;
    __half* out = bufB;
    int ld_o = ldB;
    for (int l = 0; l < s.layers; l++) {
        const bool last = l == s.layers - 1;
        if (last) layer_forward<16, MT>(in, ld_in, s.w_cols[l], sw + soff[l], s.w_cols[l] + 8, out, ld_o, row0, false);
        else layer_forward<NN, MT>(in, ld_in, s.w_cols[l], sw + soff[l], s.w_cols[l] + 8, out, ld_o, row0, hidden_act == 1);
        __syncwarp();
        __half* t = in; in = out; out = t;
        const int tl = ld_in; ld_in = ld_o; ld_o = tl;
    }
    *ld_out = ld_in;
    return in;
}

// ---------------------------------------------------------------------------------------------------
// row helpers of the visible-row kernels. Row k of a warp's block belongs to lane k (lanes >= rows mirror it).

// raw encoder input e of the rows k = 0..NR-1 (row k: primitive shfl(i, k), valid when bit k of vmask is set), one
// lane per input, all loads issued before any is used
template <int NR>
__device__ inline void load_raw_rows(const Params& P, const AppearanceConfig& A, uint32_t i, uint32_t vmask, int e, float (&vals)[NR]) {
    const int F = A.feature_dim, nraw = F + (A.base_input ? 3 : 0);
#pragma unroll
    for (int k = 0; k < NR; k++) {
        const uint32_t ik = __shfl_sync(0xffffffffu, i, k);
        vals[k] = 0.0f;
        if (((vmask >> k) & 1u) && e < nraw) vals[k] = e < F ? P.residual[static_cast<size_t>(ik) * F + e] : P.base[3ull * ik + (e - F)];
    }
}

// moves vals[k + 1] to vals[k] (the rolled row loops read row k from vals[0])
template <int NR>
__device__ inline void rotate(float (&vals)[NR]) {
#pragma unroll
    for (int k = 0; k + 1 < NR; k++) vals[k] = vals[k + 1];
}

// encoded features of the warp's NR rows into buf[k * ld + column], one lane per raw input so every row is one
// coalesced load; invalid rows are skipped
template <int NR>
__device__ inline void encode_rows(const Params& P, const AppearanceConfig& A, uint32_t i, uint32_t vmask, __half* buf, int ld) {
    const int nraw = A.feature_dim + (A.base_input ? 3 : 0), nf = A.n_freq, per = nf > 0 ? 2 * nf : 1;
    const int lane = threadIdx.x & 31;
    for (int e0 = 0; e0 < nraw; e0 += 32) {
        const int e = e0 + lane;
        float vals[NR];
        load_raw_rows<NR>(P, A, i, vmask, e, vals);
#pragma unroll 1
        for (int k = 0; k < NR; k++) {
            const float val = vals[0];
            rotate<NR>(vals);
            if (!((vmask >> k) & 1u) || e >= nraw) continue;
            __half* row = buf + k * ld;
            if (nf == 0) {
                row[e] = __float2half_rn(val);
            } else {
                for (int f = 0; f < nf; f++) {
                    float sn, cs;
                    enc_sincos(octave(val, f), &sn, &cs);
                    *reinterpret_cast<__half2*>(row + e * per + 2 * f) = __floats2half2_rn(sn, cs);
                }
            }
        }
    }
}

// SH band inputs and padding ones of one row (the calling lane's), or an all-zero row for an invalid row
__device__ inline void direction_inputs(const AppearanceConfig& A, int deg, bool valid, f3 d, __half* row, int kin) {
    const int nraw = A.feature_dim + (A.base_input ? 3 : 0), per = A.n_freq > 0 ? 2 * A.n_freq : 1;
    if (!valid) {
        for (int o = 0; o < kin; o++) row[o] = __float2half_rn(0.0f);
        return;
    }
    const int o0 = nraw * per;
    int o = o0 + sh_band_values(A.sh_mask, deg, d, [&](int k, float val) { row[o0 + k] = __float2half_rn(val); });
    for (; o < kin; o++) row[o] = __float2half_rn(1.0f);
}

// feature (and base-input) gradients of the warp's NR rows from the loss-scaled fp32 input gradient rows gx;
// feature gradients go to O.residual, base-input gradients to base_in[k * 3 + c]
template <int NR>
__device__ inline void feature_grads(const Params& P, const AppearanceConfig& A, const GradOut& O, uint32_t i, uint32_t vmask, const float* gx,
                                     int ldg, float* base_in, int acc) {
    const int F = A.feature_dim, nraw = F + (A.base_input ? 3 : 0), nf = A.n_freq, per = nf > 0 ? 2 * nf : 1;
    const int lane = threadIdx.x & 31;
    const float inv = 1.0f / kLossScale;
    for (int e0 = 0; e0 < nraw; e0 += 32) {
        const int e = e0 + lane;
        float vals[NR], olds[NR];
        if (nf > 0) load_raw_rows<NR>(P, A, i, vmask, e, vals);
        if (acc) {  // the accumulated gradients, loaded up front so the row loop never waits on memory
#pragma unroll
            for (int k = 0; k < NR; k++) {
                const uint32_t ik = __shfl_sync(0xffffffffu, i, k);
                olds[k] = (((vmask >> k) & 1u) && e < F) ? O.residual[static_cast<size_t>(ik) * F + e] : 0.0f;
            }
        }
#pragma unroll 1
        for (int k = 0; k < NR; k++) {
            const float val = vals[0], old = olds[0];
            if (nf > 0) rotate<NR>(vals);
            if (acc) rotate<NR>(olds);
            const uint32_t ik = __shfl_sync(0xffffffffu, i, k);
            if (!((vmask >> k) & 1u) || e >= nraw) continue;
            const float* g = gx + k * ldg;
            float gv = 0.0f;
            if (nf == 0) gv = g[e];
            else
                for (int f = 0; f < nf; f++) {
                    float sn, cs;
                    enc_sincos(octave(val, f), &sn, &cs);
                    gv += static_cast<float>(1 << f) * (cs * g[e * per + 2 * f] - sn * g[e * per + 2 * f + 1]);
                }
            gv *= inv;
            if (e < F) {
                O.residual[static_cast<size_t>(ik) * F + e] = acc ? old + gv : gv;
            } else {
                base_in[k * 3 + (e - F)] = gv;
            }
        }
    }
}

// ---------------------------------------------------------------------------------------------------
// forward colour pass over the visible rows: the geometry pass already wrote the records (with the colour of a
// zero residual); this overwrites the colour of every visible primitive with the MLP's
__host__ __device__ inline int color_buf_halves(const MlpShape& s, int nn) {
    const int ldA = (s.kin > nn ? s.kin : nn) + 8, ldB = nn + 8;
    return 32 * (ldA + ldB);
}

template <int NN>
__global__ void __launch_bounds__(256) neural_color_kernel(Params P, AppearanceConfig A, View v, const uint32_t* __restrict__ vis, uint32_t n_rows,
                                                           Record* __restrict__ rec) {
    extern __shared__ __align__(16) unsigned char smem[];
    __shared__ MlpShape s_shape;
    __shared__ int s_soff[10];
    __shared__ int s_wh;
    if (threadIdx.x == 0) {
        s_shape = mlp_shape(A);
        s_wh = smem_weights_halves(s_shape, s_soff);
    }
    __syncthreads();
    const MlpShape& s = s_shape;  // uniform tables read from shared memory (no local-memory copies)
    const int* soff = s_soff;
    const int wh = s_wh;
    __half* sw = reinterpret_cast<__half*>(smem);
    const int ldA = (s.kin > NN ? s.kin : NN) + 8, ldB = NN + 8;
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5, nwarps = blockDim.x >> 5;
    __half* bufA = sw + ((wh + 7) & ~7) + warp * color_buf_halves(s, NN);
    __half* bufB = bufA + 32 * ldA;
    load_weights(s, P.mlp, sw, soff);
    __syncthreads();
    const int deg = min(v.degree, A.max_degree);
    const uint32_t n_tiles = (n_rows + 31) / 32, stride = gridDim.x * nwarps;
    for (uint32_t t = blockIdx.x * nwarps + warp; t < n_tiles; t += stride) {
        const uint32_t gi = t * 32 + lane;
        const bool valid = gi < n_rows;
        const uint32_t i = valid ? vis[gi] : 0u;
        const uint32_t vmask = __ballot_sync(0xffffffffu, valid);
        const f3 d = valid ? view_dir(v, ld3(P.means, i), nullptr) : mk3(0.0f, 0.0f, 1.0f);
        direction_inputs(A, deg, valid, d, bufA + lane * ldA, s.kin);
        encode_rows<32>(P, A, i, vmask, bufA, ldA);
        __syncwarp();
        int ldo;
        const __half* y = mlp_forward_warp<NN, 2>(s, sw, soff, bufA, ldA, bufB, ldB, 0, A.hidden_act, &ldo);
        if (valid) {
            const __half* yr = y + lane * ldo;
            const f3 res = residual_act3(A.res_act, mk3(__half2float(yr[0]), __half2float(yr[1]), __half2float(yr[2])));
            const f3 base = base_act3(A.base_act, ld3(P.base, i));
            f3 color = color_act3(A.color_act, base + res);
            if (!v.render_base) {
                const f3 bc = color_act3(A.color_act, base);
                color = mk3(fabsf(color.x - bc.x), fabsf(color.y - bc.y), fabsf(color.z - bc.z));
            }
            float* q2 = reinterpret_cast<float*>(rec + i) + 8;
            q2[0] = color.x;
            q2[1] = color.y;
            q2[2] = color.z;
        }
        __syncwarp();
    }
}

// ---------------------------------------------------------------------------------------------------
// backward

// dIn[row][0..K) = dOut[row][0..NOUT) . W (W: [NOUT][K]) for the warp's 16 * MT rows, 32 output columns at a
// time; masked by (act_in > 0) when relu, rounded to fp16 into `out` or stored as fp32 into `out32`. `out` may
// alias `act_in` (each element is read and written by the same lane).
template <int NOUT, int MT>
__device__ inline void layer_backward_data(const __half* dout, int ld_dout, const __half* W, int ld_w, int K, const __half* act_in, int ld_act,
                                           bool relu, __half* out, int ld_out, float* out32, int ld_out32, int row0) {
    const int lane = threadIdx.x & 31, g = lane >> 2, tq = lane & 3;
    for (int c0 = 0; c0 < K; c0 += 32) {
        const int ncols = min(32, K - c0);
        float acc[MT][4][4];
#pragma unroll
        for (int m = 0; m < MT; m++)
#pragma unroll
            for (int n = 0; n < 4; n++)
#pragma unroll
                for (int q = 0; q < 4; q++) acc[m][n][q] = 0.0f;
#pragma unroll
        for (int kk = 0; kk < NOUT; kk += 16) {
            uint32_t a[MT][4];
#pragma unroll
            for (int m = 0; m < MT; m++) ldsm_x4(a[m], dout + (row0 + m * 16 + (lane & 15)) * ld_dout + kk + (lane >> 4) * 8);
#pragma unroll
            for (int n = 0; n < 4; n += 2) {
                if (n * 8 >= ncols) break;
                uint32_t b[4];
                ldsm_x4_t(b, W + (kk + ((lane >> 3) & 1) * 8 + (lane & 7)) * ld_w + c0 + n * 8 + (lane >> 4) * 8);
#pragma unroll
                for (int m = 0; m < MT; m++) {
                    mma16816(acc[m][n], a[m], b[0], b[1]);
                    mma16816(acc[m][n + 1], a[m], b[2], b[3]);
                }
            }
        }
#pragma unroll
        for (int m = 0; m < MT; m++)
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
                if (l == s.layers - 1) layer_forward<16, 2>(in, ldi, s.w_cols[l], sw + L.soff[l], s.w_cols[l] + 8, Y, L.ldY, row0, false);
                else layer_forward<NN, 2>(in, ldi, s.w_cols[l], sw + L.soff[l], s.w_cols[l] + 8, H + l * kBwdRows * L.ldH, L.ldH, row0, A.hidden_act == 1);
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
                    if (s.w_rows[l] == 16) layer_backward_data<16, 2>(dcur, ld_cur, sw + L.soff[l], s.w_cols[l] + 8, s.w_cols[l], in, ldi, A.hidden_act == 1, dnext, L.ldD, nullptr, 0, row0);
                    else layer_backward_data<NN, 2>(dcur, ld_cur, sw + L.soff[l], s.w_cols[l] + 8, s.w_cols[l], in, ldi, A.hidden_act == 1, dnext, L.ldD, nullptr, 0, row0);
                    dcur = dnext;
                    ld_cur = L.ldD;
                    pp ^= 1;
                } else {
                    if (s.w_rows[0] == 16) layer_backward_data<16, 2>(dcur, ld_cur, sw + L.soff[0], s.w_cols[0] + 8, s.w_cols[0], nullptr, 0, false, nullptr, 0, GX, L.ldG, row0);
                    else layer_backward_data<NN, 2>(dcur, ld_cur, sw + L.soff[0], s.w_cols[0] + 8, s.w_cols[0], nullptr, 0, false, nullptr, 0, GX, L.ldG, row0);
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
                            enc_sincos(octave(val, f), &sn, &cs);
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

// ---------------------------------------------------------------------------------------------------
// backward over the visible rows (8 warps x 16 rows per batch, weight gradient in registers)

constexpr int kFastWarps = 8;
constexpr int kMaxTilesPerWarp = 8;

struct FastBwdLayout {
    int soff[10];
    int ldX, ldH, ldY, ldG;
    int tb[11];  // first 16x16 weight-gradient tile of each layer; tb[layers] = number of tiles
    size_t off_x, off_h, off_y, off_g, total;
};

__host__ __device__ inline FastBwdLayout fast_bwd_layout(const MlpShape& s) {
    FastBwdLayout L;
    const int wh = smem_weights_halves(s, L.soff);
    L.ldX = s.kin + 8;
    L.ldH = s.nn + 8;
    L.ldY = 16 + 8;
    L.ldG = s.kin + 4;
    size_t off = (static_cast<size_t>(wh) * 2 + 15) & ~static_cast<size_t>(15);
    L.off_x = off;
    off += static_cast<size_t>(kBwdRows) * L.ldX * 2;
    L.off_h = off;
    const size_t hbuf = static_cast<size_t>(kBwdRows) * L.ldH * 2;
    off += hbuf * (s.layers - 1);
    L.off_y = off;
    off += static_cast<size_t>(kBwdRows) * L.ldY * 2;
    // the fp32 input gradient overwrites buffers that are dead once the second layer's gradients are done: the hidden
    // buffers after the first and the output gradient (a network without hidden layers gets its own buffer)
    L.off_g = s.layers >= 3 ? L.off_h + hbuf : (s.layers == 2 ? L.off_y : off);
    const size_t g_end = L.off_g + static_cast<size_t>(kBwdRows) * L.ldG * 4;
    L.total = g_end > off ? g_end : off;
    L.tb[0] = 0;
    for (int l = 0; l < s.layers; l++) L.tb[l + 1] = L.tb[l] + (s.w_rows[l] / 16) * (s.w_cols[l] / 16);
    return L;
}

// dW tiles of layer l owned by this warp (tile t belongs to warp t % 8, register slot t / 8) += dOut^T . In over the
// batch's rows; the row loop is outside the tile loop so the tiles' mma chains interleave
template <int T>
__device__ inline void wgrad_tiles(float (&dw)[T][2][4], int t_begin, int t_end, int tiles_k, int warp, const __half* dout, int ld_dout,
                                   const __half* in, int ld_in) {
    const int lane = threadIdx.x & 31;
    int m0[T], n0[T];
    bool own[T];
#pragma unroll
    for (int j = 0; j < T; j++) {
        const int t = warp + kFastWarps * j;
        own[j] = t >= t_begin && t < t_end;
        const int lt = own[j] ? t - t_begin : 0;
        m0[j] = (lt / tiles_k) * 16;
        n0[j] = (lt % tiles_k) * 16;
    }
    for (int k0 = 0; k0 < kBwdRows; k0 += 16) {
#pragma unroll
        for (int j = 0; j < T; j++) {
            if (!own[j]) continue;
            uint32_t a[4], b[4];
            ldsm_x4_t(a, dout + (k0 + (lane >> 4) * 8 + (lane & 7)) * ld_dout + m0[j] + ((lane >> 3) & 1) * 8);
            ldsm_x4_t(b, in + (k0 + ((lane >> 3) & 1) * 8 + (lane & 7)) * ld_in + n0[j] + (lane >> 4) * 8);
            mma16816(dw[j][0], a, b[0], b[1]);
            mma16816(dw[j][1], a, b[2], b[3]);
        }
    }
}

template <int NN, int T>
__global__ void __launch_bounds__(kFastWarps * 32, 2) neural_bwd_vis_kernel(Params P, AppearanceConfig A, View v, const uint32_t* __restrict__ vis,
                                                                          uint32_t n_rows, const uint32_t* __restrict__ rank_of,
                                                                          const Record* __restrict__ sorted_rec,
                                                                          const GradRecord* __restrict__ grads, GradOut O) {
    extern __shared__ __align__(16) unsigned char smem[];
    __shared__ float s_base_in[kBwdRows * 3];
    __shared__ MlpShape s_shape;
    __shared__ FastBwdLayout s_layout;
    if (threadIdx.x == 0) {
        s_shape = mlp_shape(A);
        s_layout = fast_bwd_layout(s_shape);
    }
    __syncthreads();
    const MlpShape& s = s_shape;  // uniform tables read from shared memory (no local-memory copies)
    const FastBwdLayout& L = s_layout;
    __half* sw = reinterpret_cast<__half*>(smem);
    __half* X = reinterpret_cast<__half*>(smem + L.off_x);
    __half* H = reinterpret_cast<__half*>(smem + L.off_h);  // slot j: output of layer j (input of layer j + 1), later its gradient
    __half* Y = reinterpret_cast<__half*>(smem + L.off_y);  // outputs, then the scaled output gradient
    float* GX = reinterpret_cast<float*>(smem + L.off_g);   // loss-scaled input gradient
    load_weights(s, P.mlp, sw, L.soff);
    __syncthreads();
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    const int deg = min(v.degree, A.max_degree);
    const int acc_mode = O.accumulate;
    const int nraw = A.feature_dim + (A.base_input ? 3 : 0), per = A.n_freq > 0 ? 2 * A.n_freq : 1;
    const int sh_col = nraw * per;
    const int row = warp * 16 + (lane & 15);  // this lane's row in the batch (lanes 16..31 mirror 0..15)
    const bool row_lane = lane < 16;
    const size_t hslot = static_cast<size_t>(kBwdRows) * L.ldH;
    float dw[T][2][4];
#pragma unroll
    for (int j = 0; j < T; j++)
#pragma unroll
        for (int n = 0; n < 2; n++)
#pragma unroll
            for (int q = 0; q < 4; q++) dw[j][n][q] = 0.0f;
    const uint32_t n_batches = (n_rows + kBwdRows - 1) / kBwdRows;
    for (uint32_t b = blockIdx.x; b < n_batches; b += gridDim.x) {
        const uint32_t gi = b * kBwdRows + row;
        const bool valid = gi < n_rows;
        const uint32_t i = valid ? vis[gi] : 0u;
        const uint32_t r = valid ? rank_of[i] : 0u;
        const uint32_t vmask = __ballot_sync(0xffffffffu, valid) & 0xffffu;
        // inputs and recomputed forward of the warp's 16 rows
        f3 gpre = mk3(0.0f, 0.0f, 0.0f);
        if (row_lane) {
            f3 d = mk3(0.0f, 0.0f, 1.0f);
            if (valid) {
                const float4 q2 = sorted_rec[r].q2, g1 = grads[r].g1;
                gpre = mk3(g1.y, g1.z, g1.w) * mk3(color_act_grad_from_y(A.color_act, q2.x), color_act_grad_from_y(A.color_act, q2.y),
                                                   color_act_grad_from_y(A.color_act, q2.z));
                d = view_dir(v, ld3(P.means, i), nullptr);
            }
            direction_inputs(A, deg, valid, d, X + row * L.ldX, s.kin);
        }
        encode_rows<16>(P, A, i, vmask, X + warp * 16 * L.ldX, L.ldX);
        __syncwarp();
        for (int l = 0; l < s.layers; l++) {
            const __half* in = l == 0 ? X : H + (l - 1) * hslot;
            const int ldi = l == 0 ? L.ldX : L.ldH;
            if (l == s.layers - 1) layer_forward<16, 1>(in, ldi, s.w_cols[l], sw + L.soff[l], s.w_cols[l] + 8, Y, L.ldY, warp * 16, false);
            else layer_forward<NN, 1>(in, ldi, s.w_cols[l], sw + L.soff[l], s.w_cols[l] + 8, H + l * hslot, L.ldH, warp * 16, A.hidden_act == 1);
            __syncwarp();
        }
        if (row_lane) {
            __half* yr = Y + row * L.ldY;
            float dy[3] = {0.0f, 0.0f, 0.0f};
            if (valid) {
                const float gv[3] = {gpre.x, gpre.y, gpre.z};
                for (int c = 0; c < 3; c++) {
                    const float y = __half2float(yr[c]);
                    dy[c] = gv[c] * residual_act_grad_from_y(A.res_act, residual_act(A.res_act, y));
                }
            }
            for (int c = 0; c < 16; c++) yr[c] = __float2half_rn(c < 3 ? kLossScale * dy[c] : 0.0f);
        }
        __syncthreads();
        // layers last to first: weight gradient over all rows (shared), data gradient of the warp's rows
        for (int l = s.layers - 1; l >= 0; l--) {
            const __half* dout = l == s.layers - 1 ? Y : H + l * hslot;
            const int ldd = l == s.layers - 1 ? L.ldY : L.ldH;
            const __half* in = l == 0 ? X : H + (l - 1) * hslot;
            const int ldi = l == 0 ? L.ldX : L.ldH;
            wgrad_tiles<T>(dw, L.tb[l], L.tb[l + 1], s.w_cols[l] / 16, warp, dout, ldd, in, ldi);
            if (l > 0) {
                __syncthreads();  // every warp has read this layer's input before it is overwritten by its gradient
                __half* hin = H + (l - 1) * hslot;
                if (s.w_rows[l] == 16)
                    layer_backward_data<16, 1>(dout, ldd, sw + L.soff[l], s.w_cols[l] + 8, s.w_cols[l], hin, L.ldH, A.hidden_act == 1, hin, L.ldH,
                                               nullptr, 0, warp * 16);
                else
                    layer_backward_data<NN, 1>(dout, ldd, sw + L.soff[l], s.w_cols[l] + 8, s.w_cols[l], hin, L.ldH, A.hidden_act == 1, hin, L.ldH,
                                               nullptr, 0, warp * 16);
                __syncthreads();
            } else {
                if (s.w_rows[0] == 16)
                    layer_backward_data<16, 1>(dout, ldd, sw + L.soff[0], s.w_cols[0] + 8, s.w_cols[0], nullptr, 0, false, nullptr, 0, GX, L.ldG, warp * 16);
                else
                    layer_backward_data<NN, 1>(dout, ldd, sw + L.soff[0], s.w_cols[0] + 8, s.w_cols[0], nullptr, 0, false, nullptr, 0, GX, L.ldG, warp * 16);
                __syncwarp();
            }
        }
        feature_grads<16>(P, A, O, i, vmask, GX + warp * 16 * L.ldG, L.ldG, s_base_in + warp * 16 * 3, acc_mode);
        __syncwarp();
        if (row_lane && valid) {
            // base colours (through the colour and, with base input, the MLP) and the view-direction part of the
            // mean gradient; the geometry chain rule follows in neural_geometry_bwd_kernel
            const float4 q2 = sorted_rec[r].q2, g1 = grads[r].g1;
            const f3 gp = mk3(g1.y, g1.z, g1.w) * mk3(color_act_grad_from_y(A.color_act, q2.x), color_act_grad_from_y(A.color_act, q2.y),
                                                       color_act_grad_from_y(A.color_act, q2.z));
            f3 gbase = mk3(0.0f, 0.0f, 0.0f);
            if (v.render_base) {
                const f3 bb = ld3(P.base, i);
                gbase = mk3(base_act_grad(A.base_act, bb.x), base_act_grad(A.base_act, bb.y), base_act_grad(A.base_act, bb.z)) * gp;
            }
            if (A.base_input) {
                const float* bi = s_base_in + row * 3;
                gbase.x += bi[0];
                gbase.y += bi[1];
                gbase.z += bi[2];
            }
            put3n(O.base, i, gbase, acc_mode);
            f3 gmean_color = mk3(0.0f, 0.0f, 0.0f);
            if (A.dir_grad) {
                float rn = 1.0f;
                const f3 d = view_dir(v, ld3(P.means, i), &rn);
                // direction gradient from the SH inputs' gradient, unscaled afterwards (scaling by 2^-7 is exact)
                const f3 gd = (1.0f / kLossScale) * sh_band_grad(A.sh_mask, deg, d, GX + row * L.ldG + sh_col);
                gmean_color = rn * (gd - dot3(gd, d) * d);
            }
            put3n(O.means, i, gmean_color, acc_mode);
        }
        __syncthreads();  // the next batch overwrites buffers other warps may still read
    }
    // flush this warp's weight-gradient tiles (unscaled)
    const float inv = 1.0f / kLossScale;
    const int g = lane >> 2, tq = lane & 3;
#pragma unroll
    for (int j = 0; j < T; j++) {
        const int t = warp + kFastWarps * j;
        if (t >= L.tb[s.layers]) continue;
        int l = 0;
        while (t >= L.tb[l + 1]) l++;
        const int lt = t - L.tb[l], tk = s.w_cols[l] / 16, cols = s.w_cols[l];
        const int m0 = (lt / tk) * 16, n0 = (lt % tk) * 16;
        float* base = O.mlp + s.w_off[l];
#pragma unroll
        for (int n = 0; n < 2; n++) {
            const int rr = m0 + g, c = n0 + n * 8 + tq * 2;
            atomicAdd(base + rr * cols + c, dw[j][n][0] * inv);
            atomicAdd(base + rr * cols + c + 1, dw[j][n][1] * inv);
            atomicAdd(base + (rr + 8) * cols + c, dw[j][n][2] * inv);
            atomicAdd(base + (rr + 8) * cols + c + 1, dw[j][n][3] * inv);
        }
    }
}

// geometry chain rule of the visible primitives (one thread per row, rows in primitive order): mean (added to the
// view-direction part written by the MLP backward), log-scale, rotation and opacity gradients, densification
__global__ void __launch_bounds__(256, 3) neural_geometry_bwd_kernel(Params P, View v, const uint32_t* __restrict__ vis, uint32_t n_rows,
                                                                  const uint32_t* __restrict__ rank_of, const Record* __restrict__ sorted_rec,
                                                                  const GradRecord* __restrict__ grads, GradOut O) {
    const uint32_t gi = blockIdx.x * blockDim.x + threadIdx.x;
    if (gi >= n_rows) return;
    const uint32_t i = vis[gi];
    const uint32_t r = rank_of[i];
    const GradRecord g = grads[r];
    const Record rq = sorted_rec[r];
    const f3 m = ld3(P.means, i);
    float gmx, gmy, gca, gcb, gcc, g_opacity;
    blend_sums_to_grads(g, rq, v.proper_aa, gmx, gmy, gca, gcb, gcc, g_opacity);
    const f3 gmean = geometry_backward(P, v, i, m, gmx, gmy, gca, gcb, gcc, g_opacity, O);
    if (O.densification != nullptr && O.densification_rows == 3) {
        const float nx = 0.5f * (g.g2.y * static_cast<float>(v.width)), ny = 0.5f * (g.g2.z * static_cast<float>(v.height));
        O.densification[2ull * P.n + i] += sqrtf(nx * nx + ny * ny);
    }
    put1(O.opacities, i, g_opacity, O.accumulate);
    put3n(O.means, i, gmean, 1);
}

// The geometry chain rule of the visible rows ahead of the warp-specialised MLP backward (tc_bwd_ws_kernel), which
// also hands that kernel each row's inputs through the activation store's row block (TcRowLayout): the two fp16 chunks
// of SH inputs, the loss-scaled output gradient chunk (from the colour pass's stored raw outputs) and the primitive
// index, 1 / distance and view direction; the base-colour gradient is written here. Same values as tc_bwd_kernel
// computes (the same functions, compiled with the same flags). This kernel writes the mean gradient first; the MLP
// backward adds its direction part.
__global__ void __launch_bounds__(256, 4) neural_geometry_rows_kernel(Params P, AppearanceConfig A, View v, const uint32_t* __restrict__ vis,
                                                                   uint32_t n_rows, const uint32_t* __restrict__ rank_of,
                                                                   const Record* __restrict__ sorted_rec, const GradRecord* __restrict__ grads,
                                                                   GradOut O, TcRowLayout L) {
    const uint32_t gi = blockIdx.x * blockDim.x + threadIdx.x;
    if (gi >= n_rows) return;
    const uint32_t i = vis[gi];
    const uint32_t r = rank_of[i];
    const GradRecord g = grads[r];
    const Record rq = sorted_rec[r];
    const f3 m = ld3(P.means, i);
    float gmx, gmy, gca, gcb, gcc, g_opacity;
    blend_sums_to_grads(g, rq, v.proper_aa, gmx, gmy, gca, gcb, gcc, g_opacity);
    const f3 gmean = geometry_backward(P, v, i, m, gmx, gmy, gca, gcb, gcc, g_opacity, O);
    if (O.densification != nullptr && O.densification_rows == 3) {
        const float nx = 0.5f * (g.g2.y * static_cast<float>(v.width)), ny = 0.5f * (g.g2.z * static_cast<float>(v.height));
        O.densification[2ull * P.n + i] += sqrtf(nx * nx + ny * ny);
    }
    put1(O.opacities, i, g_opacity, O.accumulate);
    put3n(O.means, i, gmean, O.accumulate);
    // colour-activation gradient and the base-colour gradient
    const f3 gpre = mk3(g.g1.y, g.g1.z, g.g1.w) * mk3(color_act_grad_from_y(A.color_act, rq.q2.x), color_act_grad_from_y(A.color_act, rq.q2.y),
                                                      color_act_grad_from_y(A.color_act, rq.q2.z));
    f3 gbase = mk3(0.0f, 0.0f, 0.0f);
    if (v.render_base) {
        const f3 bb = ld3(P.base, i);
        gbase = mk3(base_act_grad(A.base_act, bb.x), base_act_grad(A.base_act, bb.y), base_act_grad(A.base_act, bb.z)) * gpre;
    }
    put3n(O.base, i, gbase, O.accumulate);
    // the MLP backward's row inputs
    unsigned char* const tile = P.mlp_act + static_cast<size_t>(gi / 128) * L.tile_bytes;
    const uint32_t row = gi % 128;
    const uint2 yo = *reinterpret_cast<const uint2*>(tile + L.outputs_off + row * 8);
    const float yh[3] = {__low2float(*reinterpret_cast<const __half2*>(&yo.x)), __high2float(*reinterpret_cast<const __half2*>(&yo.x)),
                         __low2float(*reinterpret_cast<const __half2*>(&yo.y))};
    const float gv[3] = {gpre.x, gpre.y, gpre.z};
    float dy[3];
    for (int c = 0; c < 3; c++) dy[c] = gv[c] * residual_act_grad_from_y(A.res_act, residual_act(A.res_act, yh[c]));
    float rn = 1.0f;
    const f3 dir = view_dir(v, m, &rn);
    float sh[16];
    sh_band_values(15, min(v.degree, A.max_degree), dir, [&](int k, float val) { sh[k] = val; });
    auto h2 = [](float lo, float hi) {
        const __half2 h = __floats2half2_rn(lo, hi);
        return *reinterpret_cast<const uint32_t*>(&h);
    };
    uint4* const out = reinterpret_cast<uint4*>(tile + L.rows_off + row * kTcRowDataBytes);
    out[0] = make_uint4(h2(sh[0], sh[1]), h2(sh[2], sh[3]), h2(sh[4], sh[5]), h2(sh[6], sh[7]));
    out[1] = make_uint4(h2(sh[8], sh[9]), h2(sh[10], sh[11]), h2(sh[12], sh[13]), h2(sh[14], sh[15]));
    out[2] = make_uint4(h2(kMlpLossScale * dy[0], kMlpLossScale * dy[1]), h2(kMlpLossScale * dy[2], 0.0f), 0u, 0u);
    out[3] = make_uint4(i, __float_as_uint(rn), __float_as_uint(dir.x), __float_as_uint(dir.y));
    out[4] = make_uint4(__float_as_uint(dir.z), 0u, 0u, 0u);
}

// backward of a view rendered at appearance degree 0 (the MLP is not evaluated, the residual is zero): base-colour
// gradients of the visible rows; features and the view-direction part of the mean gradient are zero
__global__ void __launch_bounds__(256) neural_base_bwd_kernel(Params P, AppearanceConfig A, View v, const uint32_t* __restrict__ vis, uint32_t n_rows,
                                                              const uint32_t* __restrict__ rank_of, const Record* __restrict__ sorted_rec,
                                                              const GradRecord* __restrict__ grads, GradOut O) {
    const uint32_t gi = blockIdx.x * blockDim.x + threadIdx.x;
    if (gi >= n_rows) return;
    const uint32_t i = vis[gi];
    const uint32_t r = rank_of[i];
    const float4 q2 = sorted_rec[r].q2, g1 = grads[r].g1;
    const f3 gp = mk3(g1.y, g1.z, g1.w) * mk3(color_act_grad_from_y(A.color_act, q2.x), color_act_grad_from_y(A.color_act, q2.y),
                                               color_act_grad_from_y(A.color_act, q2.z));
    f3 gbase = mk3(0.0f, 0.0f, 0.0f);
    if (v.render_base) {
        const f3 bb = ld3(P.base, i);
        gbase = mk3(base_act_grad(A.base_act, bb.x), base_act_grad(A.base_act, bb.y), base_act_grad(A.base_act, bb.z)) * gp;
    }
    put3n(O.base, i, gbase, O.accumulate);
    if (!O.accumulate) {
        put3n(O.means, i, mk3(0.0f, 0.0f, 0.0f), 0);
        for (int j = 0; j < A.feature_dim; j++) O.residual[static_cast<size_t>(i) * A.feature_dim + j] = 0.0f;
    }
}

// zero gradients of the primitives outside the view (overwrite mode of the visible-row backward); one thread per
// primitive; vec4 bit 0: feature rows 16-byte aligned, bit 1: rotation rows 16-byte aligned (16-byte stores)
// Zero gradients of the first view (no accumulation): every per-Gaussian gradient array is cleared as a whole before
// the view's kernels store the visible rows' values (or add to them), so the rows no view touches end at zero. Plain
// memsets stream at full bandwidth, where clearing only the untouched rows took one scattered store per value.
cudaError_t zero_gradients(const GradOut& O, uint32_t n, int F, cudaStream_t st) {
    const size_t rows = n;
    const struct { float* p; size_t floats; } arrays[] = {{O.means, 3 * rows}, {O.scales, 3 * rows}, {O.rotations, 4 * rows},
                                                          {O.opacities, rows}, {O.base, 3 * rows}, {O.residual, rows * static_cast<size_t>(F)}};
    for (const auto& a : arrays) {
        if (!a.p || !a.floats) continue;
        const cudaError_t e = cudaMemsetAsync(a.p, 0, a.floats * sizeof(float), st);
        if (e != cudaSuccess) return e;
    }
    return cudaSuccess;
}

int sm_count() {
    int dev = 0, sms = 148;
    cudaGetDevice(&dev);
    cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
    return sms;
}

size_t color_smem_bytes(const AppearanceConfig& A, int warps) {
    const MlpShape s = mlp_shape(A);
    const int wh = smem_weights_halves(s, nullptr);
    return static_cast<size_t>((wh + 7) & ~7) * 2 + static_cast<size_t>(warps) * color_buf_halves(s, s.nn) * 2;
}

constexpr size_t kSmemLimit = 227 * 1024;

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

cudaError_t launch_neural_color(const Params& P, const AppearanceConfig& A, const View& v, const uint32_t* vis, uint32_t n_visible, Record* rec,
                                cudaStream_t st) {
    if (n_visible == 0 || std::min(v.degree, A.max_degree) <= 0) return cudaSuccess;
    if (tc_mlp_supported(A)) return launch_tc_color(P, A, v, vis, n_visible, rec, st);
    int warps = 8;
    while (warps > 1 && color_smem_bytes(A, warps) > kSmemLimit) warps >>= 1;
    const size_t smem = color_smem_bytes(A, warps);
    if (smem > kSmemLimit) return cudaErrorInvalidConfiguration;
    const int threads = warps * 32;
    const uint32_t n_tiles = (n_visible + 31) / 32, n_blocks = (n_tiles + warps - 1) / warps;
    int grid = 0;
    cudaError_t e = cudaSuccess;
    switch (A.n_neurons) {
        case 16: e = launch_persistent(neural_color_kernel<16>, smem, threads, n_blocks, &grid); if (!e) neural_color_kernel<16><<<grid, threads, smem, st>>>(P, A, v, vis, n_visible, rec); break;
        case 32: e = launch_persistent(neural_color_kernel<32>, smem, threads, n_blocks, &grid); if (!e) neural_color_kernel<32><<<grid, threads, smem, st>>>(P, A, v, vis, n_visible, rec); break;
        case 64: e = launch_persistent(neural_color_kernel<64>, smem, threads, n_blocks, &grid); if (!e) neural_color_kernel<64><<<grid, threads, smem, st>>>(P, A, v, vis, n_visible, rec); break;
        default: return cudaErrorInvalidValue;
    }
    if (e != cudaSuccess) return e;
    return cudaGetLastError();
}

namespace {

template <int NN, int T>
cudaError_t run_vis_bwd(const Params& P, const AppearanceConfig& A, const View& v, const uint32_t* vis, uint32_t n_visible, const uint32_t* rank_of,
                        const Record* sorted_rec, const GradRecord* grads, const GradOut& O, size_t smem, cudaStream_t st) {
    int grid = 0;
    const uint32_t n_batches = (n_visible + kBwdRows - 1) / kBwdRows;
    cudaError_t e = launch_persistent(neural_bwd_vis_kernel<NN, T>, smem, kFastWarps * 32, n_batches, &grid);
    if (e != cudaSuccess) return e;
    neural_bwd_vis_kernel<NN, T><<<grid, kFastWarps * 32, smem, st>>>(P, A, v, vis, n_visible, rank_of, sorted_rec, grads, O);
    e = cudaGetLastError();
    if (e != cudaSuccess) return e;
    neural_geometry_bwd_kernel<<<(n_visible + 255) / 256, 256, 0, st>>>(P, v, vis, n_visible, rank_of, sorted_rec, grads, O);
    return cudaGetLastError();
}

template <int NN>
cudaError_t run_vis_bwd_t(int T, const Params& P, const AppearanceConfig& A, const View& v, const uint32_t* vis, uint32_t n_visible,
                          const uint32_t* rank_of, const Record* sorted_rec, const GradRecord* grads, const GradOut& O, size_t smem, cudaStream_t st) {
    switch (T) {
        case 2: return run_vis_bwd<NN, 2>(P, A, v, vis, n_visible, rank_of, sorted_rec, grads, O, smem, st);
        case 3: return run_vis_bwd<NN, 3>(P, A, v, vis, n_visible, rank_of, sorted_rec, grads, O, smem, st);
        case 5: return run_vis_bwd<NN, 5>(P, A, v, vis, n_visible, rank_of, sorted_rec, grads, O, smem, st);
        default: return run_vis_bwd<NN, 8>(P, A, v, vis, n_visible, rank_of, sorted_rec, grads, O, smem, st);
    }
}

}  // namespace

cudaError_t launch_preprocess_bwd_neural(const Params& P, const AppearanceConfig& A, const View& v, const uint32_t* rank_of,
                                         const Record* sorted_rec, const GradRecord* grads, const GradOut& O, const uint32_t* vis,
                                         uint32_t n_visible, cudaStream_t st) {
    if (P.n == 0) return cudaSuccess;
    if (!O.accumulate) {
        cudaError_t e = cudaMemsetAsync(O.mlp, 0, static_cast<size_t>(A.n_params) * sizeof(float), st);
        if (e != cudaSuccess) return e;
    }
    if (std::min(v.degree, A.max_degree) <= 0) {
        if (!O.accumulate) {
            cudaError_t e = zero_gradients(O, P.n, A.feature_dim, st);
            if (e != cudaSuccess) return e;
        }
        if (n_visible > 0) {
            neural_base_bwd_kernel<<<(n_visible + 255) / 256, 256, 0, st>>>(P, A, v, vis, n_visible, rank_of, sorted_rec, grads, O);
            neural_geometry_bwd_kernel<<<(n_visible + 255) / 256, 256, 0, st>>>(P, v, vis, n_visible, rank_of, sorted_rec, grads, O);
        }
        return cudaGetLastError();
    }
    const MlpShape s = mlp_shape(A);
    const FastBwdLayout FL = fast_bwd_layout(s);
    const int n_tiles = FL.tb[s.layers];
    const size_t fast_smem = FL.total;
    const bool fast = tc_mlp_supported(A) ||
                      (n_tiles <= kFastWarps * kMaxTilesPerWarp && fast_smem + kBwdRows * 3 * sizeof(float) <= kSmemLimit);
    if (fast) {
        if (!O.accumulate) {
            cudaError_t e = zero_gradients(O, P.n, A.feature_dim, st);
            if (e != cudaSuccess) return e;
        }
        if (n_visible == 0) return cudaSuccess;
        if (tc_mlp_supported(A)) {
            TcRowLayout L;
            if (tc_ws_layout(P, A, O, &L)) {  // warp-specialised MLP backward: the geometry pass first hands it the row inputs
                neural_geometry_rows_kernel<<<(n_visible + 255) / 256, 256, 0, st>>>(P, A, v, vis, n_visible, rank_of, sorted_rec, grads, O, L);
                cudaError_t e = cudaGetLastError();
                if (e != cudaSuccess) return e;
                return launch_tc_backward(P, A, v, vis, n_visible, rank_of, sorted_rec, grads, O, st);
            }
            cudaError_t e = launch_tc_backward(P, A, v, vis, n_visible, rank_of, sorted_rec, grads, O, st);
            if (e != cudaSuccess) return e;
            neural_geometry_bwd_kernel<<<(n_visible + 255) / 256, 256, 0, st>>>(P, v, vis, n_visible, rank_of, sorted_rec, grads, O);
            return cudaGetLastError();
        }
        const int per_warp = (n_tiles + kFastWarps - 1) / kFastWarps;
        const int T = per_warp <= 2 ? 2 : (per_warp <= 3 ? 3 : (per_warp <= 5 ? 5 : 8));
        switch (A.n_neurons) {
            case 16: return run_vis_bwd_t<16>(T, P, A, v, vis, n_visible, rank_of, sorted_rec, grads, O, fast_smem, st);
            case 32: return run_vis_bwd_t<32>(T, P, A, v, vis, n_visible, rank_of, sorted_rec, grads, O, fast_smem, st);
            case 64: return run_vis_bwd_t<64>(T, P, A, v, vis, n_visible, rank_of, sorted_rec, grads, O, fast_smem, st);
            default: return cudaErrorInvalidValue;
        }
    }
    // general path: every primitive, weight gradient in shared memory
    const uint32_t n_chunks = (P.n + kBwdRows - 1) / kBwdRows;
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
    if (tc_mlp_supported(A)) return tc_mlp_smem_bytes(A);
    const size_t b = neural_bwd_layout(mlp_shape(A)).total, f = color_smem_bytes(A, 1);
    return b > f ? b : f;
}

}  // namespace fgs
