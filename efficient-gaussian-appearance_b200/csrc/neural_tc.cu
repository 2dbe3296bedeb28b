// Neural appearance MLP on the sm_100a tensor cores (tcgen05 + TMEM); see tc.cuh for the operand layouts.
//
// Semantics as in neural.cu (appearance_neural.cuh:10-407 of the reference: encoding, SH inputs, fp16 network
// without biases, loss scale 128 in the backward). Design: one CTA of 256 threads handles tiles of 128 visible
// rows, two threads per row (warps w and w + 4 read the same TMEM lane quarter, each taking half of the columns).
// Per layer one thread issues the K/16 MMAs (M = 128 rows, N = layer width, fp16 operands from shared memory in the
// canonical layouts, fp32 accumulator in TMEM) and commits them to an mbarrier; the threads read their row from
// TMEM, apply the activation, round to fp16 and store the next layer's operand. In training the colour pass also
// writes every hidden activation and the raw outputs of a tile to an activation store, which the backward copies
// back into its shared slots (cp.async, one tile ahead) instead of recomputing the forward. The backward issues,
// per layer, the data-gradient MMAs (into the layer accumulator) and the weight-gradient MMAs (M = 64, reduction
// over the tile's rows) into TMEM accumulators that persist over every tile the CTA processes; they are read out
// and added to the weight gradient once per CTA. Hidden gradients overwrite their activations in place after the
// MMAs that read them completed. Used for 64-wide networks with at least one hidden layer (neural.cu keeps the
// other shapes).
//
// This file also holds the tensor-core self-test behind fgs_tc_selftest: three small GEMMs covering every operand
// orientation the MLP kernels use (forward: A and B K-major; data gradient: B MN-major; weight gradient: M = 64,
// A and B MN-major, accumulated over two passes), checked exactly on the host.
#include <cuda_fp16.h>

#include <cstdint>
#include <mutex>
#include <vector>

#include "launch.h"
#include "neural_common.cuh"
#include "tc.cuh"

namespace fgs {

namespace {

constexpr int kSelfA = 128 * 32, kSelfB = 64 * 32, kSelfC = 128 * 64;  // fp16 elements

__host__ __device__ inline float self_a(int r, int k) { return static_cast<float>((r * 7 + k * 3) % 17 - 8) * 0.125f; }
__host__ __device__ inline float self_b(int n, int k) { return static_cast<float>((n * 5 + k) % 13 - 6) * 0.125f; }
__host__ __device__ inline float self_c(int r, int c) { return static_cast<float>((r * 3 + c * 5) % 11 - 5) * 0.125f; }

__global__ void __launch_bounds__(128) tc_selftest_kernel(float* out) {
    __shared__ __align__(128) __half sa[kSelfA];
    __shared__ __align__(128) __half sb[kSelfB];
    __shared__ __align__(128) __half sc[kSelfC];
    __shared__ uint64_t bar;
    __shared__ uint32_t tbase;
    const int t = threadIdx.x, warp = t >> 5, lane = t & 31;
    // operands in the canonical K-major layouts (A 128x32, B 64x32, C 128x64)
    for (int k = 0; k < 32; k++) sa[tc::kmajor_offset(t, k, 32) / 2] = __float2half_rn(self_a(t, k));
    if (t < 64)
        for (int k = 0; k < 32; k++) sb[tc::kmajor_offset(t, k, 32) / 2] = __float2half_rn(self_b(t, k));
    for (int c = 0; c < 64; c++) sc[tc::kmajor_offset(t, c, 64) / 2] = __float2half_rn(self_c(t, c));
    if (warp == 0) tc::tmem_alloc(&tbase, 128);
    if (t == 0) tc::mbar_init(&bar, 1);
    tc::fence_smem_to_async();
    tc::fence_before_sync();
    __syncthreads();
    tc::fence_after_sync();
    const uint32_t tb = tbase;
    const uint32_t a = tc::smem_addr(sa), b = tc::smem_addr(sb), c = tc::smem_addr(sc);
    if (t == 0) {
        // D1[128x64] = A . B^T (both K-major), columns 0..63
        for (int ks = 0; ks < 2; ks++)
            tc::mma(tb, tc::desc(a + ks * 256, 128, 512), tc::desc(b + ks * 256, 128, 512), tc::idesc(128, 64, 0, 0), ks > 0);
        // D2[128x32] = C . B (B read MN-major: N = B's columns, K = B's rows), columns 64..95
        for (int ks = 0; ks < 4; ks++)
            tc::mma(tb + 64, tc::desc(c + ks * 256, 128, 1024), tc::desc(b + ks * 1024, 512, 128), tc::idesc(128, 32, 0, 1), ks > 0);
        // D3[64x32] = 2 * C^T . A (both MN-major, reduction over the 128 rows, M = 64), columns 96..127
        for (int rep = 0; rep < 2; rep++)
            for (int ks = 0; ks < 8; ks++)
                tc::mma(tb + 96, tc::desc(c + ks * 2048, 1024, 128), tc::desc(a + ks * 1024, 512, 128), tc::idesc(64, 32, 1, 1),
                        (rep > 0 || ks > 0) ? 1u : 0u);
        tc::commit(&bar);
    }
    __syncwarp();
    bool ok = tc::mbar_wait(&bar, 0);
    if (!ok) ok = tc::mbar_wait(&bar, 0);  // the MMAs must not be in flight when the columns are freed
    tc::fence_after_sync();
    if (ok) {
        const uint32_t lane_base = static_cast<uint32_t>(warp * 32) << 16;
        float v[16];
        for (int c0 = 0; c0 < 64; c0 += 16) {
            tc::ld16(tb + lane_base + c0, v);
            for (int i = 0; i < 16; i++) out[t * 64 + c0 + i] = v[i];
        }
        for (int c0 = 0; c0 < 32; c0 += 16) {
            tc::ld16(tb + lane_base + 64 + c0, v);
            for (int i = 0; i < 16; i++) out[8192 + t * 32 + c0 + i] = v[i];
        }
        for (int c0 = 0; c0 < 32; c0 += 16) {
            tc::ld16(tb + lane_base + 96 + c0, v);
            if (lane < 16)  // M = 64: row m lives in lane (m % 16) + 32 * (m / 16)
                for (int i = 0; i < 16; i++) out[8192 + 4096 + (warp * 16 + lane) * 32 + c0 + i] = v[i];
        }
    }
    if (t == 0) out[kTcSelftestStatus] = ok ? 0.0f : 1.0f;
    tc::fence_before_sync();
    __syncthreads();
    tc::fence_after_sync();
    if (warp == 0) tc::tmem_dealloc(tb, 128);
}

}  // namespace

cudaError_t tc_selftest(float* scratch, int* mismatches, cudaStream_t s) {
    tc_selftest_kernel<<<1, 128, 0, s>>>(scratch);
    cudaError_t e = cudaGetLastError();
    if (e != cudaSuccess) return e;
    std::vector<float> h(kTcSelftestFloats);
    e = cudaMemcpyAsync(h.data(), scratch, h.size() * sizeof(float), cudaMemcpyDeviceToHost, s);
    if (e != cudaSuccess) return e;
    e = cudaStreamSynchronize(s);
    if (e != cudaSuccess) return e;
    int bad = h[kTcSelftestStatus] != 0.0f ? 1 : 0;
    for (int r = 0; r < 128; r++)
        for (int n = 0; n < 64; n++) {
            double ref = 0.0;
            for (int k = 0; k < 32; k++) ref += static_cast<double>(self_a(r, k)) * self_b(n, k);
            bad += h[r * 64 + n] != static_cast<float>(ref);
        }
    for (int r = 0; r < 128; r++)
        for (int n = 0; n < 32; n++) {
            double ref = 0.0;
            for (int k = 0; k < 64; k++) ref += static_cast<double>(self_c(r, k)) * self_b(k, n);
            bad += h[8192 + r * 32 + n] != static_cast<float>(ref);
        }
    for (int m = 0; m < 64; m++)
        for (int n = 0; n < 32; n++) {
            double ref = 0.0;
            for (int k = 0; k < 128; k++) ref += static_cast<double>(self_c(k, m)) * self_a(k, n);
            bad += h[8192 + 4096 + m * 32 + n] != static_cast<float>(2.0 * ref);
        }
    *mismatches = bad;
    return cudaSuccess;
}


// ---------------------------------------------------------------------------------------------------
// MLP on tcgen05: 256 threads per CTA, two threads per tile row (warps w and w + 4 read the same TMEM lane quarter);
// each half of a row's columns belongs to one of the two threads

namespace {

constexpr int kTcRows = 128;
constexpr int kTcThreads = 256;
constexpr int kTcWidth = 64;
constexpr int kTcMaxLayers = 8;
constexpr int kPrefetchFeatures = 32;  // rows of up to 32 latent floats are prefetched into registers (16 per thread)
// Activation store of the colour pass (training): per 128-row tile, every hidden activation as the 16 KB K-major fp16
// block the backward's shared slot holds, then the fp16-rounded raw outputs (4 halves per row, the last one zero), then
// the row block the geometry pass of the warp-specialised backward fills (TcRowLayout).
constexpr uint32_t kTcActLayerBytes = kTcRows * kTcWidth * 2;
constexpr uint32_t kTcActOutBytes = kTcRows * 8;

// one MLP configuration laid out for the tensor-core kernels
struct TcPlan {
    int layers, kin, backward;
    int rows[kTcMaxLayers], cols[kTcMaxLayers];  // W_l is rows x cols (out x in)
    uint32_t w_off[kTcMaxLayers];                // flat fp32 weight offsets
    uint32_t w_smem[kTcMaxLayers];               // fp16 K-major copies (bytes into dynamic shared memory)
    uint32_t x_smem, h_smem, y_smem, trig_smem, smem_bytes;
    int h_slots;                                 // activation buffers: 1 (forward, rewritten in place) or layers - 1
    uint32_t wg_col[kTcMaxLayers];               // TMEM column of each layer's weight-gradient accumulator
    uint32_t tmem_cols;                          // allocated TMEM columns (power of two)
    uint32_t act_tile_bytes;                     // activation store bytes per tile
};

__device__ __forceinline__ uint32_t h_slot(const TcPlan& p, int j) { return p.h_smem + static_cast<uint32_t>(j % p.h_slots) * (kTcRows * kTcWidth * 2); }

__device__ inline void st_shared_v4(uint32_t addr, uint32_t a, uint32_t b, uint32_t c, uint32_t d) {
    asm volatile("st.shared.v4.b32 [%0], {%1, %2, %3, %4};" ::"r"(addr), "r"(a), "r"(b), "r"(c), "r"(d) : "memory");
}
__device__ inline uint4 ld_shared_v4(uint32_t addr) {
    uint4 v;
    asm volatile("ld.shared.v4.b32 {%0, %1, %2, %3}, [%4];" : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w) : "r"(addr) : "memory");
    return v;
}
__device__ inline uint32_t pack2(float lo, float hi) {
    const __half2 h = __floats2half2_rn(lo, hi);
    return *reinterpret_cast<const uint32_t*>(&h);
}
__device__ inline float2 unpack2(uint32_t w) {
    const __half2 h = *reinterpret_cast<const __half2*>(&w);
    return __half22float2(h);
}
// 16-byte global -> shared copies that complete in the background without registers. cp_async_wait makes a thread's
// copies visible to that thread; the proxy fence and barrier of sync_tile then publish them to the tensor cores like
// ordinary shared stores.
__device__ inline void cp_async16(uint32_t dst, const void* src) {
    asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"(dst), "l"(src) : "memory");
}
__device__ inline void cp_async_commit() { asm volatile("cp.async.commit_group;" ::: "memory"); }
__device__ inline void cp_async_wait() { asm volatile("cp.async.wait_all;" ::: "memory"); }

// fp32 master weights -> fp16 K-major copies in shared memory
__device__ inline void stage_weights_tc(const TcPlan& p, const float* __restrict__ w, unsigned char* smem) {
    for (int l = 0; l < p.layers; l++) {
        const int rows = p.rows[l], cols = p.cols[l];
        __half* dst = reinterpret_cast<__half*>(smem + p.w_smem[l]);
        for (int e = threadIdx.x; e < rows * cols; e += blockDim.x) {
            const int r = e / cols, c = e - r * cols;
            dst[tc::kmajor_offset(r, c, cols) / 2] = __float2half_rn(w[p.w_off[l] + e]);
        }
    }
}

// collects fp16 values in input order and stores them 8 at a time (16 bytes) into a K-major row from `chunk` on
struct RowWriter {
    uint32_t base;  // shared address of element (row, 0)
    int chunk = 0, fill = 0;
    uint32_t w0 = 0, w1 = 0, w2 = 0, w3 = 0;
    __device__ void push(float v) {
        const uint32_t h = __half_as_ushort(__float2half_rn(v));
        w0 = (w0 >> 16) | (w1 << 16);
        w1 = (w1 >> 16) | (w2 << 16);
        w2 = (w2 >> 16) | (w3 << 16);
        w3 = (w3 >> 16) | (h << 16);
        if (++fill == 8) {
            st_shared_v4(base + chunk * 128, w0, w1, w2, w3);
            chunk++;
            fill = 0;
        }
    }
    __device__ void push8(uint32_t a, uint32_t b, uint32_t c, uint32_t d) {  // at a chunk boundary
        st_shared_v4(base + chunk * 128, a, b, c, d);
        chunk++;
    }
};

// the fast encoding path: one octave, features in groups of 8, 16-byte aligned rows, at most 32 features (split in
// halves of groups of 4 between a row's two threads)
__device__ inline bool fast_features(const Params& P, const AppearanceConfig& A) {
    return A.n_freq == 1 && A.feature_dim % 8 == 0 && A.feature_dim <= kPrefetchFeatures && (reinterpret_cast<uintptr_t>(P.residual) & 15u) == 0;
}

// per-row inputs of a tile, loaded one tile ahead so their latency hides behind the previous tile's MMAs
struct RowData {
    uint32_t i, r;
    bool valid;
    f3 mean;
    float4 f[kPrefetchFeatures / 8];  // this thread's half of the latent features (fast path)
    float4 q2, g1;                    // colour of the record and its blend gradient sums (backward)
    f3 base;                          // base colour parameters
    uint2 y;                          // stored fp16 raw outputs (backward with an activation store)
};

// The prefetch of a row runs in three stages placed in different phases of the current tile, because each stage's
// addresses come from the loads of the one before: a thread that issued a stage's loads never waits on them inside
// the same phase (in particular not before issuing the MMAs).
// stage 1: primitive index of tile row gi
__device__ inline void load_row_index(const uint32_t* __restrict__ vis, uint32_t n_rows, uint32_t gi, RowData& d) {
    d.valid = gi < n_rows;
    d.i = d.valid ? vis[gi] : 0u;
}
// stage 2: the primitive's parameters (and, backward, its depth rank)
__device__ inline void load_row_params(const Params& P, const AppearanceConfig& A, bool fast, int half, const uint32_t* __restrict__ rank_of,
                                       RowData& d) {
    if (!d.valid) return;
    d.mean = ld3(P.means, d.i);
    d.base = ld3(P.base, d.i);
    const int F = A.feature_dim;
    if (fast) {
        const float4* src = reinterpret_cast<const float4*>(P.residual + static_cast<size_t>(d.i) * F + half * (F / 2));
#pragma unroll
        for (int q = 0; q < kPrefetchFeatures / 8; q++)
            if (8 * q < F) d.f[q] = src[q];
    }
    if (rank_of) d.r = rank_of[d.i];
}
// stage 3 (backward): the record colour and blend gradient sums at the depth rank
__device__ inline void load_row_rank(const Record* __restrict__ sorted_rec, const GradRecord* __restrict__ grads, RowData& d) {
    if (!d.valid) return;
    d.q2 = sorted_rec[d.r].q2;
    d.g1 = grads[d.r].g1;
}

// this thread's part of the MLP input row: with the fast path each thread encodes its half of the features
// (sin, cos per feature), the second also the base inputs, SH inputs and padding; otherwise the first thread writes
// the whole row. With `trig` the fp32 sine and cosine of every feature are kept at trig[column * 128 + row].
__device__ inline void write_input_row(const Params& P, const AppearanceConfig& A, const View& v, int deg, const RowData& d, bool fast, int half,
                                       uint32_t row_base, int kin, float* trig, int row) {
    const int F = A.feature_dim, nf = A.n_freq;
    if (!d.valid) {
        if (half == 0)
            for (int c = 0; c < kin; c += 8) st_shared_v4(row_base + (c / 8) * 128, 0u, 0u, 0u, 0u);
        return;
    }
    if (!fast && half == 1) return;
    RowWriter w{row_base};
    const uint32_t i = d.i;
    const float* feat = P.residual + static_cast<size_t>(i) * F;
    int j0 = 0;
    if (fast) {  // 4 features = 8 encoded columns per store
        const int jb = half * (F / 2);
        w.chunk = jb / 4;
        // the prefetch holds this half's F/2 floats as F/8 float4 values
#pragma unroll
        for (int q = 0; q < kPrefetchFeatures / 8; q++) {
            if (4 * q >= F / 2) break;
            const float4 x = d.f[q];
            float s0, c0, s1, c1, s2, c2, s3, c3;
            enc_sincos(x.x, &s0, &c0);
            enc_sincos(x.y, &s1, &c1);
            enc_sincos(x.z, &s2, &c2);
            enc_sincos(x.w, &s3, &c3);
            w.push8(pack2(s0, c0), pack2(s1, c1), pack2(s2, c2), pack2(s3, c3));
            if (trig) {
                float* tq = trig + (2 * (jb + 4 * q)) * kTcRows + row;
                tq[0] = s0; tq[kTcRows] = c0; tq[2 * kTcRows] = s1; tq[3 * kTcRows] = c1;
                tq[4 * kTcRows] = s2; tq[5 * kTcRows] = c2; tq[6 * kTcRows] = s3; tq[7 * kTcRows] = c3;
            }
        }
        if (half == 0) return;
        j0 = F;
        w.chunk = F / 4;
    }
    const int nraw = F + (A.base_input ? 3 : 0);
    for (int j = j0; j < nraw; j++) {
        const float val = j < F ? feat[j] : P.base[3ull * i + (j - F)];
        if (nf == 0) {
            w.push(val);
        } else {
            for (int f = 0; f < nf; f++) {
                float sn, cs;
                enc_sincos(octave(val, f), &sn, &cs);
                w.push(sn);
                w.push(cs);
            }
        }
    }
    const f3 dir = view_dir(v, d.mean, nullptr);
    const int nsh = sh_band_values(A.sh_mask, deg, dir, [&](int, float val) { w.push(val); });
    for (int c = nraw * (nf > 0 ? 2 * nf : 1) + nsh; c < kin; c++) w.push(1.0f);
}

// forward MMAs of layer l for the whole tile into the layer accumulator (TMEM columns 0..)
__device__ inline void issue_forward(const TcPlan& p, uint32_t sbase, uint32_t tb, int l) {
    const uint32_t in = sbase + (l == 0 ? p.x_smem : h_slot(p, l - 1));
    const uint32_t K = p.cols[l], sbo = 16u * K, w = sbase + p.w_smem[l];
    const uint32_t id = tc::idesc(128, p.rows[l], 0, 0);
    const uint64_t a = tc::desc(in, 128, sbo), b = tc::desc(w, 128, sbo);
    for (uint32_t ks = 0; ks < K / 16; ks++) tc::mma(tb, tc::desc_advance(a, ks * 256), tc::desc_advance(b, ks * 256), id, ks > 0);
}

// hidden-layer epilogue, this thread's 32 columns: accumulator -> activation -> fp16 K-major row of the slot (and,
// with g_row, the same 64 bytes at the same offsets of the activation store)
__device__ inline void hidden_epilogue(uint32_t t_addr, uint32_t row_base, int half, bool relu, unsigned char* g_row) {
    float a[32];
    tc::ld32(t_addr + 32 * half, a);
#pragma unroll
    for (int q = 0; q < 4; q++) {
        float* x = a + 8 * q;
        if (relu)
#pragma unroll
            for (int k = 0; k < 8; k++) x[k] = fmaxf(x[k], 0.0f);
        const uint4 h = make_uint4(pack2(x[0], x[1]), pack2(x[2], x[3]), pack2(x[4], x[5]), pack2(x[6], x[7]));
        st_shared_v4(row_base + (4 * half + q) * 128, h.x, h.y, h.z, h.w);
        if (g_row) *reinterpret_cast<uint4*>(g_row + (4 * half + q) * 128) = h;
    }
}

// loss-scaled output gradient of a row (fp16, K-major, 16 columns) from the fp16-rounded raw outputs yh
__device__ inline void write_output_grad(const TcPlan& p, const AppearanceConfig& A, uint32_t sbase, int row, bool valid, f3 gpre,
                                         const float (&yh)[3]) {
    float dy[3] = {0.0f, 0.0f, 0.0f};
    if (valid) {
        const float gv[3] = {gpre.x, gpre.y, gpre.z};
        for (int c = 0; c < 3; c++) dy[c] = gv[c] * residual_act_grad_from_y(A.res_act, residual_act(A.res_act, yh[c]));
    }
    const uint32_t yrow = sbase + p.y_smem + tc::kmajor_offset(row, 0, 16);
    st_shared_v4(yrow, pack2(kLossScale * dy[0], kLossScale * dy[1]), pack2(kLossScale * dy[2], 0.0f), 0u, 0u);
    st_shared_v4(yrow + 128, 0u, 0u, 0u, 0u);
}

// the activation store of tile `tl`
__device__ inline const unsigned char* act_tile(const TcPlan& p, const unsigned char* act, uint32_t tl) {
    return act + static_cast<size_t>(tl) * p.act_tile_bytes;
}
// stored hidden activation j of tile `tl` into its shared slot (this thread's half of its row), asynchronously
__device__ inline void fetch_activation(const TcPlan& p, uint32_t sbase, const unsigned char* act, uint32_t tl, int j, int row, int half) {
    const uint32_t off = tc::kmajor_offset(row, 0, kTcWidth);
    const unsigned char* src = act_tile(p, act, tl) + static_cast<size_t>(j) * kTcActLayerBytes + off;
    const uint32_t dst = sbase + h_slot(p, j) + off;
#pragma unroll
    for (int q = 0; q < 4; q++) cp_async16(dst + (4 * half + q) * 128, src + (4 * half + q) * 128);
}
// stored raw outputs of row `row` of tile `tl`
__device__ inline uint2 load_outputs(const TcPlan& p, const unsigned char* act, uint32_t tl, int row) {
    return *reinterpret_cast<const uint2*>(act_tile(p, act, tl) + static_cast<size_t>(p.layers - 1) * kTcActLayerBytes + row * 8);
}

// data-gradient epilogue of a hidden layer, this thread's 32 columns: dL/d(activation), masked by the ReLU of the
// stored activation, written over that activation (fp16, in place)
__device__ inline void hidden_grad_epilogue(uint32_t t_addr, uint32_t row_base, int half, bool relu) {
    float a[32];
    tc::ld32(t_addr + 32 * half, a);
#pragma unroll
    for (int q = 0; q < 4; q++) {
        float* x = a + 8 * q;
        const uint32_t addr = row_base + (4 * half + q) * 128;
        if (relu) {
            const uint4 h = ld_shared_v4(addr);
            const uint32_t hw[4] = {h.x, h.y, h.z, h.w};
#pragma unroll
            for (int k = 0; k < 4; k++) {
                const float2 hv = unpack2(hw[k]);
                if (!(hv.x > 0.0f)) x[2 * k] = 0.0f;
                if (!(hv.y > 0.0f)) x[2 * k + 1] = 0.0f;
            }
        }
        st_shared_v4(addr, pack2(x[0], x[1]), pack2(x[2], x[3]), pack2(x[4], x[5]), pack2(x[6], x[7]));
    }
}

// bounded wait on the tile's mbarrier; flips the parity
__device__ inline bool wait_mma(uint64_t* bar, uint32_t& phase) {
    const bool ok = tc::mbar_wait(bar, phase);
    phase ^= 1u;
    return ok;
}

// every thread waits for the committed MMAs; the CTA agrees on the outcome (true: completed) and orders the
// following TMEM reads after the wait
__device__ inline bool wait_all(uint64_t* bar, uint32_t& phase) {
    const bool ok = wait_mma(bar, phase);
    const bool any_failed = __syncthreads_or(!ok) != 0;
    tc::fence_after_sync();
    return !any_failed;
}

__device__ inline void sync_tile() {
    tc::fence_smem_to_async();
    tc::fence_before_sync();
    __syncthreads();
    tc::fence_after_sync();
}

__device__ int g_tc_timeout;  // set when an mbarrier wait ran out (the kernel then stops issuing work)

__global__ void __launch_bounds__(kTcThreads, 3) tc_color_kernel(Params P, AppearanceConfig A, View v, const uint32_t* __restrict__ vis,
                                                                 uint32_t n_rows, Record* __restrict__ rec, const __grid_constant__ TcPlan plan) {
    extern __shared__ __align__(128) unsigned char smem[];
    __shared__ uint64_t bar;
    __shared__ uint32_t tbase;
    const int t = threadIdx.x, warp = t >> 5, half = t >> 7, row = t & (kTcRows - 1);
    stage_weights_tc(plan, P.mlp, smem);
    if (warp == 0) tc::tmem_alloc(&tbase, plan.tmem_cols);
    if (t == 0) tc::mbar_init(&bar, 1);
    sync_tile();
    bool alive = true;
    const uint32_t tb = tbase, sbase = tc::smem_addr(smem);
    const int wu = tc::warp_id_uniform();                 // warp-uniform operands for the elected MMA issue
    const uint32_t tbu = __shfl_sync(0xffffffffu, tb, 0);
    const uint32_t t_row = tb + (static_cast<uint32_t>((warp & 3) * 32) << 16);
    const int deg = min(v.degree, A.max_degree);
    uint32_t phase = 0;
    const uint32_t n_tiles = (n_rows + kTcRows - 1) / kTcRows;
    const bool fast = fast_features(P, A);
    const uint32_t x_row = sbase + plan.x_smem + tc::kmajor_offset(row, 0, plan.kin);
    const uint32_t h_row = tc::kmajor_offset(row, 0, kTcWidth);
    RowData cur, nxt;
    if (blockIdx.x < n_tiles) {
        load_row_index(vis, n_rows, blockIdx.x * kTcRows + row, cur);
        load_row_params(P, A, fast, half, nullptr, cur);
    }
    for (uint32_t tile = blockIdx.x; tile < n_tiles; tile += gridDim.x) {
        const uint32_t next = tile + gridDim.x;
        const bool more = next < n_tiles;
        unsigned char* const act = P.mlp_act ? P.mlp_act + static_cast<size_t>(tile) * plan.act_tile_bytes : nullptr;
        if (more) load_row_index(vis, n_rows, next * kTcRows + row, nxt);
        write_input_row(P, A, v, deg, cur, fast, half, x_row, plan.kin, nullptr, row);
        sync_tile();
        for (int l = 0; l < plan.layers; l++) {
            if (wu == 0) {
                if (tc::elect_one()) {
                    issue_forward(plan, sbase, tbu, l);
                    tc::commit(&bar);
                }
                __syncwarp();
            }
            if (l == 0 && more) load_row_params(P, A, fast, half, nullptr, nxt);
            alive = wait_all(&bar, phase);
            if (!alive) break;
            if (l < plan.layers - 1) {
                hidden_epilogue(t_row, sbase + h_slot(plan, l) + h_row, half, A.hidden_act == 1,
                                act ? act + static_cast<size_t>(l) * kTcActLayerBytes + h_row : nullptr);
            } else if (half == 0) {  // whole warps: the TMEM load is warp-collective
                float y[16];
                tc::ld16(t_row, y);
                if (act)
                    *reinterpret_cast<uint2*>(act + static_cast<size_t>(l) * kTcActLayerBytes + row * 8) =
                        make_uint2(pack2(y[0], y[1]), pack2(y[2], 0.0f));
                if (cur.valid) {
                    const f3 res = residual_act3(A.res_act, mk3(__half2float(__float2half_rn(y[0])), __half2float(__float2half_rn(y[1])),
                                                                 __half2float(__float2half_rn(y[2]))));
                    const f3 base = base_act3(A.base_act, cur.base);
                    f3 color = color_act3(A.color_act, base + res);
                    if (!v.render_base) {
                        const f3 bc = color_act3(A.color_act, base);
                        color = mk3(fabsf(color.x - bc.x), fabsf(color.y - bc.y), fabsf(color.z - bc.z));
                    }
                    float* q2 = reinterpret_cast<float*>(rec + cur.i) + 8;
                    q2[0] = color.x;
                    q2[1] = color.y;
                    q2[2] = color.z;
                }
            }
            sync_tile();
        }
        if (!alive) break;
        cur = nxt;
    }
    if (!alive) {
        tc::mbar_wait(&bar, phase ^ 1u);  // the timed-out MMAs must not be in flight when the columns are freed
        if (t == 0) atomicExch(&g_tc_timeout, 1);
    }
    tc::fence_before_sync();
    __syncthreads();
    tc::fence_after_sync();
    if (warp == 0) tc::tmem_dealloc(tb, plan.tmem_cols);
}

// Input gradient of a row (loss-scaled dL/dinput in TMEM columns 0..kin) -> feature, base-input and direction
// gradients. Fast path: each thread handles its half of the features (sine and cosine from `trig` when kept, else
// recomputed); with 32 features one TMEM load brings a thread's 32 columns. The remaining columns (base inputs, SH
// inputs, padding): with the full SH input (all four bands) and no base input, the first thread takes the SH columns
// (direction gradient) and the second the base colour; otherwise the second thread walks them. Without the fast
// path the first thread walks every column. Returns which of the row's remaining gradients this thread holds:
// kOwnDir (gdir, means) and / or kOwnBase (gbase_in, base colour).
constexpr int kOwnDir = 1, kOwnBase = 2;

__device__ inline int input_grad_row(const Params& P, const AppearanceConfig& A, const GradOut& O, uint32_t t_row, const RowData& d, bool fast,
                                     int half, const float* trig, int row, int kin, int deg, f3 dir, f3& gbase_in, f3& gdir,
                                     float* stage_row) {
    const float inv = 1.0f / kLossScale;
    const int F = A.feature_dim, nf = A.n_freq, per = nf > 0 ? 2 * nf : 1, nraw = F + (A.base_input ? 3 : 0);
    const int enc = nraw * per;
    const bool valid = d.valid;
    const uint32_t i = d.i;
    const int acc = O.accumulate;
    const float* feat = P.residual + static_cast<size_t>(i) * F;
    float* gout = O.residual + static_cast<size_t>(i) * F;
    int c = 0;
    if (fast) {
        const int jb = half * (F / 2);
        // features j .. j + 3 from their 8 columns g[0..7]
        auto group = [&](int j, const float* g) {
            float sn[4], cs[4];
            if (trig) {
#pragma unroll
                for (int k = 0; k < 4; k++) {
                    sn[k] = trig[(2 * j + 2 * k) * kTcRows + row];
                    cs[k] = trig[(2 * j + 2 * k + 1) * kTcRows + row];
                }
            } else {
                const float4 x = *reinterpret_cast<const float4*>(feat + j);
                enc_sincos(x.x, &sn[0], &cs[0]);
                enc_sincos(x.y, &sn[1], &cs[1]);
                enc_sincos(x.z, &sn[2], &cs[2]);
                enc_sincos(x.w, &sn[3], &cs[3]);
            }
            float gv[4];
#pragma unroll
            for (int k = 0; k < 4; k++) gv[k] = (cs[k] * g[2 * k] - sn[k] * g[2 * k + 1]) * inv;
            const float4 o = make_float4(gv[0], gv[1], gv[2], gv[3]);
            if (stage_row) {  // written out by whole rows afterwards (store_staged_features)
                *reinterpret_cast<float4*>(stage_row + j) = o;
                return;
            }
            float4* dst = reinterpret_cast<float4*>(gout + j);
            if (acc) atomicAdd(dst, o);  // one addition per element and launch (deterministic)
            else *dst = o;
        };
        if (F == 32) {
            float g[32];
            tc::ld32(t_row + 2 * jb, g);
            if (valid)
#pragma unroll
                for (int q = 0; q < 4; q++) group(jb + 4 * q, g + 8 * q);
        } else {
#pragma unroll
            for (int q = 0; q < kPrefetchFeatures / 8; q++) {
                if (4 * q >= F / 2) break;
                float g[8];
                tc::ld8(t_row + 2 * (jb + 4 * q), g);
                if (valid) group(jb + 4 * q, g);
            }
        }
        if (!A.base_input && A.sh_mask == 15) {  // SH columns 2F .. 2F + 15 (2F is a multiple of 16)
            gbase_in = mk3(0.0f, 0.0f, 0.0f);
            if (half == 1) return kOwnBase;
            float g[16];
            tc::ld16(t_row + 2 * F, g);
            gdir = inv * sh_band_grad(15, deg, dir, g);
            return kOwnDir;
        }
        if (half == 0) return 0;
        c = 2 * F;
    } else if (half == 1) {
        return 0;
    }
    // remaining columns in order: encoded inputs (feature j, octave f, sin then cos), SH inputs, padding
    int nsh = 0;
    for (int l = 0; l <= 3; l++)
        if (A.sh_mask & (1 << l)) nsh += 2 * l + 1;
    int j = c / per, q = c - j * per;
    float val = 0.0f, gacc = 0.0f, sn = 0.0f, cs = 0.0f, g_even = 0.0f;
    float gsh[16];
    float gb[3] = {0.0f, 0.0f, 0.0f};
    float g[8];
    for (int c0 = c & ~7; c0 < kin; c0 += 8) {
        tc::ld8(t_row + c0, g);
        if (!valid) continue;
#pragma unroll
        for (int k = 0; k < 8; k++) {
            const int col = c0 + k;
            if (col < c) continue;
            if (col < enc) {
                if (q == 0) {
                    val = j < F ? feat[j] : P.base[3ull * i + (j - F)];
                    gacc = 0.0f;
                }
                if (nf == 0) {
                    gacc = g[k];
                } else {
                    const int f = q >> 1;
                    if ((q & 1) == 0) {
                        enc_sincos(octave(val, f), &sn, &cs);
                        g_even = g[k];
                    } else {
                        gacc += static_cast<float>(1 << f) * (cs * g_even - sn * g[k]);
                    }
                }
                if (++q == per) {
                    const float gv = gacc * inv;
                    if (j < F) {
                        if (acc) atomicAdd(gout + j, gv);
                        else gout[j] = gv;
                    }
                    else gb[j - F] = gv;
                    j++;
                    q = 0;
                }
            } else if (col < enc + nsh) {
                gsh[col - enc] = g[k];
            }
        }
    }
    gbase_in = mk3(gb[0], gb[1], gb[2]);
    // direction gradient from the SH inputs' gradient, unscaled afterwards (scaling by 2^-7 is exact)
    gdir = inv * sh_band_grad(A.sh_mask, deg, dir, gsh);
    return kOwnDir | kOwnBase;
}

// Feature gradients of 32-feature rows leave through shared memory: each row's two threads put their halves into a
// staging block (rows of 36 floats, so the 16-byte stores of a warp's rows fall in different banks), and the CTA then
// writes whole 128-byte rows, four per warp instruction, instead of 32 rows 16 bytes each. The staging block lives in
// the input operand slot, free between the layer-0 MMAs and the next tile's input row.
constexpr int kStageStride = 36;
constexpr uint32_t kStageBytes = kTcRows * kStageStride * 4;
__device__ inline bool stage_features(const TcPlan& p, bool fast, const AppearanceConfig& A) {
    return fast && A.feature_dim == 32 && static_cast<uint32_t>(p.kin) * kTcRows * 2 >= kStageBytes + kTcRows * 4;
}
__device__ inline void store_staged_features(const GradOut& O, const float* stage, const uint32_t* rows_prim, int t) {
#pragma unroll
    for (int m = 0; m < 4; m++) {
        const int c = t + kTcThreads * m, r = c >> 3, q = c & 7;
        const uint32_t pi = rows_prim[r];
        if (pi == 0xffffffffu) continue;
        const float4 v = *reinterpret_cast<const float4*>(stage + r * kStageStride + 4 * q);
        float4* dst = reinterpret_cast<float4*>(O.residual + static_cast<size_t>(pi) * 32 + 4 * q);
        if (O.accumulate) atomicAdd(dst, v);  // one addition per element and launch (deterministic)
        else *dst = v;
    }
}

// backward MMAs of layer l: weight gradient (M = 64, accumulated in TMEM) and data gradient (layer accumulator)
__device__ inline void issue_backward(const TcPlan& p, uint32_t sbase, uint32_t tb, int l, bool wg_accumulate) {
    const int last = p.layers - 1;
    const uint32_t in = sbase + (l == 0 ? p.x_smem : h_slot(p, l - 1));
    const uint32_t K = p.cols[l], in_row_group = 16u * K;  // bytes per 8 rows of the layer input
    const uint32_t dout = sbase + (l == last ? p.y_smem : h_slot(p, l));
    const uint32_t R = p.rows[l], dout_row_group = 16u * R;
    const uint32_t w = sbase + p.w_smem[l];
    const uint32_t dw = tb + p.wg_col[l];
    const uint64_t in_mn = tc::desc(in, in_row_group, 128), dout_mn = tc::desc(dout, dout_row_group, 128);
    if (l == last) {  // dW^T [in x out] += In^T . dOut (M = input width 64, N = 16)
        const uint32_t id = tc::idesc(64, R, 1, 1);
        for (uint32_t ks = 0; ks < kTcRows / 16; ks++)
            tc::mma(dw, tc::desc_advance(in_mn, ks * 2 * in_row_group), tc::desc_advance(dout_mn, ks * 2 * dout_row_group), id,
                    (wg_accumulate || ks > 0) ? 1u : 0u);
    } else {  // dW [out x in] += dOut^T . In (M = 64 outputs, N = input width)
        const uint32_t id = tc::idesc(64, K, 1, 1);
        for (uint32_t ks = 0; ks < kTcRows / 16; ks++)
            tc::mma(dw, tc::desc_advance(dout_mn, ks * 2 * dout_row_group), tc::desc_advance(in_mn, ks * 2 * in_row_group), id,
                    (wg_accumulate || ks > 0) ? 1u : 0u);
    }
    // dIn [rows x in] = dOut . W (B = W read MN-major: N = inputs, K = outputs)
    const uint32_t id = tc::idesc(128, K, 0, 1);
    const uint64_t dk = tc::desc(dout, 128, dout_row_group), wmn = tc::desc(w, in_row_group, 128);
    for (uint32_t ks = 0; ks < R / 16; ks++)
        tc::mma(tb, tc::desc_advance(dk, ks * 256), tc::desc_advance(wmn, ks * 2 * in_row_group), id, ks > 0);
}

__global__ void __launch_bounds__(kTcThreads, 2) tc_bwd_kernel(Params P, AppearanceConfig A, View v, const uint32_t* __restrict__ vis,
                                                               uint32_t n_rows, const uint32_t* __restrict__ rank_of,
                                                               const Record* __restrict__ sorted_rec, const GradRecord* __restrict__ grads, GradOut O,
                                                               const __grid_constant__ TcPlan plan) {
    extern __shared__ __align__(128) unsigned char smem[];
    __shared__ uint64_t bar;
    __shared__ uint32_t tbase;
    const int t = threadIdx.x, warp = t >> 5, lane = t & 31, half = t >> 7, row = t & (kTcRows - 1);
    stage_weights_tc(plan, P.mlp, smem);
    if (warp == 0) tc::tmem_alloc(&tbase, plan.tmem_cols);
    if (t == 0) tc::mbar_init(&bar, 1);
    sync_tile();
    bool alive = true;
    const uint32_t tb = tbase, sbase = tc::smem_addr(smem);
    const int wu = tc::warp_id_uniform();                 // warp-uniform operands for the elected MMA issue
    const uint32_t tbu = __shfl_sync(0xffffffffu, tb, 0);
    const uint32_t t_row = tb + (static_cast<uint32_t>((warp & 3) * 32) << 16);
    const int deg = min(v.degree, A.max_degree);
    const int last = plan.layers - 1;
    const bool relu = A.hidden_act == 1;
    uint32_t phase = 0;
    bool wg_started = false;
    const uint32_t n_tiles = (n_rows + kTcRows - 1) / kTcRows;
    const bool fast = fast_features(P, A) && (reinterpret_cast<uintptr_t>(O.residual) & 15u) == 0;  // 16-byte gradient stores
    float* trig = fast && plan.trig_smem ? reinterpret_cast<float*>(smem + plan.trig_smem) : nullptr;
    const uint32_t x_row = sbase + plan.x_smem + tc::kmajor_offset(row, 0, plan.kin);
    const bool staged = stage_features(plan, fast, A);
    float* const fstage = reinterpret_cast<float*>(smem + plan.x_smem);
    uint32_t* const fstage_prim = reinterpret_cast<uint32_t*>(smem + plan.x_smem + kStageBytes);
    // With an activation store (the colour pass's hidden activations and raw outputs) the forward is not recomputed:
    // a tile's activations are copied into their slots while the previous tile finishes (slot j as soon as the MMAs
    // of layer j, its last reader, completed) and its raw outputs come with the row prefetch.
    const unsigned char* const act = P.mlp_act;
    RowData cur, nxt;
    if (blockIdx.x < n_tiles) {
        load_row_index(vis, n_rows, blockIdx.x * kTcRows + row, cur);
        if (act) {
            cur.y = load_outputs(plan, act, blockIdx.x, row);
            for (int j = 0; j < last; j++) fetch_activation(plan, sbase, act, blockIdx.x, j, row, half);
            cp_async_commit();
        }
        load_row_params(P, A, fast, half, rank_of, cur);
        load_row_rank(sorted_rec, grads, cur);
    }
    for (uint32_t tile = blockIdx.x; tile < n_tiles && alive; tile += gridDim.x) {
        const uint32_t next = tile + gridDim.x;
        const bool more = next < n_tiles;
        if (more) {
            load_row_index(vis, n_rows, next * kTcRows + row, nxt);
            if (act) nxt.y = load_outputs(plan, act, next, row);
        }
        const bool valid = cur.valid;
        const uint32_t i = cur.i;
        f3 gpre = mk3(0.0f, 0.0f, 0.0f);
        if (valid)
            gpre = mk3(cur.g1.y, cur.g1.z, cur.g1.w) * mk3(color_act_grad_from_y(A.color_act, cur.q2.x), color_act_grad_from_y(A.color_act, cur.q2.y),
                                                           color_act_grad_from_y(A.color_act, cur.q2.z));
        write_input_row(P, A, v, deg, cur, fast, half, x_row, plan.kin, trig, row);
        if (act) {
            if (half == 0) {
                const float2 y01 = unpack2(cur.y.x);
                const float yh[3] = {y01.x, y01.y, unpack2(cur.y.y).x};
                write_output_grad(plan, A, sbase, row, valid, gpre, yh);
            }
            cp_async_wait();  // this tile's activation slots
        }
        sync_tile();
        // recomputed forward (no activation store); the last layer's outputs become the scaled output gradient
        for (int l = 0; l < plan.layers && alive && !act; l++) {
            if (wu == 0) {
                if (tc::elect_one()) {
                    issue_forward(plan, sbase, tbu, l);
                    tc::commit(&bar);
                }
                __syncwarp();
            }
            if (l == 0 && more) load_row_params(P, A, fast, half, rank_of, nxt);
            alive = wait_all(&bar, phase);
            if (!alive) break;
            if (l < last) {
                hidden_epilogue(t_row, sbase + h_slot(plan, l) + tc::kmajor_offset(row, 0, kTcWidth), half, relu, nullptr);
            } else if (half == 0) {
                float y[16];
                tc::ld16(t_row, y);
                const float yh[3] = {__half2float(__float2half_rn(y[0])), __half2float(__float2half_rn(y[1])), __half2float(__float2half_rn(y[2]))};
                write_output_grad(plan, A, sbase, row, valid, gpre, yh);
            }
            sync_tile();
        }
        // layers last to first
        for (int l = last; l >= 0 && alive; l--) {
            if (wu == 0) {
                if (tc::elect_one()) {
                    issue_backward(plan, sbase, tbu, l, wg_started);
                    tc::commit(&bar);
                }
                __syncwarp();
            }
            if (more) {
                if (!act) {
                    if (l == last) load_row_rank(sorted_rec, grads, nxt);
                } else if (l == last) {
                    load_row_params(P, A, fast, half, rank_of, nxt);
                } else if (l == last - 1) {
                    load_row_rank(sorted_rec, grads, nxt);
                }
            }
            alive = wait_all(&bar, phase);
            if (!alive) break;
            if (act && more && l < last) {  // slot l is free: the next tile's activation l
                fetch_activation(plan, sbase, act, next, l, row, half);
                cp_async_commit();
            }
            if (l > 0) {
                hidden_grad_epilogue(t_row, sbase + h_slot(plan, l - 1) + tc::kmajor_offset(row, 0, kTcWidth), half, relu);
                sync_tile();
            }
        }
        if (!alive) break;
        wg_started = true;
        // input gradient (layer-0 data gradient) -> feature, base and direction gradients
        float rn = 1.0f;
        const f3 d = valid ? view_dir(v, cur.mean, &rn) : mk3(0.0f, 0.0f, 1.0f);
        f3 gbase_in = mk3(0.0f, 0.0f, 0.0f), gd = mk3(0.0f, 0.0f, 0.0f);
        const int own = input_grad_row(P, A, O, t_row, cur, fast, half, trig, row, plan.kin, deg, d, gbase_in, gd,
                                       staged ? fstage + row * kStageStride : nullptr);
        if (staged) {
            if (half == 0) fstage_prim[row] = valid ? i : 0xffffffffu;
            __syncthreads();
            store_staged_features(O, fstage, fstage_prim, t);
        }
        if ((own & kOwnBase) && valid) {
            f3 gbase = mk3(0.0f, 0.0f, 0.0f);
            if (v.render_base) {
                const f3 bb = cur.base;
                gbase = mk3(base_act_grad(A.base_act, bb.x), base_act_grad(A.base_act, bb.y), base_act_grad(A.base_act, bb.z)) * gpre;
            }
            if (A.base_input) gbase = gbase + gbase_in;
            put3n(O.base, i, gbase, O.accumulate);
        }
        if ((own & kOwnDir) && valid) {
            const f3 gmean_color = A.dir_grad ? rn * (gd - dot3(gd, d) * d) : mk3(0.0f, 0.0f, 0.0f);
            put3n(O.means, i, gmean_color, O.accumulate);
        }
        sync_tile();
        cur = nxt;
    }
    // weight gradients: M = 64 accumulators (row m in lane (m % 16) + 32 (m / 16)), unscaled and added once per CTA;
    // 16-column chunks alternate between the two halves
    if (wg_started && alive) {
        const float inv = 1.0f / kLossScale;
        const int m = (warp & 3) * 16 + lane;
        for (int l = 0; l < plan.layers; l++) {
            const int ncol = l == last ? plan.rows[l] : plan.cols[l];
            for (int c0 = 16 * half; c0 < ncol; c0 += 32) {
                float a[16];
                tc::ld16(t_row + plan.wg_col[l] + c0, a);
                if (lane < 16)
                    for (int k = 0; k < 16; k++) {
                        const int c = c0 + k;
                        float* dst = l == last ? O.mlp + plan.w_off[l] + c * kTcWidth + m : O.mlp + plan.w_off[l] + m * plan.cols[l] + c;
                        atomicAdd(dst, a[k] * inv);
                    }
            }
        }
    }
    if (!alive) {
        tc::mbar_wait(&bar, phase ^ 1u);  // the timed-out MMAs must not be in flight when the columns are freed
        if (t == 0) atomicExch(&g_tc_timeout, 1);
    }
    cp_async_wait();  // no activation copy outlives the CTA (only a timeout leaves one in flight)
    tc::fence_before_sync();
    __syncthreads();
    tc::fence_after_sync();
    if (warp == 0) tc::tmem_dealloc(tb, plan.tmem_cols);
}

// ---------------------------------------------------------------------------------------------------
// Warp-specialised MLP backward (training, with the colour pass's activation store): one CTA per SM, 512 threads.
//   warps 0-7    producer, two threads per tile row: gathers the row's inputs one tile ahead, encodes the input row
//                (fp16, K-major) keeping the fp32 sine and cosine for the input gradient, copies the stored activations
//                into the stage's slots (cp.async); the row's second thread also writes the SH inputs, the loss-scaled
//                output gradient and the row's view direction and base-colour gradient. Then every producer thread
//                arrives on the stage's `full` barrier.
//   warps 8-11   consumer 0 (stage 0: the CTA's even tiles) and warps 12-15 consumer 1 (stage 1: odd tiles), one
//                thread per row (warp w reads TMEM lanes 32 (w % 4) ..): the group's first thread issues the layer
//                MMAs, the group runs the data-gradient epilogues and the input-gradient epilogue, then arrives on the
//                stage's `empty` barrier. Each consumer owns 256 TMEM columns (its layer accumulator and its
//                weight-gradient accumulators, added to the output once per CTA).
// Two tiles are in flight per SM, so one consumer's epilogues overlap the other's MMAs and the producer's encoding
// of the next tiles. Same arithmetic as tc_bwd_kernel, row by row. Every wait is bounded; a wait that ran out makes
// its whole role stop (the threads of a role agree through a barrier reduction) and sets the timeout flag, and the
// other roles' bounded waits then run out in turn.
constexpr int kWsThreads = 512;
constexpr int kWsProducers = 256;

bool make_plan(const AppearanceConfig& A, bool backward, TcPlan& p);

struct WsRowInfo {      // per row of a stage: the last 32 bytes of the row block (TcRowLayout)
    uint32_t i;         // primitive index; 0xffffffff for rows past the end
    float rn;           // 1 / distance to the camera
    float dx, dy, dz;   // unit view direction
    float pad[3];
};

struct WsPlan {
    TcPlan t;                          // weights: w_smem, w_off, rows, cols, layers, kin
    uint32_t stage0, stage_bytes;      // first stage, bytes per stage
    uint32_t x_off, h_off, y_off, trig_off, info_off;  // offsets within a stage
    uint32_t wg_col[kTcMaxLayers];     // weight-gradient accumulators within a consumer's 256 columns
    uint32_t smem_bytes;
};

bool make_ws_plan(const AppearanceConfig& A, WsPlan& w) {
    if (!make_plan(A, true, w.t)) return false;
    const int F = A.feature_dim;
    if (!(A.n_freq == 1 && (F == 8 || F == 16 || F == 32) && !A.base_input && A.sh_mask == 15 && w.t.kin == 2 * F + 16)) return false;
    uint32_t wbytes = 0;
    for (int l = 0; l < w.t.layers; l++) wbytes += static_cast<uint32_t>(w.t.rows[l] * w.t.cols[l]) * 2;
    w.stage0 = (wbytes + 127) & ~127u;
    uint32_t o = 0;
    w.x_off = o;
    o += kTcRows * static_cast<uint32_t>(w.t.kin) * 2;
    w.h_off = o;
    o += static_cast<uint32_t>(w.t.layers - 1) * kTcActLayerBytes;
    w.y_off = o;
    o += kTcRows * 16 * 2;
    w.trig_off = o;
    o += static_cast<uint32_t>(2 * F) * kTcRows * 4;
    w.info_off = o;
    o += kTcRows * static_cast<uint32_t>(sizeof(WsRowInfo));
    w.stage_bytes = o;
    w.smem_bytes = w.stage0 + 2 * w.stage_bytes;
    // the feature-gradient staging block (rows of F + 4 floats, then the row's primitive) fits in the input slot
    if (static_cast<uint32_t>(F + 4) * kTcRows * 4 + kTcRows * 4 > kTcRows * static_cast<uint32_t>(w.t.kin) * 2) return false;
    uint32_t cols = static_cast<uint32_t>(w.t.kin > kTcWidth ? w.t.kin : kTcWidth);
    for (int l = 0; l < w.t.layers; l++) {
        w.wg_col[l] = cols;
        cols += static_cast<uint32_t>(l == w.t.layers - 1 ? w.t.rows[l] : w.t.cols[l]);
    }
    return cols <= 256 && w.smem_bytes + 256 <= 227u * 1024u;
}

// Split of a row's producer work: the first thread encodes feature chunks [0, kC0) (4 features = one 16-byte chunk of
// 8 encoded columns), the second thread chunks [kC0, F / 4) and copies the row block (SH inputs, output gradient, row
// info) into the stage.
template <int F>
struct WsSplit {
    static constexpr int kChunks = F / 4;
    static constexpr int kC0 = (kChunks + 1) / 2;
};

// The producer's row buffer of half H (0: first thread of the row, 1: second): the row's primitive and this thread's
// latent feature chunks.
template <int F, int H>
struct WsRow {
    static constexpr int kN = H ? WsSplit<F>::kChunks - WsSplit<F>::kC0 : WsSplit<F>::kC0;
    uint32_t i;
    bool valid;
    float4 f[kN > 0 ? kN : 1];
};

template <int F, int H>
__device__ inline void ws_load_index(const uint32_t* __restrict__ vis, uint32_t n_rows, uint32_t tile, int row, WsRow<F, H>& d) {
    const uint32_t gi = tile * kTcRows + row;
    d.valid = gi < n_rows;
    d.i = d.valid ? vis[gi] : 0u;
}
template <int F, int H>
__device__ inline void ws_load_features(const Params& P, WsRow<F, H>& d) {
    if (!d.valid) return;
    const float4* src = reinterpret_cast<const float4*>(P.residual + static_cast<size_t>(d.i) * F) + (H ? WsSplit<F>::kC0 : 0);
#pragma unroll
    for (int q = 0; q < WsRow<F, H>::kN; q++) d.f[q] = src[q];
}

// producer: this thread's feature chunks of one row of a stage (`xs`: the row's first 16-byte chunk of the input
// slot; the fp32 sine and cosine go to `trig`); the second thread also clears the output gradient's unused chunk and,
// for rows past the end, the SH chunks, the output gradient and the row info
template <int F, int H>
__device__ inline void ws_write_row(const WsRow<F, H>& d, uint4* xs, float* trig, uint4* ys, WsRowInfo* info, int row) {
    using S = WsSplit<F>;
    constexpr int c_lo = H ? S::kC0 : 0, n = WsRow<F, H>::kN;
    if (H) {
        ys[8] = make_uint4(0u, 0u, 0u, 0u);
        if (!d.valid) {
            xs[8 * S::kChunks] = make_uint4(0u, 0u, 0u, 0u);
            xs[8 * (S::kChunks + 1)] = make_uint4(0u, 0u, 0u, 0u);
            ys[0] = make_uint4(0u, 0u, 0u, 0u);
            info[row].i = 0xffffffffu;
        }
    }
    if (!d.valid) {
#pragma unroll
        for (int q = 0; q < n; q++) xs[8 * (c_lo + q)] = make_uint4(0u, 0u, 0u, 0u);
        return;
    }
#pragma unroll
    for (int q = 0; q < n; q++) {
        const float4 x = d.f[q];
        float s0, c0, s1, c1, s2, c2, s3, c3;
        enc_sincos(x.x, &s0, &c0);
        enc_sincos(x.y, &s1, &c1);
        enc_sincos(x.z, &s2, &c2);
        enc_sincos(x.w, &s3, &c3);
        xs[8 * (c_lo + q)] = make_uint4(pack2(s0, c0), pack2(s1, c1), pack2(s2, c2), pack2(s3, c3));
        float* tq = trig + (8 * (c_lo + q)) * kTcRows + row;
        tq[0] = s0; tq[kTcRows] = c0; tq[2 * kTcRows] = s1; tq[3 * kTcRows] = c1;
        tq[4 * kTcRows] = s2; tq[5 * kTcRows] = c2; tq[6 * kTcRows] = s3; tq[7 * kTcRows] = c3;
    }
}

struct WsShared {  // what the producer and consumers share besides the plan
    unsigned char* smem;
    uint32_t sbase;
    uint64_t* full_bar;
    uint64_t* empty_bar;
};

// The producer loop of half H over the CTA's tiles. Three row buffers rotate (this tile, the next, the one after the
// next), so no buffer is copied while its loads are in flight. Loads are issued after the stage's arrival (an arrival
// orders this thread's earlier memory accesses, so loads issued before it would be waited for there): the features of
// the tile after the next and the index of the tile after that. Returns false when a wait ran out.
template <int F, int H>
__device__ bool ws_producer(const Params& P, const uint32_t* __restrict__ vis, uint32_t n_rows, const WsPlan& plan, const WsShared& sh,
                            int row) {
    using S = WsSplit<F>;
    const uint32_t n_tiles = (n_rows + kTcRows - 1) / kTcRows, G = gridDim.x;
    const int last = plan.t.layers - 1;
    const unsigned char* const act = P.mlp_act;
    const uint32_t rows_off = static_cast<uint32_t>(last) * kTcActLayerBytes + kTcActOutBytes;
    WsRow<F, H> ra, rb, rc;
    uint32_t tile = blockIdx.x;
    if (tile < n_tiles) {
        ws_load_index(vis, n_rows, tile, row, ra);
        ws_load_features(P, ra);
    }
    if (tile + G < n_tiles) {
        ws_load_index(vis, n_rows, tile + G, row, rb);
        ws_load_features(P, rb);
    }
    if (tile + 2 * G < n_tiles) ws_load_index(vis, n_rows, tile + 2 * G, row, rc);
    auto produce = [&](uint32_t k, WsRow<F, H>& cur, WsRow<F, H>& n2) -> bool {
        const uint32_t s = k & 1u;
        if (k >= 2 && !tc::mbar_wait(&sh.empty_bar[s], ((k >> 1) - 1) & 1u)) return false;
        const uint32_t st = sh.sbase + plan.stage0 + s * plan.stage_bytes;
        unsigned char* const sg = sh.smem + plan.stage0 + s * plan.stage_bytes;
        const unsigned char* const at = act_tile(plan.t, act, tile);
        // this thread's half of the row's stored activations into the stage's slots; the second thread also the row
        // block (SH chunks into the input slot, the output gradient chunk, the row info); complete before the arrival
        const uint32_t off = tc::kmajor_offset(row, 0, kTcWidth);
        for (int j = 0; j < last; j++) {
            const unsigned char* src = at + static_cast<size_t>(j) * kTcActLayerBytes + off;
            const uint32_t dst = st + plan.h_off + static_cast<uint32_t>(j) * kTcActLayerBytes + off;
#pragma unroll
            for (int q = 0; q < 4; q++) cp_async16(dst + (4 * H + q) * 128, src + (4 * H + q) * 128);
        }
        const uint32_t x_row = st + plan.x_off + tc::kmajor_offset(row, 0, 2 * F + 16);
        if (H && cur.valid) {
            const unsigned char* rb_src = at + rows_off + static_cast<size_t>(row) * kTcRowDataBytes;
            cp_async16(x_row + S::kChunks * 128, rb_src);
            cp_async16(x_row + (S::kChunks + 1) * 128, rb_src + 16);
            cp_async16(st + plan.y_off + tc::kmajor_offset(row, 0, 16), rb_src + 32);
            cp_async16(st + plan.info_off + row * 32, rb_src + 48);
            cp_async16(st + plan.info_off + row * 32 + 16, rb_src + 64);
        }
        cp_async_commit();
        ws_write_row(cur, reinterpret_cast<uint4*>(sg + plan.x_off + tc::kmajor_offset(row, 0, 2 * F + 16)), reinterpret_cast<float*>(sg + plan.trig_off),
                     reinterpret_cast<uint4*>(sg + plan.y_off + tc::kmajor_offset(row, 0, 16)), reinterpret_cast<WsRowInfo*>(sg + plan.info_off), row);
        cp_async_wait();
        tc::fence_smem_to_async();
        tc::mbar_arrive(&sh.full_bar[s]);
        if (tile + 2 * G < n_tiles) ws_load_features(P, n2);
        if (tile + 3 * G < n_tiles) ws_load_index(vis, n_rows, tile + 3 * G, row, cur);
        return true;
    };
    for (uint32_t k = 0; tile < n_tiles;) {
        if (!produce(k, ra, rc)) return false;
        k++;
        if ((tile += G) >= n_tiles) break;
        if (!produce(k, rb, ra)) return false;
        k++;
        if ((tile += G) >= n_tiles) break;
        if (!produce(k, rc, rb)) return false;
        k++;
        tile += G;
    }
    return true;
}

// backward MMAs of layer l for a stage (stage base `st`) into a consumer's columns (`cb`)
__device__ inline void ws_issue_backward(const WsPlan& p, uint32_t sbase, uint32_t st, uint32_t cb, int l, bool wg_accumulate) {
    const int last = p.t.layers - 1;
    const uint32_t in = st + (l == 0 ? p.x_off : p.h_off + static_cast<uint32_t>(l - 1) * kTcActLayerBytes);
    const uint32_t K = p.t.cols[l], in_row_group = 16u * K;
    const uint32_t dout = st + (l == last ? p.y_off : p.h_off + static_cast<uint32_t>(l) * kTcActLayerBytes);
    const uint32_t R = p.t.rows[l], dout_row_group = 16u * R;
    const uint32_t w = sbase + p.t.w_smem[l];
    const uint32_t dw = cb + p.wg_col[l];
    const uint64_t in_mn = tc::desc(in, in_row_group, 128), dout_mn = tc::desc(dout, dout_row_group, 128);
    if (l == last) {
        const uint32_t id = tc::idesc(64, R, 1, 1);
        for (uint32_t ks = 0; ks < kTcRows / 16; ks++)
            tc::mma(dw, tc::desc_advance(in_mn, ks * 2 * in_row_group), tc::desc_advance(dout_mn, ks * 2 * dout_row_group), id,
                    (wg_accumulate || ks > 0) ? 1u : 0u);
    } else {
        const uint32_t id = tc::idesc(64, K, 1, 1);
        for (uint32_t ks = 0; ks < kTcRows / 16; ks++)
            tc::mma(dw, tc::desc_advance(dout_mn, ks * 2 * dout_row_group), tc::desc_advance(in_mn, ks * 2 * in_row_group), id,
                    (wg_accumulate || ks > 0) ? 1u : 0u);
    }
    const uint32_t id = tc::idesc(128, K, 0, 1);
    const uint64_t dk = tc::desc(dout, 128, dout_row_group), wmn = tc::desc(w, in_row_group, 128);
    for (uint32_t ks = 0; ks < R / 16; ks++)
        tc::mma(cb, tc::desc_advance(dk, ks * 256), tc::desc_advance(wmn, ks * 2 * in_row_group), id, ks > 0);
}

// consumer: data-gradient epilogue of a hidden layer for one row (64 columns): dL/d(activation), masked by the ReLU
// of the stored activation, written over that activation (fp16, in place; `hs`: the row's first 16-byte chunk).
// The stored chunks are read before any is written, so the loads issue together.
__device__ inline void ws_hidden_grad(uint32_t t_addr, uint4* hs, bool relu) {
    float a[64];
    tc::ld64(t_addr, a);
    uint4 h[8];
#pragma unroll
    for (int q = 0; q < 8; q++) h[q] = hs[8 * q];
#pragma unroll
    for (int q = 0; q < 8; q++) {
        float* x = a + 8 * q;
        if (relu) {
            const uint32_t hw[4] = {h[q].x, h[q].y, h[q].z, h[q].w};
#pragma unroll
            for (int k = 0; k < 4; k++) {
                const float2 hv = unpack2(hw[k]);
                if (!(hv.x > 0.0f)) x[2 * k] = 0.0f;
                if (!(hv.y > 0.0f)) x[2 * k + 1] = 0.0f;
            }
        }
        hs[8 * q] = make_uint4(pack2(x[0], x[1]), pack2(x[2], x[3]), pack2(x[4], x[5]), pack2(x[6], x[7]));
    }
}

// consumer: loss-scaled dL/d(input) of the row (TMEM columns 0 .. 2F + 15) -> feature gradients into the staging row,
// the direction gradient added to the mean gradient
template <int F>
__device__ inline void ws_input_grad(const AppearanceConfig& A, const GradOut& O, uint32_t t_row, const WsRowInfo& ri, const float* trig, int row,
                                     int deg, float* stage_row) {
    const float inv = 1.0f / kLossScale;
    const bool valid = ri.i != 0xffffffffu;
#pragma unroll
    for (int h = 0; h < (F + 15) / 16; h++) {  // 16 features (32 columns) per TMEM load
        constexpr int kf = F < 16 ? F : 16;
        float g[2 * kf];
        if constexpr (kf == 16) tc::ld32(t_row + 32 * h, g);
        else tc::ld16(t_row + 32 * h, g);
        if (valid) {
#pragma unroll
            for (int q = 0; q < kf / 4; q++) {
                float gv[4];
#pragma unroll
                for (int k = 0; k < 4; k++) {
                    const int j = 16 * h + 4 * q + k;
                    const float sn = trig[(2 * j) * kTcRows + row], cs = trig[(2 * j + 1) * kTcRows + row];
                    gv[k] = (cs * g[2 * (4 * q + k)] - sn * g[2 * (4 * q + k) + 1]) * inv;
                }
                *reinterpret_cast<float4*>(stage_row + 16 * h + 4 * q) = make_float4(gv[0], gv[1], gv[2], gv[3]);
            }
        }
    }
    float gsh[16];
    tc::ld16(t_row + 2 * F, gsh);
    if (!valid) return;
    if (!A.dir_grad) return;
    const f3 d = mk3(ri.dx, ri.dy, ri.dz);
    const f3 gd = inv * sh_band_grad(15, deg, d, gsh);
    put3n(O.means, ri.i, ri.rn * (gd - dot3(gd, d) * d), 1);  // added to the geometry pass's mean gradient
}

template <int F>
__global__ void __launch_bounds__(kWsThreads, 1) tc_bwd_ws_kernel(Params P, AppearanceConfig A, View v, const uint32_t* __restrict__ vis,
                                                                  uint32_t n_rows, const uint32_t* __restrict__ rank_of,
                                                                  const Record* __restrict__ sorted_rec, const GradRecord* __restrict__ grads,
                                                                  GradOut O, const __grid_constant__ WsPlan plan) {
    extern __shared__ __align__(128) unsigned char smem[];
    __shared__ uint64_t full_bar[2], empty_bar[2], mma_bar[2];
    __shared__ uint32_t tbase;
    const int t = threadIdx.x, warp = t >> 5, lane = t & 31, row = t & (kTcRows - 1);
    const int role = t < kWsProducers ? 0 : 1 + ((t - kWsProducers) >> 7);  // 0 producer, 1 / 2 consumer 0 / 1
    stage_weights_tc(plan.t, P.mlp, smem);
    if (warp == 0) tc::tmem_alloc(&tbase, 512);
    if (t == 0)
        for (int s = 0; s < 2; s++) {
            tc::mbar_init(&full_bar[s], kWsProducers);
            tc::mbar_init(&empty_bar[s], kTcRows);
            tc::mbar_init(&mma_bar[s], 1);
        }
    sync_tile();
    const uint32_t tb = tbase, sbase = tc::smem_addr(smem);
    const uint32_t n_tiles = (n_rows + kTcRows - 1) / kTcRows, G = gridDim.x;
    const int deg = min(v.degree, A.max_degree);
    const int last = plan.t.layers - 1;
    bool alive = true;
    bool wg_started = false, mma_pending = false;
    uint32_t mma_parity = 0;
    if (role == 0) {
        // ---- producer (the two threads of a row are in different warps, so the branch is warp-uniform) ----
        const WsShared sh{smem, sbase, full_bar, empty_bar};
        alive = (t >> 7) ? ws_producer<F, 1>(P, vis, n_rows, plan, sh, row) : ws_producer<F, 0>(P, vis, n_rows, plan, sh, row);
    } else {
        // ---- consumer g: the CTA's tiles k = g, g + 2, ... on stage g ----
        // the MMA operands derive from warp-uniform values only (warp index and TMEM base through a shuffle), so the
        // elected lane issues them from uniform registers
        const int wu = tc::warp_id_uniform();
        const uint32_t g = static_cast<uint32_t>((wu - kWsProducers / 32) >> 2), bar_id = 1 + g;
        const uint32_t cb = __shfl_sync(0xffffffffu, tb, 0) + g * 256u;
        const uint32_t t_row = cb + (static_cast<uint32_t>((wu & 3) * 32) << 16);
        const uint32_t st = sbase + plan.stage0 + g * plan.stage_bytes;
        unsigned char* const sg = smem + plan.stage0 + g * plan.stage_bytes;
        const bool issuer_warp = (wu & 3) == 0;
        const bool relu = A.hidden_act == 1;
        float* const fstage = reinterpret_cast<float*>(sg + plan.x_off);
        uint32_t* const fprim = reinterpret_cast<uint32_t*>(sg + plan.x_off + static_cast<uint32_t>(F + 4) * kTcRows * 4);
        const float* const trig = reinterpret_cast<const float*>(sg + plan.trig_off);
        const WsRowInfo* const info = reinterpret_cast<const WsRowInfo*>(sg + plan.info_off);
        for (uint32_t k = g, tile = blockIdx.x + g * G; tile < n_tiles; k += 2, tile += 2 * G) {
            const bool ok = tc::mbar_wait(&full_bar[g], (k >> 1) & 1u);
            if (tc::bar_or(bar_id, kTcRows, !ok)) {
                alive = false;
                break;
            }
            tc::fence_after_sync();
            for (int l = last; l >= 0; l--) {
                if (issuer_warp) {
                    if (tc::elect_one()) {
                        ws_issue_backward(plan, sbase, st, cb, l, wg_started);
                        tc::commit(&mma_bar[g]);
                    }
                    __syncwarp();
                }
                mma_pending = true;
                const bool done = tc::mbar_wait(&mma_bar[g], mma_parity);
                if (tc::bar_or(bar_id, kTcRows, !done)) {
                    alive = false;
                    break;
                }
                mma_pending = false;
                mma_parity ^= 1u;
                tc::fence_after_sync();
                if (l > 0) {
                    ws_hidden_grad(t_row, reinterpret_cast<uint4*>(sg + plan.h_off + static_cast<uint32_t>(l - 1) * kTcActLayerBytes +
                                                                   tc::kmajor_offset(row, 0, kTcWidth)),
                                   relu);
                    tc::fence_smem_to_async();
                    tc::fence_before_sync();
                    tc::bar_sync(bar_id, kTcRows);
                    tc::fence_after_sync();
                }
            }
            if (!alive) break;
            wg_started = true;
            const WsRowInfo ri = info[row];
            ws_input_grad<F>(A, O, t_row, ri, trig, row, deg, fstage + row * (F + 4));
            fprim[row] = ri.i;
            tc::fence_before_sync();
            tc::bar_sync(bar_id, kTcRows);
            // the staged feature gradients by whole rows
#pragma unroll
            for (int m = 0; m < F / 4; m++) {
                const int c = row + kTcRows * m, r = c / (F / 4), q = c % (F / 4);
                const uint32_t pi = fprim[r];
                if (pi == 0xffffffffu) continue;
                const float4 val = *reinterpret_cast<const float4*>(fstage + r * (F + 4) + 4 * q);
                float4* dst = reinterpret_cast<float4*>(O.residual + static_cast<size_t>(pi) * F + 4 * q);
                if (O.accumulate) atomicAdd(dst, val);  // one addition per element and launch (deterministic)
                else *dst = val;
            }
            tc::mbar_arrive(&empty_bar[g]);
        }
        if (!alive && mma_pending) tc::mbar_wait(&mma_bar[g], mma_parity);  // no MMA in flight when the columns are freed
        // weight gradients of this consumer (M = 64 accumulators: row m in lane (m % 16) + 32 (m / 16)), unscaled
        if (wg_started && alive) {
            const float inv = 1.0f / kLossScale;
            const int m = (warp & 3) * 16 + lane;
            for (int l = 0; l < plan.t.layers; l++) {
                const int ncol = l == last ? plan.t.rows[l] : plan.t.cols[l];
                for (int c0 = 0; c0 < ncol; c0 += 16) {
                    float a[16];
                    tc::ld16(t_row + plan.wg_col[l] + c0, a);
                    if (lane < 16)
                        for (int kk = 0; kk < 16; kk++) {
                            const int c = c0 + kk;
                            float* dst = l == last ? O.mlp + plan.t.w_off[l] + c * kTcWidth + m : O.mlp + plan.t.w_off[l] + m * plan.t.cols[l] + c;
                            atomicAdd(dst, a[kk] * inv);
                        }
                }
            }
        }
    }
    if (!alive && row == 0) atomicExch(&g_tc_timeout, 1);
    cp_async_wait();  // no activation copy outlives the CTA (only a timeout leaves one in flight)
    tc::fence_before_sync();
    __syncthreads();
    tc::fence_after_sync();
    if (warp == 0) tc::tmem_dealloc(tb, 512);
}

// ---------------------------------------------------------------------------------------------------
// Warp-specialised colour pass (the forward MLP): one CTA per SM, 512 threads, four stages.
//   warps 0-7    producer, two threads per row: the latent features of the row's tile, encoded into the stage's input
//                slot (fp16, K-major); the second thread fewer features, and the SH inputs and the row's primitive index.
//   warps 8-11   consumer 0 (the CTA's even tiles, stages 0 and 2) and warps 12-15 consumer 1 (odd tiles, stages 1 and
//                3), one thread per row: per layer the group's elected lane issues the MMAs into the group's TMEM
//                columns, the group applies the activation and writes the fp16 activations over the stage's input slot
//                (and, training, into the activation store); after the last layer the colour goes to the record.
// A stage holds only the input slot and the row info, so four fit and the producer runs two tiles ahead of each
// consumer. Same arithmetic as tc_color_kernel.
constexpr int kCwStages = 4;

// Split of a row's encoding: the first thread chunks [0, kC0), the second the rest plus the view direction and SH inputs.
template <int F>
struct CwSplit {
    static constexpr int kChunks = F / 4;
    static constexpr int kC0 = (kChunks * 5 + 7) / 8;
};

struct CwPlan {
    TcPlan t;
    uint32_t stage0, stage_bytes, info_off, smem_bytes;
};

bool make_cw_plan(const AppearanceConfig& A, CwPlan& w) {
    if (!make_plan(A, false, w.t)) return false;
    const int F = A.feature_dim;
    if (!(A.n_freq == 1 && (F == 8 || F == 16 || F == 32) && !A.base_input && A.sh_mask == 15 && w.t.kin == 2 * F + 16)) return false;
    uint32_t wbytes = 0;
    for (int l = 0; l < w.t.layers; l++) wbytes += static_cast<uint32_t>(w.t.rows[l] * w.t.cols[l]) * 2;
    w.stage0 = (wbytes + 127) & ~127u;
    const uint32_t in_bytes = kTcRows * static_cast<uint32_t>(w.t.kin > kTcWidth ? w.t.kin : kTcWidth) * 2;  // input, then activations
    w.info_off = in_bytes;
    w.stage_bytes = in_bytes + kTcRows * 4;  // then the rows' primitive indices (0xffffffff past the end)
    w.smem_bytes = w.stage0 + kCwStages * w.stage_bytes;
    return w.smem_bytes + 256 <= 227u * 1024u;
}

template <int F, int H>
struct CwRow {
    static constexpr int kN = H ? CwSplit<F>::kChunks - CwSplit<F>::kC0 : CwSplit<F>::kC0;
    uint32_t i;
    bool valid;
    f3 mean;                       // second thread only
    float4 f[kN > 0 ? kN : 1];
};

template <int F, int H>
__device__ inline void cw_load(const Params& P, CwRow<F, H>& d) {
    if (!d.valid) return;
    const float4* src = reinterpret_cast<const float4*>(P.residual + static_cast<size_t>(d.i) * F) + (H ? CwSplit<F>::kC0 : 0);
#pragma unroll
    for (int q = 0; q < CwRow<F, H>::kN; q++) d.f[q] = src[q];
    if (H) d.mean = ld3(P.means, d.i);
}

// The colour pass's producer loop of half H; three row buffers rotate as in ws_producer. Returns false when a wait
// ran out.
template <int F, int H>
__device__ bool cw_producer(const Params& P, const View& v, int deg, const uint32_t* __restrict__ vis, uint32_t n_rows, const CwPlan& plan,
                            const WsShared& sh, int row) {
    using S = CwSplit<F>;
    constexpr int c_lo = H ? S::kC0 : 0;
    const uint32_t n_tiles = (n_rows + kTcRows - 1) / kTcRows, G = gridDim.x;
    auto index = [&](uint32_t tile, CwRow<F, H>& d) {
        const uint32_t gi = tile * kTcRows + row;
        d.valid = gi < n_rows;
        d.i = d.valid ? vis[gi] : 0u;
    };
    CwRow<F, H> ra, rb, rc;
    uint32_t tile = blockIdx.x;
    if (tile < n_tiles) {
        index(tile, ra);
        cw_load(P, ra);
    }
    if (tile + G < n_tiles) {
        index(tile + G, rb);
        cw_load(P, rb);
    }
    if (tile + 2 * G < n_tiles) index(tile + 2 * G, rc);
    auto produce = [&](uint32_t k, CwRow<F, H>& cur, CwRow<F, H>& n2) -> bool {
        const uint32_t s = k % kCwStages;
        if (k >= kCwStages && !tc::mbar_wait(&sh.empty_bar[s], ((k / kCwStages) - 1) & 1u)) return false;
        unsigned char* const sg = sh.smem + plan.stage0 + s * plan.stage_bytes;
        uint4* const xs = reinterpret_cast<uint4*>(sg + tc::kmajor_offset(row, 0, 2 * F + 16));
        uint32_t* const info = reinterpret_cast<uint32_t*>(sg + plan.info_off);
        if (!cur.valid) {
#pragma unroll
            for (int q = 0; q < CwRow<F, H>::kN; q++) xs[8 * (c_lo + q)] = make_uint4(0u, 0u, 0u, 0u);
            if (H) {
                xs[8 * S::kChunks] = make_uint4(0u, 0u, 0u, 0u);
                xs[8 * (S::kChunks + 1)] = make_uint4(0u, 0u, 0u, 0u);
                info[row] = 0xffffffffu;
            }
        } else {
#pragma unroll
            for (int q = 0; q < CwRow<F, H>::kN; q++) {
                const float4 x = cur.f[q];
                float s0, c0, s1, c1, s2, c2, s3, c3;
                enc_sincos(x.x, &s0, &c0);
                enc_sincos(x.y, &s1, &c1);
                enc_sincos(x.z, &s2, &c2);
                enc_sincos(x.w, &s3, &c3);
                xs[8 * (c_lo + q)] = make_uint4(pack2(s0, c0), pack2(s1, c1), pack2(s2, c2), pack2(s3, c3));
            }
            if (H) {
                const f3 dir = view_dir(v, cur.mean, nullptr);
                float shv[16];
                sh_band_values(15, deg, dir, [&](int kk, float val) { shv[kk] = val; });
                xs[8 * S::kChunks] = make_uint4(pack2(shv[0], shv[1]), pack2(shv[2], shv[3]), pack2(shv[4], shv[5]), pack2(shv[6], shv[7]));
                xs[8 * (S::kChunks + 1)] =
                    make_uint4(pack2(shv[8], shv[9]), pack2(shv[10], shv[11]), pack2(shv[12], shv[13]), pack2(shv[14], shv[15]));
                info[row] = cur.i;
            }
        }
        tc::fence_smem_to_async();
        tc::mbar_arrive(&sh.full_bar[s]);
        // loads after the arrival (which orders this thread's earlier memory accesses)
        if (tile + 2 * G < n_tiles) cw_load(P, n2);
        if (tile + 3 * G < n_tiles) index(tile + 3 * G, cur);
        return true;
    };
    for (uint32_t k = 0; tile < n_tiles;) {
        if (!produce(k, ra, rc)) return false;
        k++;
        if ((tile += G) >= n_tiles) break;
        if (!produce(k, rb, ra)) return false;
        k++;
        if ((tile += G) >= n_tiles) break;
        if (!produce(k, rc, rb)) return false;
        k++;
        tile += G;
    }
    return true;
}

template <int F>
__global__ void __launch_bounds__(kWsThreads, 1) tc_color_ws_kernel(Params P, AppearanceConfig A, View v, const uint32_t* __restrict__ vis,
                                                                    uint32_t n_rows, Record* __restrict__ rec, const __grid_constant__ CwPlan plan) {
    extern __shared__ __align__(128) unsigned char smem[];
    __shared__ uint64_t full_bar[kCwStages], empty_bar[kCwStages], mma_bar[2];
    __shared__ uint32_t tbase;
    const int t = threadIdx.x, warp = t >> 5, row = t & (kTcRows - 1);
    const bool producer = t < kWsProducers;
    stage_weights_tc(plan.t, P.mlp, smem);
    if (warp == 0) tc::tmem_alloc(&tbase, 256);
    if (t == 0) {
        for (int s = 0; s < kCwStages; s++) {
            tc::mbar_init(&full_bar[s], kWsProducers);
            tc::mbar_init(&empty_bar[s], kTcRows);
        }
        tc::mbar_init(&mma_bar[0], 1);
        tc::mbar_init(&mma_bar[1], 1);
    }
    sync_tile();
    const uint32_t sbase = tc::smem_addr(smem);
    const uint32_t n_tiles = (n_rows + kTcRows - 1) / kTcRows, G = gridDim.x;
    const int deg = min(v.degree, A.max_degree);
    bool alive = true;
    bool mma_pending = false;
    uint32_t mma_parity = 0;
    if (producer) {
        const WsShared sh{smem, sbase, full_bar, empty_bar};
        alive = (t >> 7) ? cw_producer<F, 1>(P, v, deg, vis, n_rows, plan, sh, row) : cw_producer<F, 0>(P, v, deg, vis, n_rows, plan, sh, row);
    } else {
        // ---- consumer g: the CTA's tiles k = g, g + 2, ... (stage k % 4) ----
        const int wu = tc::warp_id_uniform();
        const uint32_t g = static_cast<uint32_t>((wu - kWsProducers / 32) >> 2), bar_id = 1 + g;
        const uint32_t cb = __shfl_sync(0xffffffffu, tbase, 0) + g * 128u;
        const uint32_t t_row = cb + (static_cast<uint32_t>((wu & 3) * 32) << 16);
        const bool issuer_warp = (wu & 3) == 0;
        const bool relu = A.hidden_act == 1;
        const int last = plan.t.layers - 1;
        const uint32_t h_row = tc::kmajor_offset(row, 0, kTcWidth);
        for (uint32_t k = g, tile = blockIdx.x + g * G; tile < n_tiles; k += 2, tile += 2 * G) {
            const uint32_t s = k % kCwStages;
            const bool ok = tc::mbar_wait(&full_bar[s], (k / kCwStages) & 1u);
            if (tc::bar_or(bar_id, kTcRows, !ok)) {
                alive = false;
                break;
            }
            tc::fence_after_sync();
            const uint32_t st = sbase + plan.stage0 + s * plan.stage_bytes;
            unsigned char* const sg = smem + plan.stage0 + s * plan.stage_bytes;
            const uint32_t pi = reinterpret_cast<const uint32_t*>(sg + plan.info_off)[row];
            // the base colour, needed after the last layer: loaded now so its latency passes under the MMAs
            const f3 base_p = pi != 0xffffffffu ? ld3(P.base, pi) : mk3(0.0f, 0.0f, 0.0f);
            unsigned char* const act = P.mlp_act ? P.mlp_act + static_cast<size_t>(tile) * plan.t.act_tile_bytes : nullptr;
            for (int l = 0; l <= last; l++) {
                if (issuer_warp) {
                    if (tc::elect_one()) {
                        // the input (layer 0) or the previous activations, written over the input slot
                        const uint32_t K = plan.t.cols[l], sbo = 16u * K, w = sbase + plan.t.w_smem[l];
                        const uint32_t id = tc::idesc(128, plan.t.rows[l], 0, 0);
                        const uint64_t a = tc::desc(st, 128, sbo), b = tc::desc(w, 128, sbo);
                        for (uint32_t ks = 0; ks < K / 16; ks++) tc::mma(cb, tc::desc_advance(a, ks * 256), tc::desc_advance(b, ks * 256), id, ks > 0);
                        tc::commit(&mma_bar[g]);
                    }
                    // training: the previous layer's activations (the 16 KB K-major block in the slot) into the
                    // activation store with one bulk copy, by the group's first thread
                    if (act && l > 0 && row == 0) {
                        tc::bulk_s2g(act + static_cast<size_t>(l - 1) * kTcActLayerBytes, st, kTcActLayerBytes);
                        tc::bulk_commit();
                    }
                    __syncwarp();
                }
                mma_pending = true;
                const bool done = tc::mbar_wait(&mma_bar[g], mma_parity);
                // the copy has read the slot before the epilogue below (or the next tile) writes it again
                if (act && l > 0 && row == 0) tc::bulk_wait_read();
                if (tc::bar_or(bar_id, kTcRows, !done)) {
                    alive = false;
                    break;
                }
                mma_pending = false;
                mma_parity ^= 1u;
                tc::fence_after_sync();
                if (l < last) {
                    float a[64];
                    tc::ld64(t_row, a);
                    uint4* const hs = reinterpret_cast<uint4*>(sg + h_row);
#pragma unroll
                    for (int q = 0; q < 8; q++) {
                        float* x = a + 8 * q;
                        if (relu)
#pragma unroll
                            for (int kk = 0; kk < 8; kk++) x[kk] = fmaxf(x[kk], 0.0f);
                        hs[8 * q] = make_uint4(pack2(x[0], x[1]), pack2(x[2], x[3]), pack2(x[4], x[5]), pack2(x[6], x[7]));
                    }
                    tc::fence_smem_to_async();
                    tc::fence_before_sync();
                    tc::bar_sync(bar_id, kTcRows);
                    tc::fence_after_sync();
                } else {
                    float y[16];
                    tc::ld16(t_row, y);
                    if (act)
                        *reinterpret_cast<uint2*>(act + static_cast<size_t>(l) * kTcActLayerBytes + row * 8) =
                            make_uint2(pack2(y[0], y[1]), pack2(y[2], 0.0f));
                    if (pi != 0xffffffffu) {
                        const f3 res = residual_act3(A.res_act, mk3(__half2float(__float2half_rn(y[0])), __half2float(__float2half_rn(y[1])),
                                                                     __half2float(__float2half_rn(y[2]))));
                        const f3 base = base_act3(A.base_act, base_p);
                        f3 color = color_act3(A.color_act, base + res);
                        if (!v.render_base) {
                            const f3 bc = color_act3(A.color_act, base);
                            color = mk3(fabsf(color.x - bc.x), fabsf(color.y - bc.y), fabsf(color.z - bc.z));
                        }
                        float* q2 = reinterpret_cast<float*>(rec + pi) + 8;
                        q2[0] = color.x;
                        q2[1] = color.y;
                        q2[2] = color.z;
                    }
                    tc::fence_before_sync();
                }
            }
            if (!alive) break;
            tc::mbar_arrive(&empty_bar[s]);
        }
        if (!alive && mma_pending) tc::mbar_wait(&mma_bar[g], mma_parity);  // no MMA in flight when the columns are freed
        if (row == 0) tc::bulk_wait();  // the activation-store copies have completed before the CTA ends
    }
    if (!alive && row == 0) atomicExch(&g_tc_timeout, 1);
    tc::fence_before_sync();
    __syncthreads();
    tc::fence_after_sync();
    if (warp == 0) tc::tmem_dealloc(tbase, 256);
}

bool make_plan(const AppearanceConfig& A, bool backward, TcPlan& p) {
    if (A.n_neurons != kTcWidth || A.n_hidden < 1 || A.n_hidden + 1 > kTcMaxLayers) return false;
    p = TcPlan{};
    p.layers = A.n_hidden + 1;
    p.kin = A.n_input_pad;
    p.backward = backward ? 1 : 0;
    p.act_tile_bytes = static_cast<uint32_t>(p.layers - 1) * kTcActLayerBytes + kTcActOutBytes + kTcRows * kTcRowDataBytes;
    if (p.kin % 16 != 0 || p.kin > 256) return false;
    uint32_t off = 0, w = 0;
    for (int l = 0; l < p.layers; l++) {
        p.cols[l] = l == 0 ? p.kin : kTcWidth;
        p.rows[l] = l == p.layers - 1 ? 16 : kTcWidth;
        p.w_off[l] = w;
        w += static_cast<uint32_t>(p.rows[l] * p.cols[l]);
        p.w_smem[l] = off;
        off += static_cast<uint32_t>(p.rows[l] * p.cols[l]) * 2;
    }
    off = (off + 127) & ~127u;
    p.x_smem = off;
    off += kTcRows * static_cast<uint32_t>(p.kin) * 2;
    p.h_slots = backward ? (p.layers - 1) : 1;
    if (backward) {
        p.h_smem = off;
        off += static_cast<uint32_t>(p.h_slots) * kTcRows * kTcWidth * 2;
        p.y_smem = off;
        off += kTcRows * 16 * 2;
        // fp32 sine / cosine of the encoding (fast path) for the input gradient
        if (A.n_freq == 1 && A.feature_dim % 8 == 0 && A.feature_dim <= kPrefetchFeatures) {
            p.trig_smem = off;
            off += static_cast<uint32_t>(2 * A.feature_dim) * kTcRows * 4;
        }
    } else {
        // the forward's activations overwrite its input (each layer's MMAs completed before its epilogue writes)
        p.h_smem = p.x_smem;
        const uint32_t h_bytes = kTcRows * kTcWidth * 2;
        if (h_bytes > static_cast<uint32_t>(kTcRows * p.kin * 2)) off = p.x_smem + h_bytes;
    }
    p.smem_bytes = off;
    uint32_t cols = static_cast<uint32_t>(p.kin > kTcWidth ? p.kin : kTcWidth);
    if (backward)
        for (int l = 0; l < p.layers; l++) {
            p.wg_col[l] = cols;
            cols += static_cast<uint32_t>(l == p.layers - 1 ? p.rows[l] : p.cols[l]);
        }
    uint32_t alloc = 32;
    while (alloc < cols) alloc <<= 1;
    if (alloc > 512) return false;
    p.tmem_cols = alloc;
    return p.smem_bytes + 64 <= 227u * 1024u;
}

int tc_sm_count() {
    int dev = 0, sms = 148;
    cudaGetDevice(&dev);
    cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
    return sms;
}

template <typename K>
cudaError_t tc_grid(K kernel, const TcPlan& p, uint32_t n_tiles, int max_per_sm, int* grid) {
    cudaError_t e = cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, static_cast<int>(p.smem_bytes));
    if (e != cudaSuccess) return e;
    e = cudaFuncSetAttribute(kernel, cudaFuncAttributePreferredSharedMemoryCarveout, cudaSharedmemCarveoutMaxShared);
    if (e != cudaSuccess) return e;
    // resident CTAs per SM: shared memory (1 KiB reserved per CTA), TMEM (512 columns per SM), registers (launch bounds)
    int dev = 0, smem_sm = 0;
    cudaGetDevice(&dev);
    e = cudaDeviceGetAttribute(&smem_sm, cudaDevAttrMaxSharedMemoryPerMultiprocessor, dev);
    if (e != cudaSuccess) return e;
    int per_sm = smem_sm / static_cast<int>(p.smem_bytes + 1024 + 256);
    const int tmem_cap = static_cast<int>(512 / p.tmem_cols);
    if (per_sm > tmem_cap) per_sm = tmem_cap;
    if (per_sm > max_per_sm) per_sm = max_per_sm;
    if (per_sm < 1) return cudaErrorInvalidConfiguration;
    const uint32_t cap = static_cast<uint32_t>(per_sm) * static_cast<uint32_t>(tc_sm_count());
    *grid = static_cast<int>(n_tiles < cap ? n_tiles : cap);
    return cudaSuccess;
}

}  // namespace

bool tc_mlp_supported(const AppearanceConfig& A) {
    TcPlan p;
    return make_plan(A, true, p) && make_plan(A, false, p);
}

size_t tc_activation_bytes(const AppearanceConfig& A, uint64_t n_rows) {
    TcPlan p;
    if (!make_plan(A, true, p) || !make_plan(A, false, p)) return 0;
    return static_cast<size_t>((n_rows + kTcRows - 1) / kTcRows) * p.act_tile_bytes;
}

bool tc_ws_layout(const Params& P, const AppearanceConfig& A, const GradOut& O, TcRowLayout* L) {
    WsPlan w;
    if (!P.mlp_act || !make_ws_plan(A, w) || (reinterpret_cast<uintptr_t>(P.residual) & 15u) != 0 ||
        (reinterpret_cast<uintptr_t>(O.residual) & 15u) != 0)
        return false;
    L->tile_bytes = w.t.act_tile_bytes;
    L->outputs_off = static_cast<uint32_t>(w.t.layers - 1) * kTcActLayerBytes;
    L->rows_off = L->outputs_off + kTcActOutBytes;
    return true;
}

size_t tc_mlp_smem_bytes(const AppearanceConfig& A) {
    TcPlan f, b;
    if (!make_plan(A, false, f) || !make_plan(A, true, b)) return 0;
    return f.smem_bytes > b.smem_bytes ? f.smem_bytes : b.smem_bytes;
}

cudaError_t launch_tc_color(const Params& P, const AppearanceConfig& A, const View& v, const uint32_t* vis, uint32_t n_visible, Record* rec,
                            cudaStream_t s) {
    TcPlan p;
    if (!make_plan(A, false, p)) return cudaErrorInvalidConfiguration;
    if (n_visible == 0) return cudaSuccess;
    const uint32_t n_tiles = (n_visible + kTcRows - 1) / kTcRows;
    CwPlan w;
    if (make_cw_plan(A, w) && (reinterpret_cast<uintptr_t>(P.residual) & 15u) == 0) {
        auto launch = [&](auto kernel) -> cudaError_t {
            cudaError_t e = cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, static_cast<int>(w.smem_bytes));
            if (e != cudaSuccess) return e;
            const int grid = static_cast<int>(n_tiles < static_cast<uint32_t>(tc_sm_count()) ? n_tiles : tc_sm_count());
            kernel<<<grid, kWsThreads, w.smem_bytes, s>>>(P, A, v, vis, n_visible, rec, w);
            return cudaGetLastError();
        };
        switch (A.feature_dim) {
            case 8: return launch(tc_color_ws_kernel<8>);
            case 16: return launch(tc_color_ws_kernel<16>);
            default: return launch(tc_color_ws_kernel<32>);
        }
    }
    int grid = 0;
    cudaError_t e = tc_grid(tc_color_kernel, p, n_tiles, 3, &grid);
    if (e != cudaSuccess) return e;
    tc_color_kernel<<<grid, kTcThreads, p.smem_bytes, s>>>(P, A, v, vis, n_visible, rec, p);
    return cudaGetLastError();
}

cudaError_t launch_tc_backward(const Params& P, const AppearanceConfig& A, const View& v, const uint32_t* vis, uint32_t n_visible,
                               const uint32_t* rank_of, const Record* sorted_rec, const GradRecord* grads, const GradOut& O, cudaStream_t s) {
    TcPlan p;
    if (!make_plan(A, true, p)) return cudaErrorInvalidConfiguration;
    if (n_visible == 0) return cudaSuccess;
    const uint32_t n_tiles = (n_visible + kTcRows - 1) / kTcRows;
    WsPlan w;
    TcRowLayout L;
    if (tc_ws_layout(P, A, O, &L) && make_ws_plan(A, w)) {
        auto launch = [&](auto kernel) -> cudaError_t {
            cudaError_t e = cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, static_cast<int>(w.smem_bytes));
            if (e != cudaSuccess) return e;
            const int grid = static_cast<int>(n_tiles < static_cast<uint32_t>(tc_sm_count()) ? n_tiles : tc_sm_count());
            kernel<<<grid, kWsThreads, w.smem_bytes, s>>>(P, A, v, vis, n_visible, rank_of, sorted_rec, grads, O, w);
            return cudaGetLastError();
        };
        switch (A.feature_dim) {
            case 8: return launch(tc_bwd_ws_kernel<8>);
            case 16: return launch(tc_bwd_ws_kernel<16>);
            default: return launch(tc_bwd_ws_kernel<32>);
        }
    }
    int grid = 0;
    cudaError_t e = tc_grid(tc_bwd_kernel, p, n_tiles, 2, &grid);
    if (e != cudaSuccess) return e;
    tc_bwd_kernel<<<grid, kTcThreads, p.smem_bytes, s>>>(P, A, v, vis, n_visible, rank_of, sorted_rec, grads, O, p);
    return cudaGetLastError();
}

// device address of this device's timeout flag (cached per device)
cudaError_t tc_timeout_flag(int** flag) {
    static std::mutex mu;
    static int* addr[64] = {};
    int dev = 0;
    cudaError_t e = cudaGetDevice(&dev);
    if (e != cudaSuccess) return e;
    if (dev < 0 || dev >= 64) return cudaErrorInvalidDevice;
    std::lock_guard<std::mutex> lock(mu);
    if (!addr[dev]) {
        void* p = nullptr;
        e = cudaGetSymbolAddress(&p, g_tc_timeout);
        if (e != cudaSuccess) return e;
        addr[dev] = static_cast<int*>(p);
    }
    *flag = addr[dev];
    return cudaSuccess;
}

}  // namespace fgs
