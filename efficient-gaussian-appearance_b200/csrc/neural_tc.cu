// Neural appearance MLP on the sm_100a tensor cores (tcgen05 + TMEM); see tc.cuh for the operand layouts.
//
// This file also holds the tensor-core self-test behind fgs_tc_selftest: three small GEMMs covering every operand
// orientation the MLP kernels use (forward: A and B K-major; data gradient: B MN-major; weight gradient: M = 64,
// A and B MN-major, accumulated over two passes), checked exactly on the host.
#include <cuda_fp16.h>

#include <cstdint>
#include <vector>

#include "launch.h"
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

}  // namespace fgs
