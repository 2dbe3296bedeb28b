// Fused photometric loss of the training step: l1_weight * mean|x - t| + dssim_weight * (1 - mean SSIM(x, t)) and
// its gradient with respect to the rendered image x, for planar [C,H,W] fp32 images.
//
// Semantics: FasterGSVDA/Loss.py:14-15 (L1 with LAMBDA_L1, DSSIM with LAMBDA_DSSIM through NeRFICG's fused_dssim,
// which is absent here). SSIM uses an 11x11 Gaussian window (sigma 1.5, separable, normalised), zero padding outside
// the image, C1 = 0.01^2, C2 = 0.03^2, and the mean over every channel and pixel.
//
// Design: two tiled passes over 32x32 output tiles with a 5-pixel halo staged in shared memory, separable blurs
// (rows, then columns). Pass 1 computes the five local moments, the SSIM map and, per pixel, the partial
// derivatives of SSIM with respect to the moments (a = dS/dmu_x - 2 mu_x dS/dsxx - mu_y dS/dsxy, b = dS/dsxx,
// c = dS/dsxy), plus per-tile sums of SSIM and |x - t|. Pass 2 blurs a, b, c and forms
// dL/dx = l1 * sign(x - t) / n - dssim / n * (G*a + 2 x G*b + t G*c). A one-CTA pass sums the tile partials in
// double in a fixed order, so the loss is deterministic.
#include <cmath>
#include <cstdint>

#include <cuda_runtime.h>

#include "launch.h"

namespace fgs {

namespace {

constexpr int kT = 32;            // output tile edge
constexpr int kR = 5;             // window radius
constexpr int kE = kT + 2 * kR;   // staged edge (42)
constexpr int kThreads = 256;
constexpr float kC1 = 0.01f * 0.01f;
constexpr float kC2 = 0.03f * 0.03f;

struct Window { float w[2 * kR + 1]; };

// stages a kE x kE tile of `src` (channel plane) with zero padding; row stride kE + 1
__device__ inline void stage(const float* __restrict__ src, int H, int W, int x0, int y0, float* dst) {
    for (int idx = threadIdx.x; idx < kE * kE; idx += kThreads) {
        const int r = idx / kE, c = idx - r * kE;
        const int gy = y0 - kR + r, gx = x0 - kR + c;
        dst[r * (kE + 1) + c] = (gy >= 0 && gy < H && gx >= 0 && gx < W) ? src[static_cast<size_t>(gy) * W + gx] : 0.0f;
    }
}

__global__ void __launch_bounds__(kThreads) ssim_stats_kernel(const float* __restrict__ x, const float* __restrict__ t, int H, int W, Window win,
                                                              float* __restrict__ A, float* __restrict__ B, float* __restrict__ Cm,
                                                              float2* __restrict__ partial) {
    __shared__ float xs[kE * (kE + 1)], ts[kE * (kE + 1)];
    __shared__ float hs[5][kE * kT];
    __shared__ float red[2][kThreads / 32];
    const int x0 = blockIdx.x * kT, y0 = blockIdx.y * kT, ch = blockIdx.z;
    const size_t plane = static_cast<size_t>(H) * W;
    const float* xp = x + ch * plane;
    const float* tp = t + ch * plane;
    stage(xp, H, W, x0, y0, xs);
    stage(tp, H, W, x0, y0, ts);
    __syncthreads();
    // rows: five moments of every staged row at every output column
    for (int idx = threadIdx.x; idx < kE * kT; idx += kThreads) {
        const int r = idx / kT, c = idx - r * kT;
        float m0 = 0.0f, m1 = 0.0f, m2 = 0.0f, m3 = 0.0f, m4 = 0.0f;
#pragma unroll
        for (int k = 0; k <= 2 * kR; k++) {
            const float a = xs[r * (kE + 1) + c + k], b = ts[r * (kE + 1) + c + k], w = win.w[k];
            m0 += w * a;
            m1 += w * b;
            m2 += w * (a * a);
            m3 += w * (b * b);
            m4 += w * (a * b);
        }
        hs[0][idx] = m0;
        hs[1][idx] = m1;
        hs[2][idx] = m2;
        hs[3][idx] = m3;
        hs[4][idx] = m4;
    }
    __syncthreads();
    float sum_s = 0.0f, sum_l1 = 0.0f;
    const int c = threadIdx.x & (kT - 1);
    for (int r = threadIdx.x / kT; r < kT; r += kThreads / kT) {
        float mu_x = 0.0f, mu_y = 0.0f, exx = 0.0f, eyy = 0.0f, exy = 0.0f;
#pragma unroll
        for (int k = 0; k <= 2 * kR; k++) {
            const int o = (r + k) * kT + c;
            const float w = win.w[k];
            mu_x += w * hs[0][o];
            mu_y += w * hs[1][o];
            exx += w * hs[2][o];
            eyy += w * hs[3][o];
            exy += w * hs[4][o];
        }
        const int gy = y0 + r, gx = x0 + c;
        if (gy >= H || gx >= W) continue;
        const float sxx = exx - mu_x * mu_x, syy = eyy - mu_y * mu_y, sxy = exy - mu_x * mu_y;
        const float a1 = 2.0f * mu_x * mu_y + kC1, a2 = 2.0f * sxy + kC2;
        const float b1 = mu_x * mu_x + mu_y * mu_y + kC1, b2 = sxx + syy + kC2;
        const float den = b1 * b2;
        const float s = a1 * a2 / den;
        const float ds_dmu = 2.0f * mu_y * a2 / den - s * 2.0f * mu_x / b1;
        const float ds_dsxx = -s / b2;
        const float ds_dsxy = 2.0f * a1 / den;
        const size_t p = ch * plane + static_cast<size_t>(gy) * W + gx;
        A[p] = ds_dmu - 2.0f * mu_x * ds_dsxx - mu_y * ds_dsxy;
        B[p] = ds_dsxx;
        Cm[p] = ds_dsxy;
        sum_s += s;
        sum_l1 += fabsf(xs[(r + kR) * (kE + 1) + c + kR] - ts[(r + kR) * (kE + 1) + c + kR]);
    }
    for (int o = 16; o > 0; o >>= 1) {
        sum_s += __shfl_down_sync(0xffffffffu, sum_s, o);
        sum_l1 += __shfl_down_sync(0xffffffffu, sum_l1, o);
    }
    if ((threadIdx.x & 31) == 0) {
        red[0][threadIdx.x >> 5] = sum_s;
        red[1][threadIdx.x >> 5] = sum_l1;
    }
    __syncthreads();
    if (threadIdx.x == 0) {
        float a = 0.0f, b = 0.0f;
        for (int w = 0; w < kThreads / 32; w++) {
            a += red[0][w];
            b += red[1][w];
        }
        partial[(static_cast<size_t>(ch) * gridDim.y + blockIdx.y) * gridDim.x + blockIdx.x] = make_float2(a, b);
    }
}

__global__ void __launch_bounds__(kThreads) ssim_grad_kernel(const float* __restrict__ x, const float* __restrict__ t, int H, int W, Window win,
                                                             const float* __restrict__ A, const float* __restrict__ B, const float* __restrict__ Cm,
                                                             float l1_scale, float ssim_scale, float* __restrict__ grad) {
    __shared__ float as[kE * (kE + 1)], bs[kE * (kE + 1)], cs[kE * (kE + 1)];
    __shared__ float hs[3][kE * kT];
    const int x0 = blockIdx.x * kT, y0 = blockIdx.y * kT, ch = blockIdx.z;
    const size_t plane = static_cast<size_t>(H) * W;
    stage(A + ch * plane, H, W, x0, y0, as);
    stage(B + ch * plane, H, W, x0, y0, bs);
    stage(Cm + ch * plane, H, W, x0, y0, cs);
    __syncthreads();
    for (int idx = threadIdx.x; idx < kE * kT; idx += kThreads) {
        const int r = idx / kT, c = idx - r * kT;
        float m0 = 0.0f, m1 = 0.0f, m2 = 0.0f;
#pragma unroll
        for (int k = 0; k <= 2 * kR; k++) {
            const int o = r * (kE + 1) + c + k;
            const float w = win.w[k];
            m0 += w * as[o];
            m1 += w * bs[o];
            m2 += w * cs[o];
        }
        hs[0][idx] = m0;
        hs[1][idx] = m1;
        hs[2][idx] = m2;
    }
    __syncthreads();
    const int c = threadIdx.x & (kT - 1);
    for (int r = threadIdx.x / kT; r < kT; r += kThreads / kT) {
        const int gy = y0 + r, gx = x0 + c;
        if (gy >= H || gx >= W) continue;
        float ga = 0.0f, gb = 0.0f, gc = 0.0f;
#pragma unroll
        for (int k = 0; k <= 2 * kR; k++) {
            const int o = (r + k) * kT + c;
            const float w = win.w[k];
            ga += w * hs[0][o];
            gb += w * hs[1][o];
            gc += w * hs[2][o];
        }
        const size_t p = ch * plane + static_cast<size_t>(gy) * W + gx;
        const float xv = x[p], tv = t[p], d = xv - tv;
        const float sgn = d > 0.0f ? 1.0f : (d < 0.0f ? -1.0f : 0.0f);
        grad[p] = l1_scale * sgn - ssim_scale * (ga + 2.0f * xv * gb + tv * gc);
    }
}

__global__ void loss_reduce_kernel(const float2* __restrict__ partial, uint32_t n, double n_pixels, float l1_weight, float dssim_weight,
                                   float* __restrict__ loss) {
    __shared__ double rs[256], rl[256];
    double s = 0.0, l = 0.0;
    for (uint32_t k = threadIdx.x; k < n; k += blockDim.x) {
        s += partial[k].x;
        l += partial[k].y;
    }
    rs[threadIdx.x] = s;
    rl[threadIdx.x] = l;
    __syncthreads();
    for (int o = blockDim.x / 2; o > 0; o >>= 1) {
        if (threadIdx.x < o) {
            rs[threadIdx.x] += rs[threadIdx.x + o];
            rl[threadIdx.x] += rl[threadIdx.x + o];
        }
        __syncthreads();
    }
    if (threadIdx.x == 0) loss[0] = static_cast<float>(l1_weight * (rl[0] / n_pixels) + dssim_weight * (1.0 - rs[0] / n_pixels));
}

Window gaussian_window() {
    // fp32 as the loss definition computes it: exp(-(k - 5)^2 / (2 sigma^2)) normalised by its sum
    Window w;
    float sum = 0.0f;
    for (int k = 0; k <= 2 * kR; k++) {
        const float d = static_cast<float>(k - kR);
        w.w[k] = std::exp(-(d * d) / (2.0f * 1.5f * 1.5f));
        sum += w.w[k];
    }
    for (int k = 0; k <= 2 * kR; k++) w.w[k] /= sum;
    return w;
}

uint32_t n_tiles(int C, int H, int W) {
    return static_cast<uint32_t>(C) * static_cast<uint32_t>((H + kT - 1) / kT) * static_cast<uint32_t>((W + kT - 1) / kT);
}

}  // namespace

size_t loss_workspace_bytes(int C, int H, int W) {
    const size_t px = static_cast<size_t>(C) * H * W;
    return 3 * px * sizeof(float) + static_cast<size_t>(n_tiles(C, H, W)) * sizeof(float2) + 256;
}

cudaError_t launch_l1_dssim(const float* image, const float* target, int C, int H, int W, float l1_weight, float dssim_weight, float* grad,
                            float* loss, void* ws, cudaStream_t s) {
    const size_t px = static_cast<size_t>(C) * H * W;
    float* A = static_cast<float*>(ws);
    float* B = A + px;
    float* Cm = B + px;
    float2* partial = reinterpret_cast<float2*>((reinterpret_cast<uintptr_t>(Cm + px) + 15) & ~static_cast<uintptr_t>(15));
    const Window win = gaussian_window();
    const dim3 grid((W + kT - 1) / kT, (H + kT - 1) / kT, C);
    ssim_stats_kernel<<<grid, kThreads, 0, s>>>(image, target, H, W, win, A, B, Cm, partial);
    cudaError_t e = cudaGetLastError();
    if (e != cudaSuccess) return e;
    const double n = static_cast<double>(px);
    ssim_grad_kernel<<<grid, kThreads, 0, s>>>(image, target, H, W, win, A, B, Cm, static_cast<float>(l1_weight / n),
                                               static_cast<float>(dssim_weight / n), grad);
    e = cudaGetLastError();
    if (e != cudaSuccess) return e;
    loss_reduce_kernel<<<1, 256, 0, s>>>(partial, n_tiles(C, H, W), n, l1_weight, dssim_weight, loss);
    return cudaGetLastError();
}

}  // namespace fgs
