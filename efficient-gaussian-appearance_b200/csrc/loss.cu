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

// stages the kE x kE tiles of up to three channel planes (zero padding outside the image; row stride kE + 1): a warp
// per staged row, its lanes along the row; tiles whose halo lies inside the image skip the bounds tests
template <int N>
__device__ inline void stage(const float* const (&src)[N], int H, int W, int x0, int y0, float* const (&dst)[N]) {
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    const bool interior = x0 >= kR && y0 >= kR && x0 + kT + kR <= W && y0 + kT + kR <= H;
    for (int r = warp; r < kE; r += kThreads / 32) {
        const int gy = y0 - kR + r;
        const bool row_in = interior || (gy >= 0 && gy < H);
        const size_t roff = static_cast<size_t>(gy) * W + (x0 - kR);
        for (int c = lane; c < kE; c += 32) {
            const int gx = x0 - kR + c;
            const bool in = interior || (row_in && gx >= 0 && gx < W);
#pragma unroll
            for (int q = 0; q < N; q++) dst[q][r * (kE + 1) + c] = in ? src[q][roff + c] : 0.0f;
        }
    }
}

__global__ void __launch_bounds__(kThreads) ssim_stats_kernel(const float* __restrict__ x, const float* __restrict__ t, int H, int W, Window win,
                                                              float* __restrict__ A, float* __restrict__ B, float* __restrict__ Cm,
                                                              float2* __restrict__ partial) {
    __shared__ float xs[kE * (kE + 1)], ts[kE * (kE + 1)];
    __shared__ __align__(16) float hs[5][kE * kT];  // 16-byte aligned rows: float4 stores
    __shared__ float red[2][kThreads / 32];
    const int x0 = blockIdx.x * kT, y0 = blockIdx.y * kT, ch = blockIdx.z;
    const size_t plane = static_cast<size_t>(H) * W;
    {
        const float* const src[2] = {x + ch * plane, t + ch * plane};
        float* const dst[2] = {xs, ts};
        stage<2>(src, H, W, x0, y0, dst);
    }
    __syncthreads();
    // rows: five moments of every staged row at every output column; a thread takes 4 consecutive columns of a row
    // (14 staged values feed its 4 outputs)
    for (int job = threadIdx.x; job < kE * (kT / 4); job += kThreads) {
        const int r = job / (kT / 4), c0 = (job - r * (kT / 4)) * 4;
        // the staged values and their products, once per staged element
        float xa[4 + 2 * kR], ta[4 + 2 * kR], xx[4 + 2 * kR], tt[4 + 2 * kR], xt[4 + 2 * kR];
#pragma unroll
        for (int j = 0; j < 4 + 2 * kR; j++) {
            xa[j] = xs[r * (kE + 1) + c0 + j];
            ta[j] = ts[r * (kE + 1) + c0 + j];
            xx[j] = xa[j] * xa[j];
            tt[j] = ta[j] * ta[j];
            xt[j] = xa[j] * ta[j];
        }
        float m[5][4];
#pragma unroll
        for (int o = 0; o < 4; o++) m[0][o] = m[1][o] = m[2][o] = m[3][o] = m[4][o] = 0.0f;
#pragma unroll
        for (int k = 0; k <= 2 * kR; k++) {
            const float w = win.w[k];
#pragma unroll
            for (int o = 0; o < 4; o++) {
                m[0][o] += w * xa[o + k];
                m[1][o] += w * ta[o + k];
                m[2][o] += w * xx[o + k];
                m[3][o] += w * tt[o + k];
                m[4][o] += w * xt[o + k];
            }
        }
#pragma unroll
        for (int q = 0; q < 5; q++)
            *reinterpret_cast<float4*>(&hs[q][r * kT + c0]) = make_float4(m[q][0], m[q][1], m[q][2], m[q][3]);
    }
    __syncthreads();
    // columns: a thread takes 4 consecutive rows of one column (14 row-pass values per moment feed them)
    float sum_s = 0.0f, sum_l1 = 0.0f;
    {
        const int c = threadIdx.x & (kT - 1), r0 = (threadIdx.x / kT) * 4;
        float mu_x[4], mu_y[4], exx[4], eyy[4], exy[4];
#pragma unroll
        for (int o = 0; o < 4; o++) mu_x[o] = mu_y[o] = exx[o] = eyy[o] = exy[o] = 0.0f;
#pragma unroll
        for (int j = 0; j < 4 + 2 * kR; j++) {
            const int i = (r0 + j) * kT + c;
            const float h0 = hs[0][i], h1 = hs[1][i], h2 = hs[2][i], h3 = hs[3][i], h4 = hs[4][i];
#pragma unroll
            for (int o = 0; o < 4; o++) {
                const int k = j - o;
                if (k < 0 || k > 2 * kR) continue;
                const float w = win.w[k];
                mu_x[o] += w * h0;
                mu_y[o] += w * h1;
                exx[o] += w * h2;
                eyy[o] += w * h3;
                exy[o] += w * h4;
            }
        }
#pragma unroll
        for (int o = 0; o < 4; o++) {
            const int r = r0 + o;
            const int gy = y0 + r, gx = x0 + c;
            if (gy >= H || gx >= W) continue;
            const float sxx = exx[o] - mu_x[o] * mu_x[o], syy = eyy[o] - mu_y[o] * mu_y[o], sxy = exy[o] - mu_x[o] * mu_y[o];
            const float a1 = 2.0f * mu_x[o] * mu_y[o] + kC1, a2 = 2.0f * sxy + kC2;
            const float b1 = mu_x[o] * mu_x[o] + mu_y[o] * mu_y[o] + kC1, b2 = sxx + syy + kC2;
            // one division: 1 / (b1 b2), and from it 1 / b1 = b2 / (b1 b2) and 1 / b2 = b1 / (b1 b2)
            const float rden = 1.0f / (b1 * b2), rb1 = b2 * rden, rb2 = b1 * rden;
            const float s = a1 * a2 * rden;
            const float ds_dmu = 2.0f * mu_y[o] * a2 * rden - s * 2.0f * mu_x[o] * rb1;
            const float ds_dsxx = -s * rb2;
            const float ds_dsxy = 2.0f * a1 * rden;
            const size_t p = ch * plane + static_cast<size_t>(gy) * W + gx;
            A[p] = ds_dmu - 2.0f * mu_x[o] * ds_dsxx - mu_y[o] * ds_dsxy;
            B[p] = ds_dsxx;
            Cm[p] = ds_dsxy;
            sum_s += s;
            sum_l1 += fabsf(xs[(r + kR) * (kE + 1) + c + kR] - ts[(r + kR) * (kE + 1) + c + kR]);
        }
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
    __shared__ __align__(16) float hs[3][kE * kT];  // 16-byte aligned rows: float4 stores
    const int x0 = blockIdx.x * kT, y0 = blockIdx.y * kT, ch = blockIdx.z;
    const size_t plane = static_cast<size_t>(H) * W;
    {
        const float* const src[3] = {A + ch * plane, B + ch * plane, Cm + ch * plane};
        float* const dst[3] = {as, bs, cs};
        stage<3>(src, H, W, x0, y0, dst);
    }
    __syncthreads();
    for (int job = threadIdx.x; job < kE * (kT / 4); job += kThreads) {
        const int r = job / (kT / 4), c0 = (job - r * (kT / 4)) * 4;
        float m[3][4];
#pragma unroll
        for (int o = 0; o < 4; o++) m[0][o] = m[1][o] = m[2][o] = 0.0f;
#pragma unroll
        for (int j = 0; j < 4 + 2 * kR; j++) {
            const int i = r * (kE + 1) + c0 + j;
            const float va = as[i], vb = bs[i], vc = cs[i];
#pragma unroll
            for (int o = 0; o < 4; o++) {
                const int k = j - o;
                if (k < 0 || k > 2 * kR) continue;
                const float w = win.w[k];
                m[0][o] += w * va;
                m[1][o] += w * vb;
                m[2][o] += w * vc;
            }
        }
#pragma unroll
        for (int q = 0; q < 3; q++)
            *reinterpret_cast<float4*>(&hs[q][r * kT + c0]) = make_float4(m[q][0], m[q][1], m[q][2], m[q][3]);
    }
    __syncthreads();
    const int c = threadIdx.x & (kT - 1), r0 = (threadIdx.x / kT) * 4;
    float ga[4], gb[4], gc[4];
#pragma unroll
    for (int o = 0; o < 4; o++) ga[o] = gb[o] = gc[o] = 0.0f;
#pragma unroll
    for (int j = 0; j < 4 + 2 * kR; j++) {
        const int i = (r0 + j) * kT + c;
        const float h0 = hs[0][i], h1 = hs[1][i], h2 = hs[2][i];
#pragma unroll
        for (int o = 0; o < 4; o++) {
            const int k = j - o;
            if (k < 0 || k > 2 * kR) continue;
            const float w = win.w[k];
            ga[o] += w * h0;
            gb[o] += w * h1;
            gc[o] += w * h2;
        }
    }
#pragma unroll
    for (int o = 0; o < 4; o++) {
        const int gy = y0 + r0 + o, gx = x0 + c;
        if (gy >= H || gx >= W) continue;
        const size_t p = ch * plane + static_cast<size_t>(gy) * W + gx;
        const float xv = x[p], tv = t[p], d = xv - tv;
        const float sgn = d > 0.0f ? 1.0f : (d < 0.0f ? -1.0f : 0.0f);
        grad[p] = l1_scale * sgn - ssim_scale * (ga[o] + 2.0f * xv * gb[o] + tv * gc[o]);
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
