// Fused multi-tensor Adam: one launch updates every parameter segment (a whole tensor, or the shard of
// a flat parameter buffer owned by this rank). Per-element update as in
// FasterGSVDACudaBackend/.../adam/src/adam.cu:18-42: m = fma(b1, m - g, g), v = fma(b2, v - g^2, g^2),
// p -= lr_col / (1 - b1^t) * m / (sqrt(v) / sqrt(1 - b2^t) + eps), with the learning rate cycled per
// column (index modulo the number of learning rates, at most 7; used by the spherical Voronoi layout).
#include "launch.h"

namespace fgs {

struct AdamTable {
    AdamSegment seg[kMaxAdamSegments];
    uint64_t start[kMaxAdamSegments + 1];
    int n;
};

__global__ void __launch_bounds__(256) adam_kernel(const AdamTable tab) {
    const uint64_t total = tab.start[tab.n];
    const uint64_t stride = static_cast<uint64_t>(gridDim.x) * blockDim.x;
    int s = 0;
    for (uint64_t e = static_cast<uint64_t>(blockIdx.x) * blockDim.x + threadIdx.x; e < total; e += stride) {
        while (e >= tab.start[s + 1]) s++;
        const AdamSegment& S = tab.seg[s];
        const uint64_t j = e - tab.start[s];
        const float g = S.grad[j];
        const float m0 = S.m[j], v0 = S.v[j];
        const float g2 = g * g;
        const float m = fmaf(S.beta1, m0 - g, g);
        const float v = fmaf(S.beta2, v0 - g2, g2);
        const float denom = sqrtf(v) * S.bc2_sqrt_rcp + S.eps;
        const float lr = S.lr[(S.col_offset + j) % static_cast<uint64_t>(S.n_lr)];
        S.param[j] -= lr * m / denom;
        S.m[j] = m;
        S.v[j] = v;
    }
}

cudaError_t launch_adam(const AdamSegment* segs, int n_segs, cudaStream_t s) {
    if (n_segs <= 0) return cudaSuccess;
    if (n_segs > kMaxAdamSegments) return cudaErrorInvalidValue;
    AdamTable tab;
    tab.n = n_segs;
    tab.start[0] = 0;
    for (int i = 0; i < n_segs; i++) {
        tab.seg[i] = segs[i];
        tab.start[i + 1] = tab.start[i] + segs[i].n;
    }
    for (int i = n_segs; i < kMaxAdamSegments; i++) tab.start[i + 1] = tab.start[n_segs];
    const uint64_t total = tab.start[n_segs];
    if (total == 0) return cudaSuccess;
    int dev = 0, sms = 148;
    cudaGetDevice(&dev);
    cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
    const uint64_t want = (total + 255) / 256;
    const int grid = static_cast<int>(want < static_cast<uint64_t>(sms) * 8 ? want : static_cast<uint64_t>(sms) * 8);
    adam_kernel<<<grid, 256, 0, s>>>(tab);
    return cudaGetLastError();
}

}  // namespace fgs
