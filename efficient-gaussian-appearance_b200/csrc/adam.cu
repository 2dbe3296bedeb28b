// Fused multi-tensor Adam: one launch updates every parameter segment (a whole tensor, or the shard of
// a flat parameter buffer owned by this rank). Per-element update as in
// FasterGSVDACudaBackend/.../adam/src/adam.cu:18-42: m = fma(b1, m - g, g), v = fma(b2, v - g^2, g^2),
// p -= lr_col / (1 - b1^t) * m / (sqrt(v) / sqrt(1 - b2^t) + eps), with the learning rate cycled per
// column (index modulo the number of learning rates, at most 7; used by the spherical Voronoi layout).
#include "launch.h"

namespace fgs {

struct AdamTable {
    AdamSegment seg[kMaxAdamSegments];
    int n;
};

__device__ inline void adam_one(const AdamSegment& S, float& p, float g, float& m, float& v, float lr) {
    const float g2 = g * g;
    const float mm = fmaf(S.beta1, m - g, g);
    const float vv = fmaf(S.beta2, v - g2, g2);
    const float denom = sqrtf(vv) * S.bc2_sqrt_rcp + S.eps;
    p -= lr * mm / denom;
    m = mm;
    v = vv;
}

// blockIdx.y selects the segment; the x blocks stride over it, four elements per thread when the four arrays
// are 16-byte aligned
__global__ void __launch_bounds__(256) adam_kernel(const AdamTable tab) {
    if (static_cast<int>(blockIdx.y) >= tab.n) return;
    const AdamSegment& S = tab.seg[blockIdx.y];
    const uint64_t stride = static_cast<uint64_t>(gridDim.x) * blockDim.x;
    const uint64_t tid = static_cast<uint64_t>(blockIdx.x) * blockDim.x + threadIdx.x;
    const uint32_t nl = static_cast<uint32_t>(S.n_lr);
    const bool vec = ((reinterpret_cast<uintptr_t>(S.param) | reinterpret_cast<uintptr_t>(S.grad) | reinterpret_cast<uintptr_t>(S.m) |
                       reinterpret_cast<uintptr_t>(S.v)) & 15u) == 0;
    uint64_t done = 0;
    if (vec) {
        const uint64_t n4 = S.n / 4;
        float4* P4 = reinterpret_cast<float4*>(S.param);
        const float4* G4 = reinterpret_cast<const float4*>(S.grad);
        float4* M4 = reinterpret_cast<float4*>(S.m);
        float4* V4 = reinterpret_cast<float4*>(S.v);
        for (uint64_t q = tid; q < n4; q += stride) {
            float4 p = P4[q], m = M4[q], v = V4[q];
            const float4 g = G4[q];
            uint32_t c = nl == 1 ? 0u : static_cast<uint32_t>((S.col_offset + 4 * q) % nl);
            adam_one(S, p.x, g.x, m.x, v.x, S.lr[c]);
            c = c + 1 == nl ? 0u : c + 1;
            adam_one(S, p.y, g.y, m.y, v.y, S.lr[c]);
            c = c + 1 == nl ? 0u : c + 1;
            adam_one(S, p.z, g.z, m.z, v.z, S.lr[c]);
            c = c + 1 == nl ? 0u : c + 1;
            adam_one(S, p.w, g.w, m.w, v.w, S.lr[c]);
            P4[q] = p;
            M4[q] = m;
            V4[q] = v;
        }
        done = 4 * n4;
    }
    for (uint64_t j = done + tid; j < S.n; j += stride) {
        const uint32_t c = nl == 1 ? 0u : static_cast<uint32_t>((S.col_offset + j) % nl);
        adam_one(S, S.param[j], S.grad[j], S.m[j], S.v[j], S.lr[c]);
    }
}

cudaError_t launch_adam(const AdamSegment* segs, int n_segs, cudaStream_t s) {
    if (n_segs <= 0) return cudaSuccess;
    if (n_segs > kMaxAdamSegments) return cudaErrorInvalidValue;
    AdamTable tab;
    tab.n = n_segs;
    uint64_t largest = 0;
    for (int i = 0; i < n_segs; i++) {
        tab.seg[i] = segs[i];
        largest = segs[i].n > largest ? segs[i].n : largest;
    }
    if (largest == 0) return cudaSuccess;
    int dev = 0, sms = 148;
    cudaGetDevice(&dev);
    cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
    const uint64_t want = (largest / 4 + 255) / 256 + 1;
    const uint64_t cap = static_cast<uint64_t>(sms) * 4;
    const dim3 grid(static_cast<unsigned>(want < cap ? want : cap), static_cast<unsigned>(n_segs));
    adam_kernel<<<grid, 256, 0, s>>>(tab);
    return cudaGetLastError();
}

// ---------------------------------------------------------------------------------------------------
// Data-parallel exchange fused with the sharded Adam: every rank holds the same flat parameter and gradient layout;
// rank r owns a contiguous slice. For each element of its slice the kernel sums the gradients of all ranks (peer
// loads over NVLink in rank order, or one multimem.ld_reduce through the NVSwitch when a multicast mapping exists),
// applies Adam to the local moments, and writes the new parameter into every rank's buffer (peer stores, or one
// multimem.st). It replaces reduce-scatter + Adam + all-gather; the caller fences it with a barrier on each side.

struct PeerTable {
    const float* grads[kMaxPeers];
    float* params[kMaxPeers];
    const float* local_params;
    const float* mc_grads;  // multicast addresses (nullptr: peer loads / stores)
    float* mc_params;
    int n;
};

__device__ inline float4 ld_reduce4(const float* a) {
    float4 r;
    asm volatile("multimem.ld_reduce.relaxed.sys.global.add.v4.f32 {%0, %1, %2, %3}, [%4];"
                 : "=f"(r.x), "=f"(r.y), "=f"(r.z), "=f"(r.w)
                 : "l"(a)
                 : "memory");
    return r;
}
__device__ inline void st_multi4(float* a, float4 v) {
    asm volatile("multimem.st.relaxed.sys.global.v4.f32 [%0], {%1, %2, %3, %4};" ::"l"(a), "f"(v.x), "f"(v.y), "f"(v.z), "f"(v.w) : "memory");
}
__device__ inline float ld_reduce1(const float* a) {
    float r;
    asm volatile("multimem.ld_reduce.relaxed.sys.global.add.f32 %0, [%1];" : "=f"(r) : "l"(a) : "memory");
    return r;
}
__device__ inline void st_multi1(float* a, float v) { asm volatile("multimem.st.relaxed.sys.global.f32 [%0], %1;" ::"l"(a), "f"(v) : "memory"); }

__global__ void __launch_bounds__(256) dp_shard_adam_kernel(const AdamTable tab, const PeerTable pt) {
    if (static_cast<int>(blockIdx.y) >= tab.n) return;
    const AdamSegment& S = tab.seg[blockIdx.y];
    const uint64_t base = static_cast<uint64_t>(S.param - pt.local_params);  // offset of the segment in the flat buffers
    const uint64_t stride = static_cast<uint64_t>(gridDim.x) * blockDim.x;
    const uint64_t tid = static_cast<uint64_t>(blockIdx.x) * blockDim.x + threadIdx.x;
    const uint32_t nl = static_cast<uint32_t>(S.n_lr);
    const bool mc = pt.mc_grads != nullptr;
    uint64_t done = 0;
    if ((base & 3u) == 0) {  // flat buffers are 16-byte aligned: four elements per thread
        const uint64_t n4 = S.n / 4;
        float4* P4 = reinterpret_cast<float4*>(S.param);
        float4* M4 = reinterpret_cast<float4*>(S.m);
        float4* V4 = reinterpret_cast<float4*>(S.v);
        for (uint64_t q = tid; q < n4; q += stride) {
            const uint64_t e = base + 4 * q;
            float4 g;
            if (mc) {
                g = ld_reduce4(pt.mc_grads + e);
            } else {
                g = reinterpret_cast<const float4*>(pt.grads[0] + e)[0];
                for (int r = 1; r < pt.n; r++) {
                    const float4 h = reinterpret_cast<const float4*>(pt.grads[r] + e)[0];
                    g = make_float4(g.x + h.x, g.y + h.y, g.z + h.z, g.w + h.w);
                }
            }
            float4 p = P4[q], m = M4[q], v = V4[q];
            uint32_t c = nl == 1 ? 0u : static_cast<uint32_t>((S.col_offset + 4 * q) % nl);
            adam_one(S, p.x, g.x, m.x, v.x, S.lr[c]);
            c = c + 1 == nl ? 0u : c + 1;
            adam_one(S, p.y, g.y, m.y, v.y, S.lr[c]);
            c = c + 1 == nl ? 0u : c + 1;
            adam_one(S, p.z, g.z, m.z, v.z, S.lr[c]);
            c = c + 1 == nl ? 0u : c + 1;
            adam_one(S, p.w, g.w, m.w, v.w, S.lr[c]);
            M4[q] = m;
            V4[q] = v;
            if (mc) {
                st_multi4(pt.mc_params + e, p);
            } else {
                for (int r = 0; r < pt.n; r++) reinterpret_cast<float4*>(pt.params[r] + e)[0] = p;
            }
        }
        done = 4 * n4;
    }
    for (uint64_t j = done + tid; j < S.n; j += stride) {
        const uint64_t e = base + j;
        float g;
        if (mc) {
            g = ld_reduce1(pt.mc_grads + e);
        } else {
            g = pt.grads[0][e];
            for (int r = 1; r < pt.n; r++) g += pt.grads[r][e];
        }
        float p = S.param[j];
        const uint32_t c = nl == 1 ? 0u : static_cast<uint32_t>((S.col_offset + j) % nl);
        adam_one(S, p, g, S.m[j], S.v[j], S.lr[c]);
        if (mc) st_multi1(pt.mc_params + e, p);
        else
            for (int r = 0; r < pt.n; r++) pt.params[r][e] = p;
    }
}

cudaError_t launch_dp_shard_adam(const AdamSegment* segs, int n_segs, const float* const* grads, float* const* params, int n_ranks,
                                 const float* local_params, const float* mc_grads, float* mc_params, cudaStream_t s) {
    if (n_segs <= 0) return cudaSuccess;
    if (n_segs > kMaxAdamSegments || n_ranks < 1 || n_ranks > kMaxPeers) return cudaErrorInvalidValue;
    AdamTable tab;
    tab.n = n_segs;
    uint64_t largest = 0;
    for (int i = 0; i < n_segs; i++) {
        tab.seg[i] = segs[i];
        largest = segs[i].n > largest ? segs[i].n : largest;
    }
    PeerTable pt{};
    for (int r = 0; r < n_ranks; r++) {
        pt.grads[r] = grads[r];
        pt.params[r] = params[r];
    }
    pt.n = n_ranks;
    pt.local_params = local_params;
    pt.mc_grads = mc_grads;
    pt.mc_params = mc_params;
    if (largest == 0) return cudaSuccess;
    int dev = 0, sms = 148;
    cudaGetDevice(&dev);
    cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
    const uint64_t want = (largest / 4 + 255) / 256 + 1;
    const uint64_t cap = static_cast<uint64_t>(sms) * 8;
    const dim3 grid(static_cast<unsigned>(want < cap ? want : cap), static_cast<unsigned>(n_segs));
    dp_shard_adam_kernel<<<grid, 256, 0, s>>>(tab, pt);
    return cudaGetLastError();
}

}  // namespace fgs
