// Training-loop helpers of the reference backend that sit around the rasterizer: the 3DGS-MCMC relocation
// adjustment and position noise, and the 3D (Mip-Splatting) filter update.
//
// Semantics:
//   relocation: FasterGSVDACudaBackend/.../densification/include/kernels_mcmc.cuh:10-54 (Eq. 9 of 3DGS-MCMC: a
//     primitive duplicated into N copies keeps its composite opacity, 1 - (1 - o')^N = o, and its scales are
//     rescaled by o / sum_{n<N} sum_{k<=n} C(n, k) (-1)^k o'^(k+1) / sqrt(k + 1); N clamped to [1, 50]);
//   noise: kernels_mcmc.cuh:64-146 (means += lr * s(o) * Sigma * z with Sigma = R diag(exp(2 s)) R^T, z three
//     standard normals from one Philox4x32-10 draw per primitive (counter (offset / 4, primitive), key = seed)
//     through Box-Muller, s(o) = 1 / (1 + exp(100 o - 0.5)) of the activated opacity o; primitives with a degenerate
//     quaternion are left unchanged);
//   3D filter: filter3d/src/filter3d.cu:11-90 (for points inside the view frustum with the clipping tolerance, the
//     filter becomes min(filter, distance2filter * depth) and the point is marked visible);
//   Morton codes of the means for the periodic reordering of the Gaussians (Model.py:449-453 with NeRFICG's
//     morton_encode, absent here): each coordinate quantised to 21 bits over the given box, bits interleaved x, y, z.
// The relocation coefficients are evaluated in double on the host and kept in each device's constant memory.
#include <curand_philox4x32_x.h>

#include <cmath>
#include <mutex>

#include "launch.h"

namespace fgs {

namespace {

constexpr int kMaxRelocationSamples = 50;

__constant__ float c_reloc[kMaxRelocationSamples * kMaxRelocationSamples];  // [n][k], k <= n

constexpr int kMaxDevices = 64;
std::mutex g_reloc_mutex;
bool g_reloc_ready[kMaxDevices] = {};

// C(n, k) (-1)^k / sqrt(k + 1) for n < 50, k <= n, copied once into the current device's constant memory (constant
// memory is per device)
cudaError_t upload_relocation_coefficients() {
    int dev = 0;
    cudaError_t e = cudaGetDevice(&dev);
    if (e != cudaSuccess) return e;
    if (dev < 0 || dev >= kMaxDevices) return cudaErrorInvalidDevice;
    std::lock_guard<std::mutex> lock(g_reloc_mutex);
    if (g_reloc_ready[dev]) return cudaSuccess;
    static float h[kMaxRelocationSamples * kMaxRelocationSamples];
    for (int n = 0; n < kMaxRelocationSamples; n++) {
        double binom = 1.0;
        for (int k = 0; k <= n; k++) {
            const double sign = (k & 1) ? -1.0 : 1.0;
            h[n * kMaxRelocationSamples + k] = static_cast<float>(sign * binom / std::sqrt(static_cast<double>(k + 1)));
            binom = binom * static_cast<double>(n - k) / static_cast<double>(k + 1);
        }
    }
    e = cudaMemcpyToSymbol(c_reloc, h, sizeof(h));
    if (e == cudaSuccess) g_reloc_ready[dev] = true;
    return e;
}

__global__ void __launch_bounds__(256) relocation_kernel(const float* __restrict__ old_opacity, const float* __restrict__ old_scale,
                                                         const int64_t* __restrict__ n_samples, float* __restrict__ new_opacity,
                                                         float* __restrict__ new_scale, uint32_t n) {
    const uint32_t i = blockIdx.x * blockDim.x + threadIdx.x;
    if (i >= n) return;
    const float o = old_opacity[i];
    const int64_t raw = n_samples[i];
    const int N = raw < 1 ? 1 : (raw > kMaxRelocationSamples ? kMaxRelocationSamples : static_cast<int>(raw));
    const float p = 1.0f - powf(1.0f - o, 1.0f / static_cast<float>(N));
    // sum over n < N of sum over k <= n of c[n][k] p^(k+1), rows in order
    float denom = 0.0f;
    for (int r = 0; r < N; r++) {
        float pk = p;
        for (int k = 0; k <= r; k++) {
            denom += c_reloc[r * kMaxRelocationSamples + k] * pk;
            pk *= p;
        }
    }
    const float f = o / denom;
    new_opacity[i] = p;
    new_scale[3ull * i] = f * old_scale[3ull * i];
    new_scale[3ull * i + 1] = f * old_scale[3ull * i + 1];
    new_scale[3ull * i + 2] = f * old_scale[3ull * i + 2];
}

// two standard normals from two 32-bit uniforms: u in (0, 1] from the first, the angle in [0, 2 pi) from the second
__device__ inline float2 box_muller(uint32_t bu, uint32_t bv) {
    const float u = fmaf(static_cast<float>(bu), 2.3283064365386963e-10f, 1.1641532182693481e-10f);
    const float radius = sqrtf(-2.0f * logf(u));
    float s, c;
    sincosf(static_cast<float>(bv) * 1.4629180792671596e-09f, &s, &c);
    return make_float2(radius * c, radius * s);
}

__global__ void __launch_bounds__(256) add_noise_kernel(const float* __restrict__ raw_scales, const float4* __restrict__ raw_rotations,
                                                        const float* __restrict__ raw_opacities, float* __restrict__ means, uint32_t n,
                                                        float lr, uint64_t seed, uint64_t offset) {
    const uint32_t i = blockIdx.x * blockDim.x + threadIdx.x;
    if (i >= n) return;
    const float4 q = raw_rotations[i];
    const float r = q.x, x = q.y, y = q.z, z = q.w;
    const float nsq = r * r + x * x + y * y + z * z;
    if (nsq < 1e-8f) return;
    const float s = 1.0f / nsq;
    // rotation (normalised quaternion) and covariance R diag(exp(2 scale)) R^T
    const float R11 = 1.0f - 2.0f * (y * y + z * z) * s, R12 = 2.0f * (x * y - r * z) * s, R13 = 2.0f * (x * z + r * y) * s;
    const float R21 = 2.0f * (x * y + r * z) * s, R22 = 1.0f - 2.0f * (x * x + z * z) * s, R23 = 2.0f * (y * z - r * x) * s;
    const float R31 = 2.0f * (x * z - r * y) * s, R32 = 2.0f * (y * z + r * x) * s, R33 = 1.0f - 2.0f * (x * x + y * y) * s;
    const float vx = expf(2.0f * raw_scales[3ull * i]), vy = expf(2.0f * raw_scales[3ull * i + 1]), vz = expf(2.0f * raw_scales[3ull * i + 2]);
    const float a11 = R11 * vx, a12 = R12 * vy, a13 = R13 * vz;  // rows of R diag(v)
    const float a21 = R21 * vx, a22 = R22 * vy, a23 = R23 * vz;
    const float a31 = R31 * vx, a32 = R32 * vy, a33 = R33 * vz;
    const float c11 = a11 * R11 + a12 * R12 + a13 * R13;
    const float c12 = a11 * R21 + a12 * R22 + a13 * R23;
    const float c13 = a11 * R31 + a12 * R32 + a13 * R33;
    const float c22 = a21 * R21 + a22 * R22 + a23 * R23;
    const float c23 = a21 * R31 + a22 * R32 + a23 * R33;
    const float c33 = a31 * R31 + a32 * R32 + a33 * R33;
    const uint64_t ctr = offset / 4;
    const uint4 bits = curand_Philox4x32_10(make_uint4(static_cast<uint32_t>(ctr), static_cast<uint32_t>(ctr >> 32), i, 0u),
                                            make_uint2(static_cast<uint32_t>(seed), static_cast<uint32_t>(seed >> 32)));
    const float2 nxy = box_muller(bits.x, bits.y);
    const float nz = box_muller(bits.z, bits.w).x;
    const float o = 1.0f / (1.0f + expf(-raw_opacities[i]));
    const float k = lr / (1.0f + expf(100.0f * o - 0.5f));
    means[3ull * i] += k * (c11 * nxy.x + c12 * nxy.y + c13 * nz);
    means[3ull * i + 1] += k * (c12 * nxy.x + c22 * nxy.y + c23 * nz);
    means[3ull * i + 2] += k * (c13 * nxy.x + c23 * nxy.y + c33 * nz);
}

__global__ void __launch_bounds__(256) filter3d_kernel(const float* __restrict__ pos, const float4* __restrict__ w2c, float* __restrict__ filter,
                                                       uint8_t* __restrict__ visible, uint32_t n, float left, float right, float top,
                                                       float bottom, float near_plane, float far_plane, float d2f) {
    const uint32_t i = blockIdx.x * blockDim.x + threadIdx.x;
    if (i >= n) return;
    const float px = pos[3ull * i], py = pos[3ull * i + 1], pz = pos[3ull * i + 2];
    const float4 r2 = w2c[2];
    const float depth = r2.x * px + r2.y * py + r2.z * pz + r2.w;
    if (depth < near_plane || depth > far_plane) return;
    const float4 r0 = w2c[0];
    const float xc = r0.x * px + r0.y * py + r0.z * pz + r0.w;
    if (xc < left * depth || xc > right * depth) return;
    const float4 r1 = w2c[1];
    const float yc = r1.x * px + r1.y * py + r1.z * pz + r1.w;
    if (yc < top * depth || yc > bottom * depth) return;
    const float f = d2f * depth;
    if (filter[i] < f) return;
    filter[i] = f;
    visible[i] = 1;
}

// 21 bits of x spread to every third bit of a 63-bit word
__device__ inline uint64_t spread3(uint64_t x) {
    x &= 0x1fffffull;
    x = (x | (x << 32)) & 0x1f00000000ffffull;
    x = (x | (x << 16)) & 0x1f0000ff0000ffull;
    x = (x | (x << 8)) & 0x100f00f00f00f00full;
    x = (x | (x << 4)) & 0x10c30c30c30c30c3ull;
    x = (x | (x << 2)) & 0x1249249249249249ull;
    return x;
}

__device__ inline uint64_t quantize21(float v, float lo, float scale) {
    const float q = (v - lo) * scale;  // [0, 2^21) inside the box
    return q <= 0.0f ? 0ull : (q >= 2097151.0f ? 2097151ull : static_cast<uint64_t>(q));
}

__global__ void __launch_bounds__(256) morton_kernel(const float* __restrict__ means, uint64_t* __restrict__ codes, uint32_t n, float3 lo,
                                                     float3 scale) {
    const uint32_t i = blockIdx.x * blockDim.x + threadIdx.x;
    if (i >= n) return;
    const uint64_t qx = quantize21(means[3ull * i], lo.x, scale.x);
    const uint64_t qy = quantize21(means[3ull * i + 1], lo.y, scale.y);
    const uint64_t qz = quantize21(means[3ull * i + 2], lo.z, scale.z);
    codes[i] = spread3(qx) | (spread3(qy) << 1) | (spread3(qz) << 2);
}

unsigned blocks_of(uint64_t n) { return static_cast<unsigned>((n + 255) / 256); }

}  // namespace

cudaError_t launch_relocation(const float* old_opacity, const float* old_scale, const int64_t* n_samples, float* new_opacity, float* new_scale,
                              uint32_t n, cudaStream_t s) {
    const cudaError_t e = upload_relocation_coefficients();
    if (e != cudaSuccess) return e;
    if (n == 0) return cudaSuccess;
    relocation_kernel<<<blocks_of(n), 256, 0, s>>>(old_opacity, old_scale, n_samples, new_opacity, new_scale, n);
    return cudaGetLastError();
}

cudaError_t launch_add_noise(const float* raw_scales, const float* raw_rotations, const float* raw_opacities, float* means, uint32_t n, float lr,
                             uint64_t seed, uint64_t offset, cudaStream_t s) {
    if (n == 0) return cudaSuccess;
    add_noise_kernel<<<blocks_of(n), 256, 0, s>>>(raw_scales, reinterpret_cast<const float4*>(raw_rotations), raw_opacities, means, n, lr, seed,
                                                  offset);
    return cudaGetLastError();
}

cudaError_t launch_morton(const float* means, uint64_t* codes, uint32_t n, const float lo[3], const float hi[3], cudaStream_t s) {
    if (n == 0) return cudaSuccess;
    float sc[3];
    for (int a = 0; a < 3; a++) {
        const float ext = hi[a] - lo[a];
        sc[a] = ext > 0.0f ? 2097152.0f / ext : 0.0f;
    }
    morton_kernel<<<blocks_of(n), 256, 0, s>>>(means, codes, n, make_float3(lo[0], lo[1], lo[2]), make_float3(sc[0], sc[1], sc[2]));
    return cudaGetLastError();
}

cudaError_t launch_filter3d(const float* positions, const float* w2c, float* filter, uint8_t* visible, uint32_t n, float left, float right,
                            float top, float bottom, float near_plane, float far_plane, float distance2filter, cudaStream_t s) {
    if (n == 0) return cudaSuccess;
    filter3d_kernel<<<blocks_of(n), 256, 0, s>>>(positions, reinterpret_cast<const float4*>(w2c), filter, visible, n, left, right, top, bottom,
                                                 near_plane, far_plane, distance2filter);
    return cudaGetLastError();
}

}  // namespace fgs
