// Test infrastructure only: a C-ABI around the reference's own rasterizer, for parity tests on the GPU. Nothing in
// the product path links or loads it.
//
// oracle/ref_build.py compiles this file together with the reference's unmodified host and kernel sources
// (FasterGSVDACudaBackend/FasterGSVDACudaBackend/rasterization/src/forward.cu, backward.cu, inference.cu and the
// include/kernels_*.cuh they pull in) with the reference's nvcc flags, and compiles the reference's NVRTC preprocess
// kernels (rasterization/rtc/preprocess_forward.cu, preprocess_backward.cu with their appearance chunks) to cubins.
// The functions below do what the reference's torch glue does (rasterization/src/rasterization_api.cu:16-123,
// 125-247, 249-335): grow-on-demand device blobs for the four buffer groups, the AppearanceInputs /
// AppearanceGradients bundles, and one call of faster_gs::rasterization::forward / backward / inference. The neural
// model is not covered (its preprocess splices tiny-cuda-nn device functions that are absent).
#include <cuda.h>
#include <cuda_runtime.h>

#include <cstdint>
#include <cstring>
#include <exception>
#include <functional>
#include <memory>
#include <string>

#include "forward.h"
#include "backward.h"
#include "inference.h"
#include "buffer_utils.h"
#include "rasterization_config.h"
#include <tiny-cuda-nn/rtc_kernel.h>

namespace {

namespace R = faster_gs::rasterization;

thread_local std::string g_error;

struct Blob {
    char* ptr = nullptr;
    size_t size = 0;
    char* resize(size_t n) {
        if (n > size) {
            if (ptr) cudaFree(ptr);
            ptr = nullptr;
            size = 0;
            if (cudaMalloc(&ptr, n) != cudaSuccess) throw std::runtime_error("reference harness: cudaMalloc failed");
            size = n;
        }
        return ptr;
    }
    ~Blob() { if (ptr) cudaFree(ptr); }
};

struct RefRasterizer {
    std::unique_ptr<tcnn::CudaRtcKernel> forward_kernel, backward_kernel;
    Blob prim, tile, inst, bucket;
    int n_primitives = 0, n_instances = 0, n_buckets = 0, selector = 0, width = 0, height = 0;
};

int load_kernel(const void* image, const char* name, std::unique_ptr<tcnn::CudaRtcKernel>* out) {
    if (!image) return 0;
    CUmodule module = nullptr;
    CUfunction function = nullptr;
    CUresult r = cuModuleLoadData(&module, image);
    if (r != CUDA_SUCCESS) { g_error = "cuModuleLoadData failed: " + std::to_string(static_cast<int>(r)); return 1; }
    r = cuModuleGetFunction(&function, module, name);
    if (r != CUDA_SUCCESS) { cuModuleUnload(module); g_error = std::string("kernel not found: ") + name; return 1; }
    out->reset(new tcnn::CudaRtcKernel(module, function));
    return 0;
}

R::AppearanceInputs appearance_of(const float* precomputed, const float* base, const float* residual) {
    return R::AppearanceInputs{reinterpret_cast<const float3*>(precomputed), reinterpret_cast<const float3*>(base), residual, nullptr, nullptr,
                               nullptr};
}

template <typename F>
int guarded(F&& f) {
    try {
        f();
        const cudaError_t e = cudaGetLastError();
        if (e != cudaSuccess) { g_error = cudaGetErrorString(e); return 1; }
        return 0;
    } catch (const std::exception& e) {
        g_error = e.what();
        return 1;
    }
}

}  // namespace

extern "C" {

const char* ref_last_error(void) { return g_error.c_str(); }

// forward / backward preprocess cubins (either may be NULL) and their kernel names
int ref_create(const void* fwd_cubin, const char* fwd_name, const void* bwd_cubin, const char* bwd_name, void** out) {
    cudaFree(nullptr);  // the runtime's primary context becomes current for the driver-API module loads
    auto* r = new RefRasterizer();
    if (load_kernel(fwd_cubin, fwd_name, &r->forward_kernel) || load_kernel(bwd_cubin, bwd_name, &r->backward_kernel)) {
        delete r;
        return 1;
    }
    *out = r;
    return 0;
}

void ref_destroy(void* h) { delete static_cast<RefRasterizer*>(h); }

// training forward (rasterization_api.cu:16-123); counts[0..2] = n_instances, n_buckets, instance selector
int ref_forward(void* h, const float* means, const float* scales, const float* rotations, const float* opacities, const float* precomputed,
                const float* base, const float* residual, const float* w2c, const float* cam_position, const float* bg, float* image,
                int n_primitives, int appearance_degree, int width, int height, float fx, float fy, float cx, float cy, float near_plane,
                float far_plane, int proper_aa, int render_base, void* stream, int* counts) {
    auto* r = static_cast<RefRasterizer*>(h);
    return guarded([&] {
        std::function<char*(size_t)> rp = [r](size_t n) { return r->prim.resize(n); };
        std::function<char*(size_t)> rt = [r](size_t n) { return r->tile.resize(n); };
        std::function<char*(size_t)> ri = [r](size_t n) { return r->inst.resize(n); };
        std::function<char*(size_t)> rb = [r](size_t n) { return r->bucket.resize(n); };
        auto [ni, nb, sel] = R::forward(rp, rt, ri, rb, r->forward_kernel.get(), reinterpret_cast<const float3*>(means),
                                        reinterpret_cast<const float3*>(scales), reinterpret_cast<const float4*>(rotations), opacities,
                                        appearance_of(precomputed, base, residual), reinterpret_cast<const float4*>(w2c),
                                        reinterpret_cast<const float3*>(cam_position), reinterpret_cast<const float3*>(bg), image, n_primitives,
                                        appearance_degree, width, height, fx, fy, cx, cy, near_plane, far_plane, proper_aa != 0, render_base != 0,
                                        static_cast<cudaStream_t>(stream));
        r->n_primitives = n_primitives;
        r->n_instances = ni;
        r->n_buckets = nb;
        r->selector = sel;
        r->width = width;
        r->height = height;
        counts[0] = ni;
        counts[1] = nb;
        counts[2] = sel;
    });
}

// backward of the last forward (rasterization_api.cu:125-247); every output and helper buffer is caller-allocated
// with the reference's initialisation (helpers and grad_opacities zero)
int ref_backward(void* h, const float* grad_image, const float* means, const float* scales, const float* rotations, const float* opacities,
                 const float* precomputed, const float* base, const float* residual, const float* w2c, const float* cam_position, const float* bg,
                 const float* image, float* grad_mean2d_helper, float* grad_conic_helper, float* grad_mean2d_abs_helper, float* grad_color_helper,
                 float* grad_means, float* grad_scales, float* grad_rotations, float* grad_opacities, float* grad_precomputed, float* grad_base,
                 float* grad_residual, float* densification_info, int appearance_degree, float fx, float fy, float cx, float cy, int proper_aa,
                 int render_base, void* stream) {
    auto* r = static_cast<RefRasterizer*>(h);
    return guarded([&] {
        const R::AppearanceGradients ga{reinterpret_cast<float3*>(grad_precomputed), reinterpret_cast<float3*>(grad_base), grad_residual, nullptr};
        R::backward(r->backward_kernel.get(), grad_image, reinterpret_cast<const float3*>(means), reinterpret_cast<const float3*>(scales),
                    reinterpret_cast<const float4*>(rotations), opacities, appearance_of(precomputed, base, residual),
                    reinterpret_cast<const float4*>(w2c), reinterpret_cast<const float3*>(cam_position), reinterpret_cast<const float3*>(bg), image,
                    r->prim.ptr, r->tile.ptr, r->inst.ptr, r->bucket.ptr, reinterpret_cast<float2*>(grad_mean2d_helper), grad_conic_helper,
                    reinterpret_cast<float2*>(grad_mean2d_abs_helper), grad_color_helper, reinterpret_cast<float3*>(grad_means),
                    reinterpret_cast<float3*>(grad_scales), reinterpret_cast<float4*>(grad_rotations), grad_opacities, ga, densification_info,
                    r->n_primitives, r->n_instances, r->n_buckets, r->selector, 0, appearance_degree, r->width, r->height, fx, fy, cx, cy,
                    proper_aa != 0, render_base != 0, static_cast<cudaStream_t>(stream));
    });
}

// inference render (rasterization_api.cu:249-335); image is [H,W,3] or [3,H,W]
int ref_inference(void* h, const float* means, const float* scales, const float* rotations, const float* opacities, const float* precomputed,
                  const float* base, const float* residual, const float* w2c, const float* cam_position, const float* bg, float* image,
                  int n_primitives, int appearance_degree, int width, int height, float fx, float fy, float cx, float cy, float near_plane,
                  float far_plane, int proper_aa, int render_base, int to_chw, int clamp_output, void* stream) {
    auto* r = static_cast<RefRasterizer*>(h);
    return guarded([&] {
        std::function<char*(size_t)> rp = [r](size_t n) { return r->prim.resize(n); };
        std::function<char*(size_t)> rt = [r](size_t n) { return r->tile.resize(n); };
        std::function<char*(size_t)> ri = [r](size_t n) { return r->inst.resize(n); };
        R::inference(rp, rt, ri, r->forward_kernel.get(), reinterpret_cast<const float3*>(means), reinterpret_cast<const float3*>(scales),
                     reinterpret_cast<const float4*>(rotations), opacities, appearance_of(precomputed, base, residual),
                     reinterpret_cast<const float4*>(w2c), reinterpret_cast<const float3*>(cam_position), reinterpret_cast<const float3*>(bg), image,
                     n_primitives, appearance_degree, width, height, fx, fy, cx, cy, near_plane, far_plane, proper_aa != 0, render_base != 0,
                     to_chw != 0, clamp_output != 0, static_cast<cudaStream_t>(stream));
    });
}

// copies one buffer of the last training forward to host memory `dst` (`bytes` at most); returns the bytes copied
// or -1. which: 0 n_touched u32[N], 1 screen bounds ushort4[N], 2 mean2d float2[N], 3 conic+opacity float4[N],
// 4 color float3[N], 5 tile keys (u16 or u32)[I], 6 instance primitive indices u32[I] (tile-sorted), 7 tile ranges
// uint2[T], 8 final transmittance f32[T*192] (image order), 9 contributors u32[T*192] (image order), 10 per-tile max
// contributors u32[T], 11 counters uint2 (visible, instances)
long long ref_copy(void* h, int which, void* dst, size_t bytes) {
    auto* r = static_cast<RefRasterizer*>(h);
    const int tiles_x = (r->width + R::config::tile_width - 1) / R::config::tile_width;
    const int tiles_y = (r->height + R::config::tile_height - 1) / R::config::tile_height;
    const int n_tiles = tiles_x * tiles_y;
    const int end_bit = R::extract_end_bit(n_tiles - 1);
    char* pb = r->prim.ptr;
    char* tb = r->tile.ptr;
    char* ib = r->inst.ptr;
    R::PrimitiveBuffers P = R::PrimitiveBuffers::from_blob(pb, r->n_primitives);
    R::TileBuffers T = R::TileBuffers::from_blob(tb, n_tiles);
    const void* src = nullptr;
    size_t n = 0;
    const size_t N = static_cast<size_t>(r->n_primitives), I = static_cast<size_t>(r->n_instances);
    switch (which) {
        case 0: src = P.n_touched_tiles; n = N * 4; break;
        case 1: src = P.screen_bounds; n = N * 8; break;
        case 2: src = P.mean2d; n = N * 8; break;
        case 3: src = P.conic_opacity; n = N * 16; break;
        case 4: src = P.color; n = N * 12; break;
        case 5:
        case 6:
            if (end_bit <= 16) {
                auto B = R::InstanceBuffers<ushort>::from_blob(ib, r->n_instances, end_bit);
                B.keys.selector = r->selector;
                B.primitive_indices.selector = r->selector;
                src = which == 5 ? static_cast<const void*>(B.keys.Current()) : static_cast<const void*>(B.primitive_indices.Current());
                n = which == 5 ? I * 2 : I * 4;
            } else {
                auto B = R::InstanceBuffers<uint>::from_blob(ib, r->n_instances, end_bit);
                B.keys.selector = r->selector;
                B.primitive_indices.selector = r->selector;
                src = which == 5 ? static_cast<const void*>(B.keys.Current()) : static_cast<const void*>(B.primitive_indices.Current());
                n = I * 4;
            }
            break;
        case 7: src = T.instance_ranges; n = static_cast<size_t>(n_tiles) * 8; break;
        case 8: src = T.final_transmittances; n = static_cast<size_t>(r->width) * r->height * 4; break;
        case 9: src = T.n_processed; n = static_cast<size_t>(r->width) * r->height * 4; break;
        case 10: src = T.max_n_processed; n = static_cast<size_t>(n_tiles) * 4; break;
        case 11: src = P.counters; n = 8; break;
        default: g_error = "unknown buffer"; return -1;
    }
    if (n > bytes) { g_error = "destination too small"; return -1; }
    if (n == 0) return 0;
    if (cudaMemcpy(dst, src, n, cudaMemcpyDeviceToHost) != cudaSuccess) { g_error = "copy failed"; return -1; }
    return static_cast<long long>(n);
}

}  // extern "C"
