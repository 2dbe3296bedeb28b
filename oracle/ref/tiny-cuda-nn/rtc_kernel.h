// Test infrastructure only (the reference harness under oracle/, never the product path).
//
// Stand-in for tiny-cuda-nn's CudaRtcKernel, whose sources are absent from the reference checkout. The reference's
// host code (rasterization/include/rtc_preprocess.h:31-70, rasterization/src/backward.cu:101-131) only calls
// `launch(grid, block, shared_bytes, stream, args...)` on it; here the kernel is a function of a cubin that
// oracle/ref_build.py compiled with NVRTC from the reference's own preprocess sources, and launch passes the
// arguments to cuLaunchKernel exactly as given (each one by value, in order).
#pragma once

#include <cuda.h>
#include <cuda_runtime.h>

#include <cstdint>
#include <stdexcept>
#include <string>

namespace tcnn {

class CudaRtcKernel {
public:
    CudaRtcKernel(CUmodule module, CUfunction function) : module_(module), function_(function) {}
    ~CudaRtcKernel() { if (module_) cuModuleUnload(module_); }
    CudaRtcKernel(const CudaRtcKernel&) = delete;
    CudaRtcKernel& operator=(const CudaRtcKernel&) = delete;

    template <typename... Args>
    void launch(uint32_t grid, uint32_t block, uint32_t shared_bytes, cudaStream_t stream, Args... args) {
        if (grid == 0) return;
        void* params[] = {static_cast<void*>(&args)...};
        const CUresult r = cuLaunchKernel(function_, grid, 1, 1, block, 1, 1, shared_bytes, stream, params, nullptr);
        if (r != CUDA_SUCCESS) throw std::runtime_error("reference preprocess launch failed: CUresult " + std::to_string(static_cast<int>(r)));
    }

private:
    CUmodule module_;
    CUfunction function_;
};

}  // namespace tcnn
