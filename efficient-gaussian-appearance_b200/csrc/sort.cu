// Stable key/value radix sorts and exclusive scans of the binning stage (CUB onesweep from the CUDA
// toolkit headers). Depth sort: 32-bit depth keys of the visible primitives
// (FasterGSVDACudaBackend/.../rasterization/src/forward.cu:88-97); tile sort: 16- or 32-bit tile keys over
// [0, end_bit) (forward.cu:182-191, key width rule forward.cu:139-140). Both sorts are stable, so the
// tile lists keep depth order and equal depth keys keep primitive order.
#include <cub/device/device_radix_sort.cuh>
#include <cub/device/device_scan.cuh>
#include "launch.h"

namespace fgs {

size_t depth_sort_temp_bytes(uint32_t n) {
    size_t bytes = 0;
    cub::DoubleBuffer<uint32_t> k(nullptr, nullptr), v(nullptr, nullptr);
    cub::DeviceRadixSort::SortPairs(nullptr, bytes, k, v, static_cast<int>(n), 0, 32);
    return bytes;
}

cudaError_t depth_sort(PrimBuffers& B, uint32_t n_visible, cudaStream_t s) {
    cub::DoubleBuffer<uint32_t> k(B.keys_a, B.keys_b), v(B.idx_a, B.idx_b);
    size_t bytes = B.cub_temp_bytes;
    cudaError_t e = cub::DeviceRadixSort::SortPairs(B.cub_temp, bytes, k, v, static_cast<int>(n_visible), 0, 32, s);
    B.sorted_idx = v.Current();
    return e;
}

size_t exclusive_scan_temp_bytes(uint32_t n) {
    size_t bytes = 0;
    cub::DeviceScan::ExclusiveSum(nullptr, bytes, static_cast<uint32_t*>(nullptr), static_cast<uint32_t*>(nullptr), static_cast<int>(n));
    return bytes;
}

cudaError_t exclusive_scan_u32(uint32_t* data, uint32_t n, void* temp, size_t temp_bytes, cudaStream_t s) {
    if (n == 0) return cudaSuccess;
    return cub::DeviceScan::ExclusiveSum(temp, temp_bytes, data, data, static_cast<int>(n), s);
}

template <typename K>
static size_t tile_temp(uint64_t n, int end_bit) {
    size_t bytes = 0;
    cub::DoubleBuffer<K> k(nullptr, nullptr);
    cub::DoubleBuffer<uint32_t> v(nullptr, nullptr);
    cub::DeviceRadixSort::SortPairs(nullptr, bytes, k, v, static_cast<int>(n), 0, end_bit);
    return bytes;
}

size_t tile_sort_temp_bytes(uint64_t n, int end_bit, bool wide) {
    return wide ? tile_temp<uint32_t>(n, end_bit) : tile_temp<uint16_t>(n, end_bit);
}

template <typename K>
static cudaError_t tile_sort_t(void* ka, void* kb, uint32_t* va, uint32_t* vb, uint64_t n, int end_bit, void* temp, size_t bytes,
                               const void** kout, const uint32_t** vout, cudaStream_t s) {
    cub::DoubleBuffer<K> k(static_cast<K*>(ka), static_cast<K*>(kb));
    cub::DoubleBuffer<uint32_t> v(va, vb);
    cudaError_t e = cudaSuccess;
    if (n > 0) e = cub::DeviceRadixSort::SortPairs(temp, bytes, k, v, static_cast<int>(n), 0, end_bit, s);
    *kout = k.Current();
    *vout = v.Current();
    return e;
}

cudaError_t tile_sort(void* keys_a, void* keys_b, uint32_t* vals_a, uint32_t* vals_b, uint64_t n, int end_bit, bool wide, void* temp,
                      size_t temp_bytes, const void** keys_out, const uint32_t** vals_out, cudaStream_t s) {
    if (wide) return tile_sort_t<uint32_t>(keys_a, keys_b, vals_a, vals_b, n, end_bit, temp, temp_bytes, keys_out, vals_out, s);
    return tile_sort_t<uint16_t>(keys_a, keys_b, vals_a, vals_b, n, end_bit, temp, temp_bytes, keys_out, vals_out, s);
}

}  // namespace fgs
