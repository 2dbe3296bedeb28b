// Host-side launchers of the kernel translation units (called by the C-ABI layer in capi.cu).
#pragma once

#include "preprocess.cuh"

namespace fgs {

struct GradOut;

// preprocess.cu
cudaError_t launch_preprocess_fwd(const Params& P, const AppearanceConfig& A, const View& v, const PrimBuffers& B, bool precomputed,
                                  cudaStream_t s);
cudaError_t launch_compaction(const PrimBuffers& B, uint32_t n, cudaStream_t s);
cudaError_t launch_reorder(const PrimBuffers& B, uint32_t n_visible, cudaStream_t s);
cudaError_t launch_preprocess_bwd(const Params& P, const AppearanceConfig& A, const View& v, const uint32_t* rank_of,
                                  const Record* sorted_rec, const GradRecord* grads, const GradOut& O, bool precomputed,
                                  const uint32_t* vis_idx, uint32_t n_visible, cudaStream_t s);

// neural.cu
// colour pass of the visible primitives (after the compaction): overwrites the colours the geometry pass wrote
cudaError_t launch_neural_color(const Params& P, const AppearanceConfig& A, const View& v, const uint32_t* vis_idx, uint32_t n_visible,
                                Record* rec, cudaStream_t s);
cudaError_t launch_preprocess_bwd_neural(const Params& P, const AppearanceConfig& A, const View& v, const uint32_t* rank_of,
                                         const Record* sorted_rec, const GradRecord* grads, const GradOut& O, const uint32_t* vis_idx,
                                         uint32_t n_visible, cudaStream_t s);
size_t neural_grad_scratch_floats(const AppearanceConfig& A);
size_t neural_smem_bytes(const AppearanceConfig& A);  // largest dynamic shared memory of the neural kernels

// sort.cu (depth sort, instance offsets, tile sort, scans)
size_t depth_sort_temp_bytes(uint32_t n);
cudaError_t depth_sort(PrimBuffers& B, uint32_t n_visible, cudaStream_t s);  // sets B.sorted_idx, fills B.inst_off via scan
size_t tile_sort_temp_bytes(uint64_t n_instances, int end_bit, bool wide);
cudaError_t tile_sort(void* keys_a, void* keys_b, uint32_t* vals_a, uint32_t* vals_b, uint64_t n, int end_bit, bool wide,
                      void* temp, size_t temp_bytes, const void** keys_out, const uint32_t** vals_out, cudaStream_t s);
cudaError_t exclusive_scan_u32(uint32_t* data, uint32_t n, void* temp, size_t temp_bytes, cudaStream_t s);
size_t exclusive_scan_temp_bytes(uint32_t n);

// binning.cu
struct TileBuffers {
    uint2* ranges;          // [T] instance range per tile
    uint32_t* bucket_off;   // [T] inclusive bucket offsets
    uint32_t* tile_max;     // [T] max contributor count per tile
    float* final_T;         // [T * 192] tile-local layout
    uint32_t* n_contrib;    // [T * 192]
};
cudaError_t launch_emit(const Record* sorted_rec, const uint32_t* inst_off, void* keys, uint32_t* vals, uint32_t n_visible,
                        int grid_w, bool wide, uint64_t n_instances, cudaStream_t s);
cudaError_t launch_ranges(const void* keys, uint64_t n_instances, bool wide, const TileBuffers& T, int n_tiles, cudaStream_t s);

// blend.cu
struct BlendArgs {
    const uint2* ranges;
    const uint32_t* bucket_off;
    const uint32_t* vals;        // instance -> depth rank
    const Record* rec;           // depth-ordered records
    const float* bg;
    int width, height, grid_w, grid_h;
};
cudaError_t launch_blend_train(const BlendArgs& a, float* image, const TileBuffers& T, cudaStream_t s);
cudaError_t launch_blend_inference(const BlendArgs& a, float* image, int chw, int clamp, cudaStream_t s);
cudaError_t launch_blend_backward(const BlendArgs& a, const float* image, const float* grad_image, const TileBuffers& T, GradRecord* grads,
                                  int abs_grad, cudaStream_t s);
cudaError_t launch_pruning_scores(const BlendArgs& a, const float* image, const TileBuffers& T, const uint32_t* rank_to_prim, float* scores,
                                  cudaStream_t s);

// loss.cu
size_t loss_workspace_bytes(int C, int H, int W);
cudaError_t launch_l1_dssim(const float* image, const float* target, int C, int H, int W, float l1_weight, float dssim_weight, float* grad,
                            float* loss, void* ws, cudaStream_t s);

// neural_tc.cu
bool tc_mlp_supported(const AppearanceConfig& A);  // 64-wide MLP with hidden layers: the tcgen05 kernels apply
size_t tc_mlp_smem_bytes(const AppearanceConfig& A);  // their largest dynamic shared memory (0 when unsupported)
// bytes of the activation store the tcgen05 colour pass fills for the backward (Params::mlp_act) for up to n_rows
// visible rows; 0 when the tcgen05 kernels do not apply
size_t tc_activation_bytes(const AppearanceConfig& A, uint64_t n_rows);
cudaError_t launch_tc_color(const Params& P, const AppearanceConfig& A, const View& v, const uint32_t* vis_idx, uint32_t n_visible,
                            Record* rec, cudaStream_t s);
// Activation store of a training workspace, per 128-row tile: the hidden activations, the raw outputs (4 halves per
// row) at outputs_off, and a row block at rows_off of kTcRowDataBytes per row that the geometry pass of the
// warp-specialised MLP backward fills: SH input chunks (2 x 16 bytes of fp16), the loss-scaled output gradient chunk
// (16 bytes), then primitive index, 1 / distance and the view direction (u32, 4 floats, padded to 32 bytes).
constexpr uint32_t kTcRowDataBytes = 80;
struct TcRowLayout {
    uint32_t tile_bytes, outputs_off, rows_off;
};
// whether launch_tc_backward runs the warp-specialised kernel for these inputs (training with an activation store,
// one octave, full SH input, no base input, 8 / 16 / 32 features, 16-byte aligned features and gradients); then *L
// is the store's layout
bool tc_ws_layout(const Params& P, const AppearanceConfig& A, const GradOut& O, TcRowLayout* L);
cudaError_t launch_tc_backward(const Params& P, const AppearanceConfig& A, const View& v, const uint32_t* vis_idx, uint32_t n_visible,
                               const uint32_t* rank_of, const Record* sorted_rec, const GradRecord* grads, const GradOut& O, cudaStream_t s);
constexpr int kTcSelftestFloats = 14400;
constexpr int kTcSelftestStatus = 14336;
cudaError_t tc_selftest(float* scratch, int* mismatches, cudaStream_t s);
// device address of the flag the tcgen05 kernels set when a bounded mbarrier wait ran out (their outputs are then
// invalid); it stays set until cleared
cudaError_t tc_timeout_flag(int** flag);

// adam.cu
struct AdamSegment {
    float* param; const float* grad; float* m; float* v;
    uint64_t n;            // elements
    uint64_t col_offset;   // index of the first element within its tensor (selects the per-column lr)
    float lr[7]; int n_lr;
    float beta1, beta2, eps, bc2_sqrt_rcp;
};
constexpr int kMaxAdamSegments = 12;
constexpr int kMaxPeers = 8;
cudaError_t launch_adam(const AdamSegment* segs, int n_segs, cudaStream_t s);
// sharded Adam fused with the gradient sum over all ranks and the parameter broadcast (peer memory / multicast)
cudaError_t launch_dp_shard_adam(const AdamSegment* segs, int n_segs, const float* const* grads, float* const* params, int n_ranks,
                                 const float* local_params, const float* mc_grads, float* mc_params, cudaStream_t s);

// densification.cu
cudaError_t launch_relocation(const float* old_opacity, const float* old_scale, const int64_t* n_samples, float* new_opacity, float* new_scale,
                              uint32_t n, cudaStream_t s);
cudaError_t launch_add_noise(const float* raw_scales, const float* raw_rotations, const float* raw_opacities, float* means, uint32_t n, float lr,
                             uint64_t seed, uint64_t offset, cudaStream_t s);
cudaError_t launch_morton(const float* means, uint64_t* codes, uint32_t n, const float lo[3], const float hi[3], cudaStream_t s);
cudaError_t launch_filter3d(const float* positions, const float* w2c, float* filter, uint8_t* visible, uint32_t n, float left, float right,
                            float top, float bottom, float near_plane, float far_plane, float distance2filter, cudaStream_t s);

}  // namespace fgs
