/*
 * C-ABI of the B200-native fused-appearance Gaussian-splatting rasterizer (libfgs_b200.so).
 *
 * Plain pointers and sizes only: every tensor argument is a device pointer owned by the caller, every
 * workspace is a caller-allocated device buffer whose size the *_bytes queries return, and `stream` is a
 * cudaStream_t passed as void*. Functions return FGS_OK (0) or an error code; fgs_last_error() returns
 * the message of the last failure on the calling thread. Nothing throws across this boundary.
 *
 * The entry points replace the pybind module of the reference backend
 * (FasterGSVDACudaBackend/FasterGSVDACudaBackend/torch_bindings/bindings.cu:14-28):
 *   _C.Rasterizer / set_appearance / set_residual_mlp -> fgs_rasterizer_create, fgs_set_appearance, fgs_set_residual_mlp
 *   _C.forward   (rasterization/src/rasterization_api.cu:16-123)  -> fgs_forward_preprocess + fgs_forward_render
 *   _C.backward  (rasterization/src/rasterization_api.cu:125-247) -> fgs_backward
 *   _C.inference (rasterization/src/rasterization_api.cu:249-335) -> fgs_forward_preprocess + fgs_inference_render
 *   _C.pruning_scores (rasterization/src/rasterization_api.cu:337-416, src/pruning_scores.cu:11-204)
 *                     -> fgs_forward_preprocess + fgs_forward_render + fgs_pruning_scores
 *   _C.adam_step (adam/src/adam.cu:44-87)                          -> fgs_adam_step (several tensors per launch)
 *   _C.relocation_adjustment / _C.add_noise (densification/src/densification_api.cu:13-72)
 *                                                                  -> fgs_relocation_adjustment, fgs_add_noise
 *   _C.update_3d_filter (filter3d/src/filter3d.cu:43-90)           -> fgs_update_3d_filter
 * The reference's forward reads the visible-primitive and instance counts back to the host in the middle
 * of the call (rasterization/src/forward.cu:82-85) to size its buffers; here that point is the boundary
 * between fgs_forward_preprocess and fgs_forward_render, so the caller allocates the instance and bucket
 * workspaces in between.
 */
#ifndef FGS_B200_H
#define FGS_B200_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

enum {
    FGS_OK = 0,
    FGS_ERR_INVALID_ARGUMENT = 1,
    FGS_ERR_NOT_CONFIGURED = 2,
    FGS_ERR_UNSUPPORTED = 3,
    FGS_ERR_CUDA = 4,
    FGS_ERR_WORKSPACE = 5
};

/* appearance model ids (rasterization/include/appearance.h:110; torch_bindings/rasterization.py:21) */
enum { FGS_MODEL_PRECOMPUTED = 0, FGS_MODEL_SH = 1, FGS_MODEL_SV = 2, FGS_MODEL_NASG = 3, FGS_MODEL_NASGABOR = 4, FGS_MODEL_NEURAL = 5 };

typedef struct fgs_rasterizer fgs_rasterizer;

/* Per-Gaussian inputs, all fp32 device pointers, rows contiguous (replaces the tensor arguments of
 * rasterization.py:86-99). Unused appearance pointers are NULL. mlp_weights is the fp32 master copy;
 * the kernels round it to fp16 when staging (the reference casts with .half() in rasterization.py:101). */
typedef struct {
    const float* means;              /* [N,3] */
    const float* scales;             /* [N,3] log scales */
    const float* rotations;          /* [N,4] unnormalised quaternions (w,x,y,z) */
    const float* opacities;          /* [N,1] logits */
    const float* precomputed_colors; /* [N,3] or NULL */
    const float* base_colors;        /* [N,3] or NULL */
    const float* residual_params;    /* [N,R] or NULL */
    const float* mlp_weights;        /* [P] or NULL */
    int64_t n_primitives;
} fgs_primitives;

/* RasterizerSettings (torch_bindings/rasterization.py:49-83); w2c, cam_position and bg_color are
 * device pointers (16, 3 and 3 floats), the rest are values. */
typedef struct {
    const float* w2c;
    const float* cam_position;
    const float* bg_color;
    int appearance_degree;
    int width;
    int height;
    float focal_x;
    float focal_y;
    float center_x;
    float center_y;
    float near_plane;
    float far_plane;
    int proper_antialiasing;
    int render_base;
    int render_residual;
} fgs_settings;

/* Host-side record of one forward pass; filled by fgs_forward_preprocess / fgs_forward_render and read
 * by fgs_backward (replaces the (n_instances, n_buckets, selector) ints the reference returns). */
typedef struct {
    int64_t n_primitives;
    int64_t n_visible;
    int64_t n_instances;
    int64_t n_buckets;   /* upper bound n_instances / 32 + n_tiles, as in forward.cu:221 */
    int32_t width, height, grid_w, grid_h, end_bit, wide_keys;
    int32_t depth_selector;  /* which half of the depth double buffer holds the sorted indices */
    int32_t tile_selector;   /* which half of the tile double buffer holds the sorted instances */
    int32_t precomputed;
    int32_t mlp_activations; /* 1: fgs_forward_preprocess kept the tensor-core MLP's activations in the primitive
                                workspace, and fgs_backward reads them instead of recomputing the MLP forward */
} fgs_frame;

/* Gradient outputs (rasterization_api.cu:170-183). Arrays are overwritten (or added to when
 * `accumulate` is set); NULL entries that the model does not use are ignored. */
typedef struct {
    float* means;
    float* scales;
    float* rotations;
    float* opacities;
    float* precomputed_colors;
    float* base_colors;
    float* residual_params;
    float* mlp_weights;  /* fp32, unscaled */
} fgs_gradients;

/* Device pointers into the workspaces of a frame, for inspection and tests. */
typedef struct {
    const uint32_t* n_touched;     /* [N] tiles touched per primitive (0 = culled) */
    const uint32_t* depth_keys;    /* [N] float bits of the view depth (valid where n_touched > 0) */
    const uint32_t* sorted_indices;/* [V] primitive index per depth rank */
    const uint32_t* rank_of;       /* [N] depth rank per primitive or 0xffffffff */
    const void* sorted_records;    /* [V] 48-byte render records in depth order */
    const uint32_t* instance_offsets; /* [V] exclusive instance offsets in depth order */
    const void* instance_keys;     /* [I] tile index per instance, uint16 or uint32 (wide_keys) */
    const uint32_t* instance_ranks;/* [I] depth rank per instance */
    const uint32_t* tile_ranges;   /* [T][2] instance range per tile */
    const uint32_t* bucket_offsets;/* [T] inclusive bucket offsets */
    const uint32_t* tile_max_contributors; /* [T] */
    const float* final_transmittance;      /* [T*192] tile-local pixel order */
    const uint32_t* n_contributors;        /* [T*192] */
} fgs_frame_views;

typedef struct {
    float* param;
    const float* grad;
    float* exp_avg;
    float* exp_avg_sq;
    int64_t n_elements;
    int64_t column_offset;   /* index of param[0] within its tensor (selects the per-column learning rate) */
    int64_t step;            /* step count after this update (>= 1) */
    double learning_rates[7];
    int32_t n_learning_rates;/* 1..7, cycled per element */
    double beta1, beta2, eps;
} fgs_adam_segment;

const char* fgs_last_error(void);
int fgs_version(void);

/* _C.Rasterizer() and its set_appearance / set_residual_mlp (rasterization/src/appearance.cu:166-201) */
int fgs_rasterizer_create(fgs_rasterizer** out);
int fgs_rasterizer_destroy(fgs_rasterizer* r);
int fgs_set_appearance(fgs_rasterizer* r, int model, int max_degree, int base_activation, int residual_activation,
                       int color_activation, int direction_gradient);
/* tinycudann FullyFusedMLP with Identity encoding and no output activation (Appearance/Neural.py:40-51):
 * hidden_activation 0 = none, 1 = ReLU; sh_degree_mask bit l = SH band l is an input (rasterization.py:45) */
int fgs_set_residual_mlp(fgs_rasterizer* r, int n_input_dims, int n_output_dims, int n_neurons, int n_hidden_layers,
                         int hidden_activation, int base_input, int n_frequencies, int sh_degree_mask);
int fgs_mlp_param_count(const fgs_rasterizer* r, int64_t* out);
int fgs_residual_stride(const fgs_rasterizer* r, int64_t* out);

/* workspace sizes (the reference's grow-on-demand blobs, rasterization/include/buffer_utils.h:35-152).
 * The primitive workspace size for a rasterizer whose Neural MLP runs on the tensor cores includes a store for the
 * MLP's hidden activations (about 264 bytes per primitive for two 64-wide hidden layers); with r = NULL the size
 * excludes it, which suits a forward that no backward follows (inference, pruning scores). */
int fgs_primitive_workspace_bytes(const fgs_rasterizer* r, int64_t n_primitives, size_t* out);
int fgs_tile_workspace_bytes(int width, int height, size_t* out);
int fgs_instance_workspace_bytes(int64_t n_instances, int width, int height, size_t* out);
int fgs_bucket_workspace_bytes(int64_t n_buckets, size_t* out);
int fgs_gradient_workspace_bytes(const fgs_rasterizer* r, int64_t n_primitives, size_t* out);

/* forward, stage 1: preprocess with the fused appearance, order-preserving compaction of the visible
 * primitives, stable depth sort, depth-ordered render records and instance offsets. Synchronises
 * `stream` once to read the visible-primitive and instance counts into `frame`. */
int fgs_forward_preprocess(fgs_rasterizer* r, const fgs_primitives* prims, const fgs_settings* settings, void* prim_ws,
                           size_t prim_ws_bytes, void* stream, fgs_frame* frame);
/* forward, stage 2 (training): instance emission, stable tile sort, ranges, buckets, blend with
 * per-bucket checkpoints; image is [3,H,W] fp32 */
int fgs_forward_render(fgs_rasterizer* r, const fgs_settings* settings, fgs_frame* frame, void* prim_ws, void* tile_ws,
                       size_t tile_ws_bytes, void* inst_ws, size_t inst_ws_bytes, void* bucket_ws, size_t bucket_ws_bytes,
                       float* image, void* stream);
/* forward, stage 2 (inference): as above without checkpoints; image is [H,W,3] or [3,H,W] */
int fgs_inference_render(fgs_rasterizer* r, const fgs_settings* settings, fgs_frame* frame, void* prim_ws, void* tile_ws,
                         size_t tile_ws_bytes, void* inst_ws, size_t inst_ws_bytes, float* image, int to_chw, int clamp_output,
                         void* stream);
/* backward of a training forward. densification_info is [2 or 3, N] (updated in place) or NULL. */
int fgs_backward(fgs_rasterizer* r, const fgs_primitives* prims, const fgs_settings* settings, const fgs_frame* frame,
                 void* prim_ws, void* tile_ws, void* inst_ws, void* bucket_ws, void* grad_ws, size_t grad_ws_bytes,
                 const float* image, const float* grad_image, const fgs_gradients* grads, float* densification_info,
                 int densification_rows, int accumulate, void* stream);
int fgs_frame_buffers(const fgs_frame* frame, void* prim_ws, void* tile_ws, void* inst_ws, fgs_frame_views* out);
/* pruning scores of a training forward (image = its [3,H,W] output): scores[N] += sum over the accepted fragments
 * of each primitive of (opacity * dL/dalpha)^2 for an all-ones image gradient
 * (rasterization/include/kernels_pruning_scores.cuh:11-173) */
int fgs_pruning_scores(const fgs_settings* settings, const fgs_frame* frame, void* prim_ws, void* tile_ws, void* inst_ws,
                       const float* image, float* scores, void* stream);

/* fused Adam over up to 12 segments in one launch (adam/src/adam.cu:18-42 per element) */
int fgs_adam_step(const fgs_adam_segment* segments, int n_segments, void* stream);

/* 3DGS-MCMC relocation (densification/include/kernels_mcmc.cuh:10-54): for each of n primitives duplicated into
 * n_samples[i] copies (clamped to 1..50), the new opacity keeps the composite opacity and the scales are rescaled.
 * old_opacities [n] activated, old_scales [n,3] activated; outputs new_opacities [n], new_scales [n,3]. */
int fgs_relocation_adjustment(const float* old_opacities, const float* old_scales, const int64_t* n_samples, float* new_opacities,
                              float* new_scales, int64_t n, void* stream);
/* 3DGS-MCMC position noise, in place on means [n,3] (kernels_mcmc.cuh:64-146): raw (pre-activation) scales [n,3],
 * quaternions [n,4] (16-byte aligned) and opacity logits [n]; one Philox4x32-10 draw per primitive with counter
 * (offset / 4, primitive index) and key `seed` (the reference takes seed and offset from torch's CUDA generator). */
int fgs_add_noise(const float* raw_scales, const float* raw_rotations, const float* raw_opacities, float* means, int64_t n, float current_lr,
                  uint64_t seed, uint64_t offset, void* stream);
/* Morton codes of means [n,3] for reordering the Gaussians (Model.py:449-453 sorts by NeRFICG's morton_encode, which
 * is absent here): box_min / box_max are 3 host floats; each coordinate is quantised to 21 bits over the box and the
 * bits are interleaved (x lowest), giving codes [n] (uint64) to argsort. */
int fgs_morton_codes(const float* means, int64_t n, const float* box_min, const float* box_max, uint64_t* codes, void* stream);
/* 3D filter update of one view (filter3d/src/filter3d.cu:11-90): positions [n,3], w2c [4,4] row-major (16-byte
 * aligned), filter_3d [n] and visibility_mask [n] (bytes) updated in place. */
int fgs_update_3d_filter(const float* positions, const float* w2c, float* filter_3d, uint8_t* visibility_mask, int64_t n, int width, int height,
                         float focal_x, float focal_y, float center_x, float center_y, float near_plane, float far_plane,
                         float clipping_tolerance, float distance2filter, void* stream);

/* Data-parallel training (no reference counterpart: the reference trains on one GPU, Renderer.py:62-65): the
 * gradient reduce-scatter, the sharded Adam and the parameter all-gather of one step in one kernel over NVLink.
 * Every rank holds identically laid-out flat fp32 parameter and gradient buffers mapped into all ranks (symmetric
 * memory); `segments` describe this rank's slice (param / grad pointers inside the local buffers, moments local).
 * Each slice element sums the gradients of all ranks (rank order, peer loads; or multimem.ld_reduce through the
 * switch when multicast addresses are given), takes the Adam step and writes the parameter into every rank's
 * buffer (peer stores, or multimem.st). The caller places a cross-rank barrier before (all gradients final) and
 * after (all parameters written). */
#define FGS_MAX_PEERS 8
typedef struct fgs_peer_buffers {
    int n_ranks;                   /* 1..8 */
    const float* grads[FGS_MAX_PEERS];   /* every rank's flat gradient buffer as mapped on this device */
    float* params[FGS_MAX_PEERS];        /* every rank's flat parameter buffer as mapped on this device */
    const float* local_params;     /* this rank's parameter buffer (the segments' parameter pointers lie in it) */
    const float* multicast_grads;  /* multicast addresses of the two buffers, or both NULL */
    float* multicast_params;
} fgs_peer_buffers;
int fgs_dp_shard_adam(const fgs_adam_segment* segments, int n_segments, const fgs_peer_buffers* peers, void* stream);

/* Fused photometric loss of the training step and its image gradient: for planar [C,H,W] fp32 images,
 * loss = l1_weight * mean|image - target| + dssim_weight * (1 - mean SSIM(image, target)) with an 11x11 Gaussian
 * window (sigma 1.5, zero padding, C1 = 0.01^2, C2 = 0.03^2). Replaces the caller-side loss of the reference
 * trainer (FasterGSVDA/Loss.py:14-15: L1 plus NeRFICG's fused_dssim, weights LAMBDA_L1 / LAMBDA_DSSIM) so the
 * whole step stays on the device; `loss` is one device float, written deterministically. */
int fgs_loss_workspace_bytes(int channels, int height, int width, size_t* out);
int fgs_l1_dssim(const float* image, const float* target, int channels, int height, int width, float l1_weight, float dssim_weight,
                 float* grad_image, float* loss, void* workspace, size_t workspace_bytes, void* stream);

/* Diagnostics (no reference counterpart): runs three small tensor-core (tcgen05) GEMMs on the current device, one
 * per operand orientation the neural MLP kernels use, and compares them exactly with host results; *mismatches
 * receives the number of differing elements (0 = pass). `scratch` is a device buffer of FGS_TC_SELFTEST_FLOATS
 * floats. Synchronises the stream. */
#define FGS_TC_SELFTEST_FLOATS 14400
int fgs_tc_selftest(float* scratch, int* mismatches, void* stream);
/* (no reference counterpart) whether a tcgen05 MLP kernel on the current device gave up a bounded wait for its MMAs
 * since the flag was last cleared (its outputs are then invalid; fgs_forward_preprocess of a Neural configuration
 * also reports it as an error and clears it). Synchronous; clear != 0 resets the flag. */
int fgs_tc_timeout(int* timed_out, int clear);

/* Optional per-stage timing: while enabled, every stage above records a CUDA event pair on its stream;
 * fgs_profile_collect waits for them, returns the summed milliseconds per stage since the last collect
 * (names comma-separated in `names`) and resets the totals. No counterpart in the reference, which has
 * none (its timing is NeRFICG wall clock). */
int fgs_profile_enable(int enabled);
int fgs_profile_collect(char* names, size_t names_bytes, double* ms, int max_entries, int* n_entries);

/* Inference render that allocates nothing (no counterpart in the reference, which always allocates its buffers
 * with torch). For callers that cannot allocate device memory while they render, such as a viewer or engine plugin
 * running inside a host application that owns a fixed device-memory budget, where a cudaMalloc in the middle of a
 * frame may stall it or fail. All workspaces live in one static device array of FGS_NOALLOC_SCRATCH_BYTES that
 * every GPU loading the library holds until exit; inputs and the output image stay caller-owned. The call rejects,
 * with FGS_ERR_WORKSPACE and a message, any scene whose workspaces do not fit. The workspaces are those of
 * fgs_primitive_workspace_bytes(NULL, N) + fgs_tile_workspace_bytes(W, H) + fgs_instance_workspace_bytes(I, W, H):
 * about 132.3 bytes per primitive, 1552 bytes per 16x12 tile (8.1 per pixel) and 12.25 bytes per tile instance
 * (16.25 beyond 65536 tiles), each sub-buffer rounded up to 256 bytes; 100,000 primitives at 1280x720 leave room for
 * 1,000,000 tile instances. Each device's first call looks up the array's address (with that device current), so
 * make it before any stream capture; after cudaDeviceReset of a device the looked-up address is stale and this entry
 * point must not be called on that device again. A Neural colour pass that gave up a bounded wait is reported as
 * FGS_ERR_CUDA (and the flag cleared), never as an image. Calls share the array, which keeps the last call's
 * contents (every buffer a call reads is rewritten or cleared by it): calls that overlap on the GPU race. Output as
 * fgs_inference_render. */
#define FGS_NOALLOC_SCRATCH_BYTES (32u * 1024u * 1024u)
int fgs_inference_noalloc(fgs_rasterizer* r, const fgs_primitives* prims, const fgs_settings* settings, float* image, int to_chw,
                          int clamp_output, void* stream, int64_t* n_visible, int64_t* n_instances);

#ifdef __cplusplus
}
#endif

#endif /* FGS_B200_H */
