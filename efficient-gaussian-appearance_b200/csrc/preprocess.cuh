// Launch-side declarations shared by the kernel translation units and the C-ABI layer.
#pragma once

#include "geometry.cuh"

namespace fgs {

constexpr int kChunk = 256;  // primitives per preprocess CTA (also the compaction granule)

struct AppearanceConfig {
    int model;          // Model enum
    int max_degree;     // SH degree / SV sites / lobes; neural: number of SH bands above 0
    int base_act, res_act, color_act;
    int dir_grad;
    // neural only
    int feature_dim;    // learned features per Gaussian
    int base_input;     // base colors appended to the encoder inputs
    int n_freq;         // frequency encoding octaves (0 = raw)
    int sh_mask;        // bit l set: SH band l is an MLP input
    int n_input;        // encoded feature dims + SH dims
    int n_input_pad;    // n_input rounded up to 16
    int n_neurons;      // hidden width
    int n_hidden;       // hidden layers (number of matmuls is n_hidden + 1)
    int n_output;       // 3
    int hidden_act;     // 0 none, 1 relu
    int n_params;       // total MLP weights
};

// pointer bundle of the per-Gaussian inputs
struct Params {
    const float* means;
    const float* scales;
    const float* rotations;
    const float* opacities;
    const float* precomputed;  // [N,3] or null
    const float* base;         // [N,3] or null
    const float* residual;     // [N, stride] or null
    const float* mlp;          // fp32 master MLP weights or null
    uint32_t n;
    unsigned char* mlp_act;    // training only: the tensor-core colour pass's hidden activations and raw outputs per
                               // 128-row tile, kept for the backward (null: not kept, the backward recomputes them)
};

// buffers of the primitive stage (all sized for N)
struct PrimBuffers {
    uint32_t* n_touched;   // [N]
    uint32_t* depth_key;   // [N]
    Record* rec;           // [N] records in primitive order (visible entries only)
    uint32_t* rank_of;     // [N] depth rank or kInvalidRank
    uint2* chunk_stats;    // [chunks] (visible, instances)
    uint32_t* chunk_off;   // [chunks] exclusive visible offsets
    uint32_t* group_vis;   // [chunks / 1024] visible sums, then their exclusive offsets
    unsigned long long* group_inst;  // [chunks / 1024] instance sums
    unsigned long long* counters;  // [0] visible, [1] instances
    uint32_t* keys_a; uint32_t* keys_b;
    uint32_t* idx_a;  uint32_t* idx_b;
    uint32_t* vis_idx;     // [V] visible primitives in primitive order (the compaction's list, kept past the depth sort)
    Record* sorted_rec;    // [V] records in depth order
    uint32_t* inst_off;    // [V] exclusive instance offsets in depth order
    void* sort_temp; size_t sort_temp_bytes;
    const uint32_t* sorted_idx;  // set after the depth sort (points at idx_a or idx_b)
    unsigned char* mlp_act; size_t mlp_act_bytes;  // tensor-core MLP activation store (training workspaces), or null
};

// gradient outputs of the backward preprocess
struct GradOut {
    float* means; float* scales; float* rotations; float* opacities;
    float* precomputed; float* base; float* residual;
    float* mlp;              // [n_params] fp32 MLP weight gradient (neural only)
    float* mlp_scratch;      // [n_params] fp32 zeroed accumulator (neural only)
    float* densification;    // [2 or 3, N] or null
    int densification_rows;
    int accumulate;          // add into the outputs instead of overwriting (multi-view accumulation)
};

}  // namespace fgs
