// C-ABI entry points (include/fgs_b200.h): argument checking, workspace layout, and the stage order of
// the reference's forward / backward / inference host code (FasterGSVDACudaBackend/.../rasterization/
// src/forward.cu:11-246, backward.cu:8-135, inference.cu:11-140, rasterization_api.cu:16-335).
#include <cmath>
#include <cstdio>
#include <cstring>
#include <mutex>
#include <string>
#include <vector>
#include <utility>
#include "../../include/fgs_b200.h"
#include "launch.h"
#include "appearance.cuh"

struct fgs_rasterizer {
    fgs::AppearanceConfig cfg;
    bool appearance_set = false;
    bool mlp_set = false;
};

namespace {

thread_local std::string g_last_error;

int fail(int code, const std::string& msg) {
    g_last_error = msg;
    return code;
}

int cuda_fail(cudaError_t e, const char* where) {
    return fail(FGS_ERR_CUDA, std::string(where) + ": " + cudaGetErrorString(e));
}

#define FGS_CUDA(call, where)                        \
    do {                                             \
        cudaError_t e_ = (call);                     \
        if (e_ != cudaSuccess) return cuda_fail(e_, where); \
    } while (0)

// carves 256-byte aligned sub-buffers out of a workspace; with base == nullptr it only measures
struct Carver {
    char* base;
    size_t off = 0;
    explicit Carver(void* b) : base(static_cast<char*>(b)) {}
    template <typename T>
    T* take(size_t count) {
        off = (off + 255) & ~static_cast<size_t>(255);
        T* p = base ? reinterpret_cast<T*>(base + off) : nullptr;
        off += count * sizeof(T);
        return p;
    }
};

int end_bit_of(uint32_t n) {
    int bits = 0;
    while (n) { bits++; n >>= 1; }
    return bits;
}

struct Grid {
    int gw, gh, tiles, end_bit;
    bool wide;
};
Grid grid_of(int width, int height) {
    Grid g;
    g.gw = (width + fgs::kTileW - 1) / fgs::kTileW;
    g.gh = (height + fgs::kTileH - 1) / fgs::kTileH;
    g.tiles = g.gw * g.gh;
    g.end_bit = end_bit_of(static_cast<uint32_t>(g.tiles > 0 ? g.tiles - 1 : 0));
    g.wide = g.end_bit > 16;
    return g;
}

fgs::PrimBuffers carve_prim(void* ws, uint64_t n, size_t* bytes, size_t act_bytes = 0) {
    Carver c(ws);
    const uint64_t chunks = (n + fgs::kChunk - 1) / fgs::kChunk;
    fgs::PrimBuffers B{};
    B.n_touched = c.take<uint32_t>(n);
    B.depth_key = c.take<uint32_t>(n);
    B.rec = c.take<fgs::Record>(n);
    B.rank_of = c.take<uint32_t>(n);
    B.chunk_stats = c.take<uint2>(chunks);
    B.chunk_off = c.take<uint32_t>(chunks);
    B.group_vis = c.take<uint32_t>((chunks + 1023) / 1024);
    B.group_inst = c.take<unsigned long long>((chunks + 1023) / 1024);
    B.counters = c.take<unsigned long long>(2);
    B.keys_a = c.take<uint32_t>(n);
    B.keys_b = c.take<uint32_t>(n);
    B.idx_a = c.take<uint32_t>(n);
    B.idx_b = c.take<uint32_t>(n);
    B.vis_idx = c.take<uint32_t>(n);
    B.sorted_rec = c.take<fgs::Record>(n);
    B.inst_off = c.take<uint32_t>(n);
    size_t tb = fgs::depth_sort_temp_bytes(static_cast<uint32_t>(n));
    const size_t sb = fgs::exclusive_scan_temp_bytes(static_cast<uint32_t>(n));
    if (sb > tb) tb = sb;
    B.sort_temp = c.take<char>(tb);
    B.sort_temp_bytes = tb;
    // the tensor-core MLP's activation store (training workspaces) comes last, so every other buffer keeps its offset
    B.mlp_act = act_bytes ? c.take<unsigned char>(act_bytes) : nullptr;
    B.mlp_act_bytes = act_bytes;
    if (bytes) *bytes = c.off;
    return B;
}

// bytes of the activation store for n primitives: nonzero only for a Neural MLP that runs on the tcgen05 kernels
size_t mlp_act_bytes(const fgs_rasterizer* r, uint64_t n) {
    if (!r || !r->appearance_set || !r->mlp_set || r->cfg.model != fgs::kNeural) return 0;
    return fgs::tc_activation_bytes(r->cfg, n);
}

fgs::TileBuffers carve_tile(void* ws, const Grid& g, size_t* bytes) {
    Carver c(ws);
    fgs::TileBuffers T{};
    T.ranges = c.take<uint2>(g.tiles);
    T.bucket_off = c.take<uint32_t>(g.tiles);
    T.tile_max = c.take<uint32_t>(g.tiles);
    T.final_T = c.take<float>(static_cast<size_t>(g.tiles) * fgs::kTilePixels);
    T.n_contrib = c.take<uint32_t>(static_cast<size_t>(g.tiles) * fgs::kTilePixels);
    if (bytes) *bytes = c.off;
    return T;
}

struct InstBuffers {
    void* keys_a; void* keys_b;
    uint32_t* vals_a; uint32_t* vals_b;
    void* temp; size_t temp_bytes;
};
InstBuffers carve_inst(void* ws, uint64_t n, const Grid& g, size_t* bytes) {
    Carver c(ws);
    InstBuffers I{};
    const size_t ks = g.wide ? 4 : 2;
    I.keys_a = c.take<char>(n * ks);
    I.keys_b = c.take<char>(n * ks);
    I.vals_a = c.take<uint32_t>(n);
    I.vals_b = c.take<uint32_t>(n);
    I.temp_bytes = fgs::tile_sort_temp_bytes(n, g.end_bit > 0 ? g.end_bit : 1, g.wide);
    I.temp = c.take<char>(I.temp_bytes);
    if (bytes) *bytes = c.off;
    return I;
}

struct GradBuffers { fgs::GradRecord* rec; float* mlp_scratch; };
GradBuffers carve_grad(void* ws, uint64_t n, uint64_t n_mlp, size_t* bytes) {
    Carver c(ws);
    GradBuffers g{};
    g.rec = c.take<fgs::GradRecord>(n);
    g.mlp_scratch = c.take<float>(n_mlp);
    if (bytes) *bytes = c.off;
    return g;
}

int check_settings(const fgs_settings* s) {
    if (!s) return fail(FGS_ERR_INVALID_ARGUMENT, "settings is NULL");
    if (!s->w2c || !s->cam_position || !s->bg_color) return fail(FGS_ERR_INVALID_ARGUMENT, "w2c, cam_position and bg_color are required");
    if (s->width <= 0 || s->height <= 0 || s->width > 65535 - 16 || s->height > 65535 - 12)
        return fail(FGS_ERR_INVALID_ARGUMENT, "image size must be in [1, 65519] x [1, 65523]");
    if (s->appearance_degree < 0) return fail(FGS_ERR_INVALID_ARGUMENT, "appearance_degree must be >= 0");
    return FGS_OK;
}

fgs::View make_view(const fgs_settings* s) {
    const Grid g = grid_of(s->width, s->height);
    fgs::View v;
    v.w2c = s->w2c;
    v.cam_pos = s->cam_position;
    v.bg = s->bg_color;
    v.width = s->width;
    v.height = s->height;
    v.fx = s->focal_x; v.fy = s->focal_y; v.cx = s->center_x; v.cy = s->center_y;
    v.near_plane = s->near_plane;
    v.far_plane = s->far_plane;
    v.grid_w = g.gw;
    v.grid_h = g.gh;
    v.proper_aa = s->proper_antialiasing ? 1 : 0;
    v.render_base = s->render_base ? 1 : 0;
    v.degree = s->render_residual ? s->appearance_degree : 0;
    return v;
}

int check_prims(const fgs_rasterizer* r, const fgs_primitives* p, bool* precomputed) {
    if (!p) return fail(FGS_ERR_INVALID_ARGUMENT, "primitives is NULL");
    if (p->n_primitives < 0 || p->n_primitives > 0x7fffff00LL) return fail(FGS_ERR_INVALID_ARGUMENT, "n_primitives out of range");
    if (p->n_primitives > 0 && (!p->means || !p->scales || !p->rotations || !p->opacities))
        return fail(FGS_ERR_INVALID_ARGUMENT, "means, scales, rotations and opacities are required");
    if (reinterpret_cast<uintptr_t>(p->rotations) % 16 != 0) return fail(FGS_ERR_INVALID_ARGUMENT, "rotations must be 16-byte aligned");
    *precomputed = p->precomputed_colors != nullptr;
    if (*precomputed) return FGS_OK;
    if (!r->appearance_set) return fail(FGS_ERR_NOT_CONFIGURED, "FasterGSVDA: appearance model is not initialized");
    if (r->cfg.model == fgs::kNeural && !r->mlp_set) return fail(FGS_ERR_NOT_CONFIGURED, "FasterGSVDA: residual mlp is not initialized");
    if (p->n_primitives > 0 && !p->base_colors) return fail(FGS_ERR_INVALID_ARGUMENT, "base_colors is required by the fused appearance");
    const int stride = fgs::residual_stride(r->cfg.model, r->cfg.max_degree, r->cfg.feature_dim);
    if (p->n_primitives > 0 && stride > 0 && !p->residual_params) return fail(FGS_ERR_INVALID_ARGUMENT, "residual_params is required");
    if (r->cfg.model == fgs::kNeural && !p->mlp_weights) return fail(FGS_ERR_INVALID_ARGUMENT, "mlp_weights is required");
    return FGS_OK;
}

fgs::Params make_params(const fgs_primitives* p) {
    fgs::Params P;
    P.means = p->means; P.scales = p->scales; P.rotations = p->rotations; P.opacities = p->opacities;
    P.precomputed = p->precomputed_colors; P.base = p->base_colors; P.residual = p->residual_params; P.mlp = p->mlp_weights;
    P.n = static_cast<uint32_t>(p->n_primitives);
    P.mlp_act = nullptr;
    return P;
}

// ---- optional per-stage timing with CUDA events on the launching stream (off unless enabled) ----
struct ProfEntry { const char* name; cudaEvent_t start, stop; };
struct Prof {
    bool enabled = false;
    std::vector<ProfEntry> pending;
    std::vector<std::pair<std::string, double>> totals;
    std::vector<cudaEvent_t> pool;
    cudaEvent_t get() {
        if (!pool.empty()) { cudaEvent_t e = pool.back(); pool.pop_back(); return e; }
        cudaEvent_t e;
        cudaEventCreate(&e);
        return e;
    }
};
Prof g_prof;

struct ProfScope {
    cudaStream_t s;
    ProfEntry e{};
    bool on;
    ProfScope(const char* name, cudaStream_t st) : s(st), on(g_prof.enabled) {
        if (!on) return;
        e.name = name;
        e.start = g_prof.get();
        e.stop = g_prof.get();
        cudaEventRecord(e.start, s);
    }
    ~ProfScope() {
        if (!on) return;
        cudaEventRecord(e.stop, s);
        g_prof.pending.push_back(e);
    }
};

unsigned long long* pinned_counters() {
    static thread_local unsigned long long* host = nullptr;
    if (!host) {
        if (cudaMallocHost(&host, 4 * sizeof(unsigned long long)) != cudaSuccess) host = nullptr;
    }
    return host;
}

}  // namespace

extern "C" {

const char* fgs_last_error(void) { return g_last_error.c_str(); }
int fgs_version(void) { return 1; }

int fgs_rasterizer_create(fgs_rasterizer** out) {
    if (!out) return fail(FGS_ERR_INVALID_ARGUMENT, "out is NULL");
    *out = new fgs_rasterizer();
    std::memset(&(*out)->cfg, 0, sizeof(fgs::AppearanceConfig));
    return FGS_OK;
}

int fgs_rasterizer_destroy(fgs_rasterizer* r) {
    delete r;
    return FGS_OK;
}

int fgs_set_appearance(fgs_rasterizer* r, int model, int max_degree, int base_act, int res_act, int color_act, int dir_grad) {
    if (!r) return fail(FGS_ERR_INVALID_ARGUMENT, "rasterizer is NULL");
    if (model < 1 || model > 5) return fail(FGS_ERR_INVALID_ARGUMENT, "FasterGSVDA: invalid appearance model id");
    if (base_act < 0 || base_act > 1) return fail(FGS_ERR_INVALID_ARGUMENT, "FasterGSVDA: invalid base activation id");
    if (res_act < 0 || res_act > 2) return fail(FGS_ERR_INVALID_ARGUMENT, "FasterGSVDA: invalid residual activation id");
    if (color_act < 0 || color_act > 5) return fail(FGS_ERR_INVALID_ARGUMENT, "FasterGSVDA: invalid color activation id");
    if (model == fgs::kSH && (max_degree < 0 || max_degree > 3)) return fail(FGS_ERR_UNSUPPORTED, "SH degree must be in [0, 3]");
    if ((model == fgs::kSV || model == fgs::kNASG || model == fgs::kNASGabor) && (max_degree < 0 || max_degree > 10))
        return fail(FGS_ERR_UNSUPPORTED, "sites / lobes must be in [0, 10]");
    std::memset(&r->cfg, 0, sizeof(fgs::AppearanceConfig));
    r->cfg.model = model;
    r->cfg.max_degree = model == fgs::kNeural ? 0 : max_degree;
    r->cfg.base_act = base_act;
    r->cfg.res_act = res_act;
    r->cfg.color_act = color_act;
    r->cfg.dir_grad = dir_grad ? 1 : 0;
    r->appearance_set = true;
    r->mlp_set = false;
    return FGS_OK;
}

int fgs_set_residual_mlp(fgs_rasterizer* r, int n_input, int n_output, int n_neurons, int n_hidden, int hidden_act, int base_input,
                         int n_freq, int sh_mask) {
    if (!r) return fail(FGS_ERR_INVALID_ARGUMENT, "rasterizer is NULL");
    if (!r->appearance_set || r->cfg.model != fgs::kNeural)
        return fail(FGS_ERR_NOT_CONFIGURED, "FasterGSVDA: set_appearance must select the neural appearance model before set_residual_mlp");
    if (n_output != 3) return fail(FGS_ERR_UNSUPPORTED, "the residual mlp must have 3 outputs");
    if (n_neurons != 16 && n_neurons != 32 && n_neurons != 64) return fail(FGS_ERR_UNSUPPORTED, "n_neurons must be 16, 32 or 64");
    if (n_hidden < 1 || n_hidden > 8) return fail(FGS_ERR_UNSUPPORTED, "n_hidden_layers must be in [1, 8]");
    if (hidden_act < 0 || hidden_act > 1) return fail(FGS_ERR_UNSUPPORTED, "hidden activation must be None or ReLU");
    if (n_freq < 0 || n_freq > 8) return fail(FGS_ERR_UNSUPPORTED, "n_frequencies must be in [0, 8]");
    if (sh_mask < 0 || sh_mask >= (1 << 4)) return fail(FGS_ERR_UNSUPPORTED, "SH degrees of the direction encoding must be in [0, 3]");
    int n_sh = 0, bands = 0;
    for (int l = 0; l <= 6; l++)
        if (sh_mask & (1 << l)) { n_sh += 2 * l + 1; if (l > 0) bands++; }
    const int enc = n_input - n_sh;
    const int per = n_freq > 0 ? 2 * n_freq : 1;
    if (enc <= 0 || enc % per != 0) return fail(FGS_ERR_INVALID_ARGUMENT, "n_input_dims does not match the encoding");
    const int raw = enc / per;
    const int feat = raw - (base_input ? 3 : 0);
    if (feat <= 0) return fail(FGS_ERR_INVALID_ARGUMENT, "no learned features left after base_input");
    const int pad = (n_input + 15) / 16 * 16;
    if (pad > 128) return fail(FGS_ERR_UNSUPPORTED, "padded mlp input width must be <= 128");
    r->cfg.feature_dim = feat;
    r->cfg.base_input = base_input ? 1 : 0;
    r->cfg.n_freq = n_freq;
    r->cfg.sh_mask = sh_mask;
    r->cfg.n_input = n_input;
    r->cfg.n_input_pad = pad;
    r->cfg.n_neurons = n_neurons;
    r->cfg.n_hidden = n_hidden;
    r->cfg.n_output = n_output;
    r->cfg.hidden_act = hidden_act;
    r->cfg.max_degree = bands;
    r->cfg.n_params = n_neurons * pad + (n_hidden - 1) * n_neurons * n_neurons + 16 * n_neurons;
    if (fgs::neural_smem_bytes(r->cfg) > 227 * 1024) {
        r->mlp_set = false;
        return fail(FGS_ERR_UNSUPPORTED, "residual mlp too large for the fused kernels' shared memory (" + std::to_string(fgs::neural_smem_bytes(r->cfg)) +
                                             " bytes > 227 KiB); reduce n_input_dims, n_neurons or n_hidden_layers");
    }
    r->mlp_set = true;
    return FGS_OK;
}

int fgs_mlp_param_count(const fgs_rasterizer* r, int64_t* out) {
    if (!r || !out) return fail(FGS_ERR_INVALID_ARGUMENT, "NULL argument");
    *out = r->mlp_set ? r->cfg.n_params : 0;
    return FGS_OK;
}

int fgs_residual_stride(const fgs_rasterizer* r, int64_t* out) {
    if (!r || !out) return fail(FGS_ERR_INVALID_ARGUMENT, "NULL argument");
    *out = r->appearance_set ? fgs::residual_stride(r->cfg.model, r->cfg.max_degree, r->cfg.feature_dim) : 0;
    return FGS_OK;
}

int fgs_primitive_workspace_bytes(const fgs_rasterizer* r, int64_t n, size_t* out) {
    if (!out || n < 0) return fail(FGS_ERR_INVALID_ARGUMENT, "bad argument");
    carve_prim(nullptr, static_cast<uint64_t>(n), out, mlp_act_bytes(r, static_cast<uint64_t>(n)));
    return FGS_OK;
}

int fgs_tile_workspace_bytes(int width, int height, size_t* out) {
    if (!out || width <= 0 || height <= 0) return fail(FGS_ERR_INVALID_ARGUMENT, "bad argument");
    carve_tile(nullptr, grid_of(width, height), out);
    return FGS_OK;
}

int fgs_instance_workspace_bytes(int64_t n, int width, int height, size_t* out) {
    if (!out || n < 0 || width <= 0 || height <= 0) return fail(FGS_ERR_INVALID_ARGUMENT, "bad argument");
    if (n > 0x7fffff00LL) return fail(FGS_ERR_UNSUPPORTED, "more than 2^31 instances");
    carve_inst(nullptr, static_cast<uint64_t>(n), grid_of(width, height), out);
    return FGS_OK;
}

int fgs_bucket_workspace_bytes(int64_t n, size_t* out) {
    if (!out || n < 0) return fail(FGS_ERR_INVALID_ARGUMENT, "bad argument");
    *out = 0;  // the backward re-derives fragments per pixel; no per-bucket checkpoints are stored
    return FGS_OK;
}

int fgs_gradient_workspace_bytes(const fgs_rasterizer* r, int64_t n, size_t* out) {
    if (!out || n < 0) return fail(FGS_ERR_INVALID_ARGUMENT, "bad argument");
    const uint64_t n_mlp = (r && r->mlp_set) ? fgs::neural_grad_scratch_floats(r->cfg) : 0;
    carve_grad(nullptr, static_cast<uint64_t>(n), n_mlp, out);
    return FGS_OK;
}

int fgs_forward_preprocess(fgs_rasterizer* r, const fgs_primitives* prims, const fgs_settings* settings, void* prim_ws, size_t prim_ws_bytes,
                           void* stream, fgs_frame* frame) {
    if (!r || !frame) return fail(FGS_ERR_INVALID_ARGUMENT, "NULL argument");
    int rc = check_settings(settings);
    if (rc) return rc;
    bool precomputed = false;
    rc = check_prims(r, prims, &precomputed);
    if (rc) return rc;
    const uint64_t n = static_cast<uint64_t>(prims->n_primitives);
    // a workspace that also covers the activation store (the size fgs_primitive_workspace_bytes gives for this
    // rasterizer) keeps the tensor-core MLP's activations for fgs_backward
    const size_t act_bytes = precomputed ? 0 : mlp_act_bytes(r, n);
    size_t need = 0, need_act = 0;
    carve_prim(nullptr, n, &need_act, act_bytes);
    const bool keep_act = act_bytes > 0 && prim_ws && prim_ws_bytes >= need_act;
    fgs::PrimBuffers B = carve_prim(prim_ws, n, &need, keep_act ? act_bytes : 0);
    if (!prim_ws || prim_ws_bytes < need) return fail(FGS_ERR_WORKSPACE, "primitive workspace too small");
    cudaStream_t s = static_cast<cudaStream_t>(stream);
    const fgs::View v = make_view(settings);
    fgs::Params P = make_params(prims);
    P.mlp_act = keep_act ? B.mlp_act : nullptr;
    const Grid g = grid_of(settings->width, settings->height);
    std::memset(frame, 0, sizeof(fgs_frame));
    frame->n_primitives = static_cast<int64_t>(n);
    frame->width = settings->width;
    frame->height = settings->height;
    frame->grid_w = g.gw;
    frame->grid_h = g.gh;
    frame->end_bit = g.end_bit;
    frame->wide_keys = g.wide ? 1 : 0;
    frame->precomputed = precomputed ? 1 : 0;
    frame->mlp_activations = keep_act ? 1 : 0;
    if (n == 0) return FGS_OK;
    {
        ProfScope p_("preprocess", s);
        FGS_CUDA(fgs::launch_preprocess_fwd(P, r->cfg, v, B, precomputed, s), "preprocess");
    }
    {
        ProfScope p_("compaction", s);
        FGS_CUDA(fgs::launch_compaction(B, static_cast<uint32_t>(n), s), "compaction");
    }
    unsigned long long* host = pinned_counters();
    if (!host) return fail(FGS_ERR_CUDA, "pinned host buffer");
    FGS_CUDA(cudaMemcpyAsync(host, B.counters, 2 * sizeof(unsigned long long), cudaMemcpyDeviceToHost, s), "counter readback");
    // the tensor-core MLP kernels' timeout flag rides along with the counters (Neural appearance only)
    const bool neural = !precomputed && r->cfg.model == fgs::kNeural;
    int* tc_flag = nullptr;
    host[2] = 0;
    if (neural) {
        FGS_CUDA(fgs::tc_timeout_flag(&tc_flag), "tensor-core timeout flag");
        FGS_CUDA(cudaMemcpyAsync(&host[2], tc_flag, sizeof(int), cudaMemcpyDeviceToHost, s), "tensor-core timeout flag");
    }
    FGS_CUDA(cudaStreamSynchronize(s), "counter readback");
    if (neural && (host[2] & 0xffffffffull)) {
        FGS_CUDA(cudaMemsetAsync(tc_flag, 0, sizeof(int), s), "tensor-core timeout flag");
        return fail(FGS_ERR_CUDA, "a tensor-core MLP kernel launched earlier on this device gave up a bounded wait for its MMAs; "
                                  "the gradients or colours it produced are invalid (the flag is now cleared)");
    }
    const uint64_t n_visible = host[0], n_inst = host[1];
    if (n_inst > 0x7fffff00ULL) return fail(FGS_ERR_UNSUPPORTED, "more than 2^31 instances");
    frame->n_visible = static_cast<int64_t>(n_visible);
    frame->n_instances = static_cast<int64_t>(n_inst);
    if (n_visible > 0 && !precomputed && r->cfg.model == fgs::kNeural) {
        ProfScope p_("appearance_mlp", s);
        FGS_CUDA(fgs::launch_neural_color(P, r->cfg, v, B.vis_idx, static_cast<uint32_t>(n_visible), B.rec, s), "appearance mlp");
    }
    if (n_visible > 0) {
        {
            ProfScope p_("depth_sort", s);
            FGS_CUDA(fgs::depth_sort(B, static_cast<uint32_t>(n_visible), s), "depth sort");
        }
        frame->depth_selector = B.sorted_idx == B.idx_b ? 1 : 0;
        ProfScope p_("reorder_scan", s);
        FGS_CUDA(fgs::launch_reorder(B, static_cast<uint32_t>(n_visible), s), "reorder");
        FGS_CUDA(fgs::exclusive_scan_u32(B.inst_off, static_cast<uint32_t>(n_visible), B.sort_temp, B.sort_temp_bytes, s), "offset scan");
    }
    return FGS_OK;
}

static int render_common(const fgs_settings* settings, fgs_frame* frame, void* prim_ws, void* tile_ws, size_t tile_ws_bytes, void* inst_ws,
                         size_t inst_ws_bytes, cudaStream_t s, fgs::BlendArgs* args, fgs::TileBuffers* T_out) {
    int rc = check_settings(settings);
    if (rc) return rc;
    if (settings->width != frame->width || settings->height != frame->height) return fail(FGS_ERR_INVALID_ARGUMENT, "settings do not match the frame");
    const Grid g = grid_of(frame->width, frame->height);
    const uint64_t n = static_cast<uint64_t>(frame->n_primitives);
    fgs::PrimBuffers B = carve_prim(prim_ws, n, nullptr);
    size_t need = 0;
    const fgs::TileBuffers T = carve_tile(tile_ws, g, &need);
    if (!tile_ws || tile_ws_bytes < need) return fail(FGS_ERR_WORKSPACE, "tile workspace too small");
    const uint64_t ni = static_cast<uint64_t>(frame->n_instances);
    InstBuffers I = carve_inst(inst_ws, ni, g, &need);
    if (ni > 0 && (!inst_ws || inst_ws_bytes < need)) return fail(FGS_ERR_WORKSPACE, "instance workspace too small");
    {
        ProfScope p_("emit", s);
        FGS_CUDA(fgs::launch_emit(B.sorted_rec, B.inst_off, I.keys_a, I.vals_a, static_cast<uint32_t>(frame->n_visible), g.gw, g.wide, ni, s), "emit");
    }
    const void* keys = nullptr;
    const uint32_t* vals = nullptr;
    {
        ProfScope p_("tile_sort", s);
        FGS_CUDA(fgs::tile_sort(I.keys_a, I.keys_b, I.vals_a, I.vals_b, ni, g.end_bit > 0 ? g.end_bit : 1, g.wide, I.temp, I.temp_bytes, &keys, &vals, s),
                 "tile sort");
    }
    frame->tile_selector = vals == I.vals_b ? 1 : 0;
    {
        ProfScope p_("ranges", s);
        FGS_CUDA(fgs::launch_ranges(keys, ni, g.wide, T, g.tiles, s), "ranges");
    }
    args->ranges = T.ranges;
    args->bucket_off = T.bucket_off;
    args->vals = vals;
    args->rec = B.sorted_rec;
    args->bg = settings->bg_color;
    args->width = frame->width;
    args->height = frame->height;
    args->grid_w = g.gw;
    args->grid_h = g.gh;
    *T_out = T;
    return FGS_OK;
}

int fgs_forward_render(fgs_rasterizer* r, const fgs_settings* settings, fgs_frame* frame, void* prim_ws, void* tile_ws, size_t tile_ws_bytes,
                       void* inst_ws, size_t inst_ws_bytes, void* bucket_ws, size_t bucket_ws_bytes, float* image, void* stream) {
    if (!r || !frame || !image) return fail(FGS_ERR_INVALID_ARGUMENT, "NULL argument");
    cudaStream_t s = static_cast<cudaStream_t>(stream);
    const Grid g = grid_of(frame->width, frame->height);
    (void)bucket_ws;
    (void)bucket_ws_bytes;
    (void)g;
    frame->n_buckets = 0;
    fgs::BlendArgs a;
    fgs::TileBuffers T;
    int rc = render_common(settings, frame, prim_ws, tile_ws, tile_ws_bytes, inst_ws, inst_ws_bytes, s, &a, &T);
    if (rc) return rc;
    ProfScope p_("blend_forward", s);
    FGS_CUDA(fgs::launch_blend_train(a, image, T, s), "blend");
    return FGS_OK;
}

int fgs_inference_render(fgs_rasterizer* r, const fgs_settings* settings, fgs_frame* frame, void* prim_ws, void* tile_ws, size_t tile_ws_bytes,
                         void* inst_ws, size_t inst_ws_bytes, float* image, int to_chw, int clamp_output, void* stream) {
    if (!r || !frame || !image) return fail(FGS_ERR_INVALID_ARGUMENT, "NULL argument");
    cudaStream_t s = static_cast<cudaStream_t>(stream);
    fgs::BlendArgs a;
    fgs::TileBuffers T;
    int rc = render_common(settings, frame, prim_ws, tile_ws, tile_ws_bytes, inst_ws, inst_ws_bytes, s, &a, &T);
    if (rc) return rc;
    ProfScope p_("blend_inference", s);
    FGS_CUDA(fgs::launch_blend_inference(a, image, to_chw, clamp_output, s), "blend");
    return FGS_OK;
}

int fgs_backward(fgs_rasterizer* r, const fgs_primitives* prims, const fgs_settings* settings, const fgs_frame* frame, void* prim_ws,
                 void* tile_ws, void* inst_ws, void* bucket_ws, void* grad_ws, size_t grad_ws_bytes, const float* image,
                 const float* grad_image, const fgs_gradients* grads, float* densification_info, int densification_rows, int accumulate,
                 void* stream) {
    if (!r || !frame || !grads || !image || !grad_image) return fail(FGS_ERR_INVALID_ARGUMENT, "NULL argument");
    int rc = check_settings(settings);
    if (rc) return rc;
    bool precomputed = false;
    rc = check_prims(r, prims, &precomputed);
    if (rc) return rc;
    if (precomputed != (frame->precomputed != 0)) return fail(FGS_ERR_INVALID_ARGUMENT, "inputs do not match the forward pass");
    if (prims->n_primitives != frame->n_primitives) return fail(FGS_ERR_INVALID_ARGUMENT, "n_primitives does not match the forward pass");
    if (densification_info && densification_rows != 2 && densification_rows != 3)
        return fail(FGS_ERR_INVALID_ARGUMENT, "densification_info must have 2 or 3 rows");
    if (!grads->means || !grads->scales || !grads->rotations || !grads->opacities)
        return fail(FGS_ERR_INVALID_ARGUMENT, "geometry gradient outputs are required");
    if (precomputed && !grads->precomputed_colors) return fail(FGS_ERR_INVALID_ARGUMENT, "precomputed color gradient output is required");
    const bool neural = !precomputed && r->cfg.model == fgs::kNeural;
    if (!precomputed && !grads->base_colors) return fail(FGS_ERR_INVALID_ARGUMENT, "base color gradient output is required");
    if (neural && !grads->mlp_weights) return fail(FGS_ERR_INVALID_ARGUMENT, "mlp weight gradient output is required");
    cudaStream_t s = static_cast<cudaStream_t>(stream);
    const uint64_t n = static_cast<uint64_t>(frame->n_primitives);
    if (n == 0) return FGS_OK;
    const Grid g = grid_of(frame->width, frame->height);
    const uint64_t nv = static_cast<uint64_t>(frame->n_visible);
    const uint64_t n_mlp = neural ? fgs::neural_grad_scratch_floats(r->cfg) : 0;
    size_t need = 0;
    GradBuffers gb = carve_grad(grad_ws, nv, n_mlp, &need);
    if (!grad_ws || grad_ws_bytes < need) return fail(FGS_ERR_WORKSPACE, "gradient workspace too small");
    const size_t act_bytes = neural && frame->mlp_activations ? mlp_act_bytes(r, n) : 0;
    fgs::PrimBuffers B = carve_prim(prim_ws, n, nullptr, act_bytes);
    const fgs::TileBuffers T = carve_tile(tile_ws, g, nullptr);
    InstBuffers I = carve_inst(inst_ws, static_cast<uint64_t>(frame->n_instances), g, nullptr);
    (void)bucket_ws;
    const fgs::View v = make_view(settings);
    fgs::Params P = make_params(prims);
    P.mlp_act = B.mlp_act;  // the forward's activation store, or null (recomputed)
    if (nv > 0) {
        FGS_CUDA(cudaMemsetAsync(gb.rec, 0, nv * sizeof(fgs::GradRecord), s), "gradient clear");
        fgs::BlendArgs a;
        a.ranges = T.ranges;
        a.bucket_off = T.bucket_off;
        a.vals = frame->tile_selector ? I.vals_b : I.vals_a;
        a.rec = B.sorted_rec;
        a.bg = settings->bg_color;
        a.width = frame->width;
        a.height = frame->height;
        a.grid_w = g.gw;
        a.grid_h = g.gh;
        ProfScope p_("blend_backward", s);
        FGS_CUDA(fgs::launch_blend_backward(a, image, grad_image, T, gb.rec, densification_rows == 3 && densification_info ? 1 : 0, s),
                 "blend backward");
    }
    if (n_mlp > 0) FGS_CUDA(cudaMemsetAsync(gb.mlp_scratch, 0, n_mlp * sizeof(float), s), "mlp gradient clear");
    fgs::GradOut O;
    O.means = grads->means; O.scales = grads->scales; O.rotations = grads->rotations; O.opacities = grads->opacities;
    O.precomputed = grads->precomputed_colors; O.base = grads->base_colors; O.residual = grads->residual_params;
    O.mlp = grads->mlp_weights; O.mlp_scratch = gb.mlp_scratch;
    O.densification = densification_info;
    O.densification_rows = densification_rows;
    O.accumulate = accumulate ? 1 : 0;
    ProfScope p_("preprocess_backward", s);
    FGS_CUDA(fgs::launch_preprocess_bwd(P, r->cfg, v, B.rank_of, B.sorted_rec, gb.rec, O, precomputed, B.vis_idx, static_cast<uint32_t>(nv), s),
             "preprocess backward");
    return FGS_OK;
}

int fgs_pruning_scores(const fgs_settings* settings, const fgs_frame* frame, void* prim_ws, void* tile_ws, void* inst_ws, const float* image,
                       float* scores, void* stream) {
    if (!frame || !image || !scores) return fail(FGS_ERR_INVALID_ARGUMENT, "NULL argument");
    int rc = check_settings(settings);
    if (rc) return rc;
    if (settings->width != frame->width || settings->height != frame->height) return fail(FGS_ERR_INVALID_ARGUMENT, "settings do not match the frame");
    const uint64_t nv = static_cast<uint64_t>(frame->n_visible);
    if (nv == 0) return FGS_OK;
    if (!prim_ws || !tile_ws || !inst_ws) return fail(FGS_ERR_INVALID_ARGUMENT, "the forward pass workspaces are required");
    cudaStream_t s = static_cast<cudaStream_t>(stream);
    const Grid g = grid_of(frame->width, frame->height);
    fgs::PrimBuffers B = carve_prim(prim_ws, static_cast<uint64_t>(frame->n_primitives), nullptr);
    const fgs::TileBuffers T = carve_tile(tile_ws, g, nullptr);
    InstBuffers I = carve_inst(inst_ws, static_cast<uint64_t>(frame->n_instances), g, nullptr);
    fgs::BlendArgs a;
    a.ranges = T.ranges;
    a.bucket_off = T.bucket_off;
    a.vals = frame->tile_selector ? I.vals_b : I.vals_a;
    a.rec = B.sorted_rec;
    a.bg = settings->bg_color;
    a.width = frame->width;
    a.height = frame->height;
    a.grid_w = g.gw;
    a.grid_h = g.gh;
    ProfScope p_("pruning_scores", s);
    FGS_CUDA(fgs::launch_pruning_scores(a, image, T, frame->depth_selector ? B.idx_b : B.idx_a, scores, s), "pruning scores");
    return FGS_OK;
}

int fgs_relocation_adjustment(const float* old_opacities, const float* old_scales, const int64_t* n_samples, float* new_opacities,
                              float* new_scales, int64_t n, void* stream) {
    if (n < 0 || n > 0xFFFFFFFFll) return fail(FGS_ERR_INVALID_ARGUMENT, "n out of range");
    if (n > 0 && (!old_opacities || !old_scales || !n_samples || !new_opacities || !new_scales)) return fail(FGS_ERR_INVALID_ARGUMENT, "NULL argument");
    FGS_CUDA(fgs::launch_relocation(old_opacities, old_scales, n_samples, new_opacities, new_scales, static_cast<uint32_t>(n),
                                    static_cast<cudaStream_t>(stream)),
             "relocation adjustment");
    return FGS_OK;
}

int fgs_add_noise(const float* raw_scales, const float* raw_rotations, const float* raw_opacities, float* means, int64_t n, float current_lr,
                  uint64_t seed, uint64_t offset, void* stream) {
    if (n < 0 || n > 0xFFFFFFFFll) return fail(FGS_ERR_INVALID_ARGUMENT, "n out of range");
    if (n > 0 && (!raw_scales || !raw_rotations || !raw_opacities || !means)) return fail(FGS_ERR_INVALID_ARGUMENT, "NULL argument");
    if (reinterpret_cast<uintptr_t>(raw_rotations) % 16 != 0) return fail(FGS_ERR_INVALID_ARGUMENT, "rotations must be 16-byte aligned");
    FGS_CUDA(fgs::launch_add_noise(raw_scales, raw_rotations, raw_opacities, means, static_cast<uint32_t>(n), current_lr, seed, offset,
                                   static_cast<cudaStream_t>(stream)),
             "add noise");
    return FGS_OK;
}

int fgs_morton_codes(const float* means, int64_t n, const float* box_min, const float* box_max, uint64_t* codes, void* stream) {
    if (n < 0 || n > 0xFFFFFFFFll) return fail(FGS_ERR_INVALID_ARGUMENT, "n out of range");
    if (!box_min || !box_max || (n > 0 && (!means || !codes))) return fail(FGS_ERR_INVALID_ARGUMENT, "NULL argument");
    FGS_CUDA(fgs::launch_morton(means, codes, static_cast<uint32_t>(n), box_min, box_max, static_cast<cudaStream_t>(stream)), "morton codes");
    return FGS_OK;
}

int fgs_update_3d_filter(const float* positions, const float* w2c, float* filter_3d, uint8_t* visibility_mask, int64_t n, int width, int height,
                         float focal_x, float focal_y, float center_x, float center_y, float near_plane, float far_plane,
                         float clipping_tolerance, float distance2filter, void* stream) {
    if (n < 0 || n > 0xFFFFFFFFll) return fail(FGS_ERR_INVALID_ARGUMENT, "n out of range");
    if (n > 0 && (!positions || !w2c || !filter_3d || !visibility_mask)) return fail(FGS_ERR_INVALID_ARGUMENT, "NULL argument");
    if (reinterpret_cast<uintptr_t>(w2c) % 16 != 0) return fail(FGS_ERR_INVALID_ARGUMENT, "w2c must be 16-byte aligned");
    // frustum slopes of the image widened by the clipping tolerance (filter3d/src/filter3d.cu:63-73)
    const float bounds = clipping_tolerance + 0.5f;
    const float w = static_cast<float>(width), h = static_cast<float>(height);
    const float ox = center_x - 0.5f * w, oy = center_y - 0.5f * h;
    const float left = (-(bounds * w) - ox) / focal_x, right = (bounds * w - ox) / focal_x;
    const float top = (-(bounds * h) - oy) / focal_y, bottom = (bounds * h - oy) / focal_y;
    FGS_CUDA(fgs::launch_filter3d(positions, w2c, filter_3d, visibility_mask, static_cast<uint32_t>(n), left, right, top, bottom, near_plane,
                                  far_plane, distance2filter, static_cast<cudaStream_t>(stream)),
             "3d filter");
    return FGS_OK;
}

int fgs_frame_buffers(const fgs_frame* frame, void* prim_ws, void* tile_ws, void* inst_ws, fgs_frame_views* out) {
    if (!frame || !out) return fail(FGS_ERR_INVALID_ARGUMENT, "NULL argument");
    std::memset(out, 0, sizeof(fgs_frame_views));
    const Grid g = grid_of(frame->width, frame->height);
    if (prim_ws) {
        fgs::PrimBuffers B = carve_prim(prim_ws, static_cast<uint64_t>(frame->n_primitives), nullptr);
        out->n_touched = B.n_touched;
        out->depth_keys = B.depth_key;
        out->sorted_indices = frame->depth_selector ? B.idx_b : B.idx_a;
        out->rank_of = B.rank_of;
        out->sorted_records = B.sorted_rec;
        out->instance_offsets = B.inst_off;
    }
    if (inst_ws) {
        InstBuffers I = carve_inst(inst_ws, static_cast<uint64_t>(frame->n_instances), g, nullptr);
        out->instance_keys = frame->tile_selector ? I.keys_b : I.keys_a;
        out->instance_ranks = frame->tile_selector ? I.vals_b : I.vals_a;
    }
    if (tile_ws) {
        const fgs::TileBuffers T = carve_tile(tile_ws, g, nullptr);
        out->tile_ranges = reinterpret_cast<const uint32_t*>(T.ranges);
        out->bucket_offsets = T.bucket_off;
        out->tile_max_contributors = T.tile_max;
        out->final_transmittance = T.final_T;
        out->n_contributors = T.n_contrib;
    }
    return FGS_OK;
}

// converts and checks the C-ABI segments; returns the number kept (empty segments are dropped) or -1
static int convert_segments(const fgs_adam_segment* segs, int n, fgs::AdamSegment* S) {
    if (n < 0 || n > fgs::kMaxAdamSegments || (n > 0 && !segs)) return fail(FGS_ERR_INVALID_ARGUMENT, "between 0 and 12 segments"), -1;
    int k = 0;
    for (int i = 0; i < n; i++) {
        const fgs_adam_segment& a = segs[i];
        if (a.n_elements <= 0) continue;
        if (!a.param || !a.grad || !a.exp_avg || !a.exp_avg_sq) return fail(FGS_ERR_INVALID_ARGUMENT, "segment pointer is NULL"), -1;
        if (a.n_learning_rates < 1 || a.n_learning_rates > 7) return fail(FGS_ERR_INVALID_ARGUMENT, "between 1 and 7 learning rates are supported"), -1;
        if (a.step < 1) return fail(FGS_ERR_INVALID_ARGUMENT, "step must be >= 1"), -1;
        const double bc1 = 1.0 / (1.0 - std::pow(a.beta1, static_cast<double>(a.step)));
        const double bc2 = 1.0 / std::sqrt(1.0 - std::pow(a.beta2, static_cast<double>(a.step)));
        fgs::AdamSegment& s = S[k++];
        s.param = a.param; s.grad = a.grad; s.m = a.exp_avg; s.v = a.exp_avg_sq;
        s.n = static_cast<uint64_t>(a.n_elements);
        s.col_offset = static_cast<uint64_t>(a.column_offset);
        for (int j = 0; j < 7; j++) s.lr[j] = j < a.n_learning_rates ? static_cast<float>(a.learning_rates[j] * bc1) : 0.0f;
        s.n_lr = a.n_learning_rates;
        s.beta1 = static_cast<float>(a.beta1);
        s.beta2 = static_cast<float>(a.beta2);
        s.eps = static_cast<float>(a.eps);
        s.bc2_sqrt_rcp = static_cast<float>(bc2);
    }
    return k;
}

int fgs_adam_step(const fgs_adam_segment* segs, int n, void* stream) {
    fgs::AdamSegment S[fgs::kMaxAdamSegments];
    const int k = convert_segments(segs, n, S);
    if (k < 0) return FGS_ERR_INVALID_ARGUMENT;
    ProfScope p_("adam", static_cast<cudaStream_t>(stream));
    FGS_CUDA(fgs::launch_adam(S, k, static_cast<cudaStream_t>(stream)), "adam");
    return FGS_OK;
}

int fgs_dp_shard_adam(const fgs_adam_segment* segs, int n, const fgs_peer_buffers* peers, void* stream) {
    if (!peers) return fail(FGS_ERR_INVALID_ARGUMENT, "peers is NULL");
    if (peers->n_ranks < 1 || peers->n_ranks > FGS_MAX_PEERS) return fail(FGS_ERR_INVALID_ARGUMENT, "n_ranks must be in [1, 8]");
    if (!peers->local_params) return fail(FGS_ERR_INVALID_ARGUMENT, "local_params is NULL");
    if ((peers->multicast_grads == nullptr) != (peers->multicast_params == nullptr))
        return fail(FGS_ERR_INVALID_ARGUMENT, "give both multicast addresses or neither");
    if (!peers->multicast_grads)
        for (int r = 0; r < peers->n_ranks; r++)
            if (!peers->grads[r] || !peers->params[r]) return fail(FGS_ERR_INVALID_ARGUMENT, "peer buffer pointer is NULL");
    fgs::AdamSegment S[fgs::kMaxAdamSegments];
    const int k = convert_segments(segs, n, S);
    if (k < 0) return FGS_ERR_INVALID_ARGUMENT;
    for (int i = 0; i < k; i++)
        if (S[i].param < peers->local_params) return fail(FGS_ERR_INVALID_ARGUMENT, "segment parameters must lie in the local flat buffer");
    static_assert(FGS_MAX_PEERS == fgs::kMaxPeers, "peer table size");
    ProfScope p_("exchange_adam", static_cast<cudaStream_t>(stream));
    FGS_CUDA(fgs::launch_dp_shard_adam(S, k, peers->grads, peers->params, peers->n_ranks, peers->local_params, peers->multicast_grads,
                                       peers->multicast_params, static_cast<cudaStream_t>(stream)),
             "exchange adam");
    return FGS_OK;
}

int fgs_loss_workspace_bytes(int channels, int height, int width, size_t* out) {
    if (!out || channels <= 0 || height <= 0 || width <= 0) return fail(FGS_ERR_INVALID_ARGUMENT, "bad argument");
    *out = fgs::loss_workspace_bytes(channels, height, width);
    return FGS_OK;
}

int fgs_l1_dssim(const float* image, const float* target, int channels, int height, int width, float l1_weight, float dssim_weight,
                 float* grad_image, float* loss, void* workspace, size_t workspace_bytes, void* stream) {
    if (!image || !target || !grad_image || !loss || !workspace) return fail(FGS_ERR_INVALID_ARGUMENT, "NULL argument");
    if (channels <= 0 || height <= 0 || width <= 0) return fail(FGS_ERR_INVALID_ARGUMENT, "bad image size");
    if (workspace_bytes < fgs::loss_workspace_bytes(channels, height, width)) return fail(FGS_ERR_WORKSPACE, "loss workspace too small");
    cudaStream_t s = static_cast<cudaStream_t>(stream);
    ProfScope p_("loss", s);
    FGS_CUDA(fgs::launch_l1_dssim(image, target, channels, height, width, l1_weight, dssim_weight, grad_image, loss, workspace, s), "loss");
    return FGS_OK;
}

int fgs_tc_timeout(int* timed_out, int clear) {
    if (!timed_out) return fail(FGS_ERR_INVALID_ARGUMENT, "NULL argument");
    int* flag = nullptr;
    FGS_CUDA(fgs::tc_timeout_flag(&flag), "tensor-core timeout flag");
    FGS_CUDA(cudaMemcpy(timed_out, flag, sizeof(int), cudaMemcpyDeviceToHost), "tensor-core timeout flag");
    if (clear && *timed_out) FGS_CUDA(cudaMemset(flag, 0, sizeof(int)), "tensor-core timeout flag");
    return FGS_OK;
}

int fgs_tc_selftest(float* scratch, int* mismatches, void* stream) {
    if (!scratch || !mismatches) return fail(FGS_ERR_INVALID_ARGUMENT, "NULL argument");
    static_assert(FGS_TC_SELFTEST_FLOATS == fgs::kTcSelftestFloats, "self-test buffer size");
    FGS_CUDA(fgs::tc_selftest(scratch, mismatches, static_cast<cudaStream_t>(stream)), "tensor-core self-test");
    return FGS_OK;
}

int fgs_profile_enable(int enabled) {
    g_prof.enabled = enabled != 0;
    return FGS_OK;
}

int fgs_profile_collect(char* names, size_t names_bytes, double* ms, int max_entries, int* n_entries) {
    if (!n_entries) return fail(FGS_ERR_INVALID_ARGUMENT, "n_entries is NULL");
    for (ProfEntry& e : g_prof.pending) {
        cudaError_t err = cudaEventSynchronize(e.stop);
        if (err != cudaSuccess) return cuda_fail(err, "profile");
        float t = 0.0f;
        cudaEventElapsedTime(&t, e.start, e.stop);
        bool found = false;
        for (auto& kv : g_prof.totals)
            if (kv.first == e.name) { kv.second += t; found = true; }
        if (!found) g_prof.totals.emplace_back(e.name, static_cast<double>(t));
        g_prof.pool.push_back(e.start);
        g_prof.pool.push_back(e.stop);
    }
    g_prof.pending.clear();
    std::string joined;
    int k = 0;
    for (auto& kv : g_prof.totals) {
        if (k < max_entries && ms) ms[k] = kv.second;
        if (k > 0) joined += ",";
        joined += kv.first;
        k++;
    }
    *n_entries = k;
    if (names && names_bytes > 0) {
        std::strncpy(names, joined.c_str(), names_bytes - 1);
        names[names_bytes - 1] = 0;
    }
    g_prof.totals.clear();
    return FGS_OK;
}

// ------------------------------------------------------------------------------------------------------
// Render entry point that allocates nothing.
//
// Some callers cannot allocate device memory while they render: a viewer or engine plugin that runs inside a
// host application owning a fixed device-memory budget, where a cudaMalloc in the middle of a frame may stall
// the frame or fail outright. For them, fgs_inference_noalloc keeps every workspace of the inference path in
// one file-scope device array of FGS_NOALLOC_SCRATCH_BYTES. The array is part of the library image, so every
// GPU that loads the library holds it until the process exits. The caller still provides the inputs and the
// output image.
//
// The device address of the array is looked up once per device, on that device's first call (with the device
// current), so the first call on each device should happen before any stream capture. The cached address
// belongs to the device's primary context: after cudaDeviceReset on that device it is stale and the process
// must not call this entry point again on that device. All calls share the array and it keeps the previous
// call's contents; every buffer the kernels read is either fully rewritten by the call or cleared by it (the
// tile ranges are set to zero before they are filled). Two calls whose work overlaps on the GPU (different
// streams or threads without synchronisation) race on the array.
static __device__ __align__(256) unsigned char g_noalloc_scratch[FGS_NOALLOC_SCRATCH_BYTES];
static std::mutex g_noalloc_mu;
static void* g_noalloc_ptr[64] = {nullptr};

int fgs_inference_noalloc(fgs_rasterizer* r, const fgs_primitives* prims, const fgs_settings* settings, float* image, int to_chw,
                          int clamp_output, void* stream, int64_t* n_visible, int64_t* n_instances) {
    if (!r || !image) return fail(FGS_ERR_INVALID_ARGUMENT, "NULL argument");
    int rc = check_settings(settings);
    if (rc) return rc;
    bool precomputed = false;
    rc = check_prims(r, prims, &precomputed);
    if (rc) return rc;
    int dev = 0;
    FGS_CUDA(cudaGetDevice(&dev), "noalloc device");
    if (dev < 0 || dev >= 64) return fail(FGS_ERR_UNSUPPORTED, "device index beyond 63");
    char* base = nullptr;
    {
        std::lock_guard<std::mutex> lock(g_noalloc_mu);
        if (!g_noalloc_ptr[dev]) {
            void* p = nullptr;
            FGS_CUDA(cudaGetSymbolAddress(&p, g_noalloc_scratch), "noalloc scratch address");
            g_noalloc_ptr[dev] = p;
        }
        base = static_cast<char*>(g_noalloc_ptr[dev]);
    }
    const uint64_t n = static_cast<uint64_t>(prims->n_primitives);
    const Grid g = grid_of(settings->width, settings->height);
    size_t prim_bytes = 0, tile_bytes = 0;
    carve_prim(nullptr, n, &prim_bytes);
    carve_tile(nullptr, g, &tile_bytes);
    prim_bytes = (prim_bytes + 255) & ~static_cast<size_t>(255);
    tile_bytes = (tile_bytes + 255) & ~static_cast<size_t>(255);
    if (prim_bytes + tile_bytes > FGS_NOALLOC_SCRATCH_BYTES)
        return fail(FGS_ERR_WORKSPACE, "fgs_inference_noalloc: " + std::to_string(n) + " primitives at " + std::to_string(settings->width) + "x" +
                                           std::to_string(settings->height) + " need " + std::to_string(prim_bytes + tile_bytes) +
                                           " bytes of scratch before binning, more than the static maximum of " +
                                           std::to_string(static_cast<size_t>(FGS_NOALLOC_SCRATCH_BYTES)));
    cudaStream_t s = static_cast<cudaStream_t>(stream);
    fgs::PrimBuffers B = carve_prim(base, n, nullptr);
    const fgs::TileBuffers T = carve_tile(base + prim_bytes, g, nullptr);
    const fgs::View v = make_view(settings);
    const fgs::Params P = make_params(prims);
    uint64_t nv = 0, ni = 0;
    if (n > 0) {
        FGS_CUDA(fgs::launch_preprocess_fwd(P, r->cfg, v, B, precomputed, s), "preprocess");
        FGS_CUDA(fgs::launch_compaction(B, static_cast<uint32_t>(n), s), "compaction");
        unsigned long long counts[2] = {0, 0};  // pageable host memory: no allocation
        FGS_CUDA(cudaMemcpyAsync(counts, B.counters, sizeof(counts), cudaMemcpyDeviceToHost, s), "counter readback");
        FGS_CUDA(cudaStreamSynchronize(s), "counter readback");
        nv = counts[0];
        ni = counts[1];
    }
    size_t inst_bytes = 0;
    InstBuffers I = carve_inst(nullptr, ni, g, &inst_bytes);
    if (prim_bytes + tile_bytes + inst_bytes > FGS_NOALLOC_SCRATCH_BYTES)
        return fail(FGS_ERR_WORKSPACE, "fgs_inference_noalloc: " + std::to_string(ni) + " tile instances need " +
                                           std::to_string(prim_bytes + tile_bytes + inst_bytes) + " bytes of scratch, more than the static maximum of " +
                                           std::to_string(static_cast<size_t>(FGS_NOALLOC_SCRATCH_BYTES)));
    I = carve_inst(base + prim_bytes + tile_bytes, ni, g, nullptr);
    if (nv > 0 && !precomputed && r->cfg.model == fgs::kNeural)
        FGS_CUDA(fgs::launch_neural_color(P, r->cfg, v, B.vis_idx, static_cast<uint32_t>(nv), B.rec, s), "appearance mlp");
    if (nv > 0) {
        FGS_CUDA(fgs::depth_sort(B, static_cast<uint32_t>(nv), s), "depth sort");
        FGS_CUDA(fgs::launch_reorder(B, static_cast<uint32_t>(nv), s), "reorder");
        FGS_CUDA(fgs::exclusive_scan_u32(B.inst_off, static_cast<uint32_t>(nv), B.sort_temp, B.sort_temp_bytes, s), "offset scan");
        FGS_CUDA(fgs::launch_emit(B.sorted_rec, B.inst_off, I.keys_a, I.vals_a, static_cast<uint32_t>(nv), g.gw, g.wide, ni, s), "emit");
    }
    const void* keys = nullptr;
    const uint32_t* vals = nullptr;
    FGS_CUDA(fgs::tile_sort(I.keys_a, I.keys_b, I.vals_a, I.vals_b, ni, g.end_bit > 0 ? g.end_bit : 1, g.wide, I.temp, I.temp_bytes, &keys, &vals, s),
             "tile sort");
    FGS_CUDA(fgs::launch_ranges(keys, ni, g.wide, T, g.tiles, s), "ranges");
    fgs::BlendArgs a;
    a.ranges = T.ranges;
    a.bucket_off = T.bucket_off;
    a.vals = vals;
    a.rec = B.sorted_rec;
    a.bg = settings->bg_color;
    a.width = settings->width;
    a.height = settings->height;
    a.grid_w = g.gw;
    a.grid_h = g.gh;
    FGS_CUDA(fgs::launch_blend_inference(a, image, to_chw, clamp_output, s), "blend");
    if (nv > 0 && !precomputed && r->cfg.model == fgs::kNeural) {
        // the tensor-core colour pass gives up a bounded wait by setting a device flag instead of faulting; read it
        // (pageable host memory, no allocation) so invalid colours never come back with FGS_OK
        int* tc_flag = nullptr;
        int flag_host = 0;
        FGS_CUDA(fgs::tc_timeout_flag(&tc_flag), "tensor-core timeout flag");
        FGS_CUDA(cudaMemcpyAsync(&flag_host, tc_flag, sizeof(int), cudaMemcpyDeviceToHost, s), "tensor-core timeout flag");
        FGS_CUDA(cudaStreamSynchronize(s), "tensor-core timeout flag");
        if (flag_host) {
            FGS_CUDA(cudaMemsetAsync(tc_flag, 0, sizeof(int), s), "tensor-core timeout flag");
            return fail(FGS_ERR_CUDA, "fgs_inference_noalloc: a tensor-core MLP kernel gave up a bounded wait for its MMAs; the image "
                                      "is invalid (the flag is now cleared)");
        }
    }
    if (n_visible) *n_visible = static_cast<int64_t>(nv);
    if (n_instances) *n_instances = static_cast<int64_t>(ni);
    return FGS_OK;
}

}  // extern "C"
