/* fgs_oracle.c -- TEST INFRASTRUCTURE, NOT PART OF THE PRODUCT.
 *
 * CPU restatement of the reference rasterizer (nerficg-project/efficient-gaussian-appearance,
 * FasterGSVDACudaBackend) used only as the checker by tests/, __graft_entry__.smoke() and the cpu_baseline
 * leg of bench.py. Built twice by oracle/Makefile:
 *   - ORC_REAL=float : the working-precision pipeline in the kernels' operation order with IEEE single-precision
 *     arithmetic (compiled with -ffp-contract=off, explicit fmaf where the kernels use one, the single-rounding forms
 *     of the reference's projection and tile test, and its exp2 fragment acceptance on the host's exp2). The GPU path
 *     evaluates those steps with the reference build's fast-math approximations (division, square root, exp, log,
 *     exp2), which C cannot reproduce, so the two agree within rounding and a decision within a rounding of its
 *     threshold may go either way; the Neural MLP (encoding, SH inputs, tensor-core accumulation, orc_neural.h) is
 *     restated exactly.
 *   - ORC_REAL=double: a smooth double-precision forward used for finite-difference checks of the backward.
 * The backward always evaluates values in double; the accept / terminate decisions come from the forward.
 *
 * Parity pinning: the appearance models are pinned against golden vectors produced by the reference's own
 * PyTorch modules (Appearance/SH.py, SV.py, NASG.py, NASGabor.py) under tests/golden/. The rasterizer (geometry,
 * binning, blending, backward) is pinned on the GPU against the reference's own kernels, built from its unmodified
 * sources by oracle/ref_build.py (oracle/reference.py); this restatement is checked against those same runs within
 * the bounds above, and its gradients against finite differences.
 *
 * Reference files followed (paths within the reference project):
 *   preprocess forward   FasterGSVDACudaBackend/FasterGSVDACudaBackend/rasterization/rtc/preprocess_forward.cu:12-278
 *   helpers              .../rasterization/rtc/preprocess_common.cuh:51-252
 *   tile culling         .../rasterization/include/tile_culling.cuh:13-65
 *   binning              .../rasterization/src/forward.cu:11-246, include/kernels_common.cuh:20-157
 *   forward blend        .../rasterization/include/kernels_forward.cuh:26-166, kernels_inference.cuh:11-126
 *   backward blend       .../rasterization/include/kernels_backward.cuh:12-231
 *   backward preprocess  .../rasterization/rtc/preprocess_backward.cu:19-404
 *   adam                 .../adam/src/adam.cu:18-87
 */
#include <stdint.h>
#include <stdlib.h>
#include <string.h>
#include <tgmath.h>
#ifdef _OPENMP
#include <omp.h>
#endif

#ifndef ORC_DOUBLE
typedef float real;
typedef float inreal;  /* type of the per-Gaussian input arrays */
#define R(x) x##f
#define RFMA fmaf
#else
typedef double real;
typedef double inreal;
#define R(x) x
#define RFMA fma
#endif

/* ------------------------------------------------------------------------------------------------ */
/* deterministic exp / log (same algorithm and constants as the kernels' fgs_common.cuh)              */

static inline float f_from_bits(uint32_t b) { float f; memcpy(&f, &b, 4); return f; }
static inline uint32_t bits_from_f(float f) { uint32_t b; memcpy(&b, &f, 4); return b; }

static float det_exp_f(float x) {
    if (x != x) return x;
    if (x < -87.0f) return 0.0f;
    if (x > 88.0f) return f_from_bits(0x7f800000u);
    const float n = rintf(x * 1.44269504088896341f);
    float r = fmaf(-n, 0.693145751953125f, x);
    r = fmaf(-n, 1.428606765330187e-06f, r);
    float p = 1.0f / 5040.0f;
    p = fmaf(p, r, 1.0f / 720.0f);
    p = fmaf(p, r, 1.0f / 120.0f);
    p = fmaf(p, r, 1.0f / 24.0f);
    p = fmaf(p, r, 1.0f / 6.0f);
    p = fmaf(p, r, 0.5f);
    p = fmaf(p, r, 1.0f);
    p = fmaf(p, r, 1.0f);
    return p * f_from_bits((uint32_t)((int)n + 127) << 23);
}

/* sine and cosine of the Neural encoding in the float build: Cody-Waite reduction modulo pi/2 in three parts,
 * Taylor series of sin through r^9 and cos through r^10, quadrant rotation, arguments clamped to |x| <= 8192; the
 * kernels' enc_sincos (fgs_common.cuh) performs the same single-rounding operations, so both give the same bits (within
 * 2.5e-7 of exact). */
static void det_sincos_f(float x, float* sp, float* cp) {
    float k = 0.0f, r;
    if (fabsf(x) <= 0.78f) {
        r = x + 0.0f;
    } else {
        x = fminf(fmaxf(x, -8192.0f), 8192.0f);
        k = rintf(x * 0.636619746685028076171875f);
        r = fmaf(-k, 1.57079637050628662109375f, x);
        r = fmaf(-k, -4.371138828673792886547744274139404296875e-08f, r);
        r = fmaf(-k, -1.7151245100058819e-15f, r);
    }
    const float r2 = r * r;
    float ps = 1.0f / 362880.0f;
    ps = fmaf(ps, r2, -1.0f / 5040.0f);
    ps = fmaf(ps, r2, 1.0f / 120.0f);
    ps = fmaf(ps, r2, -1.0f / 6.0f);
    const float s = fmaf(ps, r2 * r, r);
    float pc = -1.0f / 3628800.0f;
    pc = fmaf(pc, r2, 1.0f / 40320.0f);
    pc = fmaf(pc, r2, -1.0f / 720.0f);
    pc = fmaf(pc, r2, 1.0f / 24.0f);
    pc = fmaf(pc, r2, -0.5f);
    const float c = fmaf(pc, r2, 1.0f);
    switch (((int)k) & 3) {
        case 0: *sp = s; *cp = c; break;
        case 1: *sp = c; *cp = -s; break;
        case 2: *sp = -s; *cp = -c; break;
        default: *sp = -c; *cp = s; break;
    }
}

static float det_exp_blend_f(float x) {
    const float n = rintf(x * 1.44269504088896341f);
    float r = fmaf(-n, 0.693145751953125f, x);
    r = fmaf(-n, 1.428606765330187e-06f, r);
    float p = 1.0f / 720.0f;
    p = fmaf(p, r, 1.0f / 120.0f);
    p = fmaf(p, r, 1.0f / 24.0f);
    p = fmaf(p, r, 1.0f / 6.0f);
    p = fmaf(p, r, 0.5f);
    p = fmaf(p, r, 1.0f);
    p = fmaf(p, r, 1.0f);
    return p * f_from_bits((uint32_t)((int)n + 127) << 23);
}

static float det_log_f(float x) {
    if (!(x > 0.0f)) return x == 0.0f ? f_from_bits(0xff800000u) : f_from_bits(0x7fc00000u);
    if (x == f_from_bits(0x7f800000u)) return x;
    int k = 0;
    if (x < 1.17549435e-38f) { x = x * 16777216.0f; k = -24; }
    const uint32_t bits = bits_from_f(x);
    k += (int)((bits >> 23) & 0xffu) - 127;
    float m = f_from_bits((bits & 0x007fffffu) | 0x3f800000u);
    if (m > 1.41421356f) { m = m * 0.5f; k += 1; }
    const float s = (m - 1.0f) / (m + 1.0f);
    const float s2 = s * s;
    float p = 1.0f / 11.0f;
    p = fmaf(p, s2, 1.0f / 9.0f);
    p = fmaf(p, s2, 1.0f / 7.0f);
    p = fmaf(p, s2, 1.0f / 5.0f);
    p = fmaf(p, s2, 1.0f / 3.0f);
    p = fmaf(p, s2, 1.0f);
    const float ln_m = 2.0f * s * p;
    const float kf = (float)k;
    return fmaf(kf, 0.693145751953125f, fmaf(kf, 1.428606765330187e-06f, ln_m));
}

#ifndef ORC_DOUBLE
#define DEXP(x) det_exp_f(x)
#define DEXP_BLEND(x) det_exp_blend_f(x)
#define DLOG(x) det_log_f(x)
#else
#define DEXP(x) exp(x)
#define DEXP_BLEND(x) exp(x)
#define DLOG(x) log(x)
#endif

/* Fragment acceptance of the blend (kernels_forward.cuh:119-127 with the conic folded by -0.5 log2(e) and -log2(e),
 * kernels_common.cuh:13-17): base-2 exponent in the operation order the reference's build evaluates it with, the
 * Gaussian 2^min(e, 0), alpha = opacity * Gaussian, and the fragment is skipped when alpha < 1/255. The kernels take
 * the power of two from the GPU's exp2; this restatement takes it from the host's exp2 in double, rounded to the
 * working precision, so a fragment whose alpha lies within a rounding of 1/255 can be decided differently. Returns
 * alpha, or -1 for a skipped fragment. */
static inline real fragment_alpha_r(real opacity, real ca, real cb, real cc, real dx, real dy) {
    const real kh = (real)(-0.5f * 1.44269504089f), kc = (real)(-1.44269504089f);
    const real hx = kh * ca, hy = kc * cb, hz = kh * cc;
    const real ex = RFMA(hz * dy, dy, dx * RFMA(hx, dx, hy * dy));
    const real alpha = opacity * (real)exp2((double)fmin(ex, R(0.0)));
    return alpha < (real)(1.0f / 255.0f) ? R(-1.0) : alpha;
}

/* ------------------------------------------------------------------------------------------------ */
/* appearance models                                                                                 */

#define T real
#define SFX _r
#define K(x) R(x)
#include "orc_appearance.h"
#undef T
#undef SFX
#undef K
#define T double
#define SFX _d
#define K(x) x
#include "orc_appearance.h"
#undef T
#undef SFX
#undef K

/* ------------------------------------------------------------------------------------------------ */
/* configuration structs (mirrored by oracle/oracle.py)                                              */

typedef struct {
    float w2c[16];
    float cam[3];
    float bg[3];
    int width, height;
    float fx, fy, cx, cy, near_plane, far_plane;
    int proper_aa, render_base, degree;
} orc_view;

typedef struct {
    int model;       /* 0 precomputed, 1 sh, 2 sv, 3 nasg, 4 nasgabor, 5 neural */
    int max_degree;
    int base_act, res_act, color_act, dir_grad;
    /* neural */
    int feature_dim, base_input, n_freq, sh_mask, n_input, n_input_pad, n_neurons, n_hidden, hidden_act;
} orc_appearance;

enum { TILE_W = 16, TILE_H = 12, TILE_PIX = 192, SUB_W = 8, SUB_H = 4 };

int orc_residual_stride(const orc_appearance* A) {
    switch (A->model) {
        case 1: return 3 * ((A->max_degree + 1) * (A->max_degree + 1) - 1);
        case 2: return 7 * A->max_degree;
        case 3: return 8 * A->max_degree;
        case 4: return 9 * A->max_degree;
        case 5: return A->feature_dim;
        default: return 0;
    }
}

static int residual_active(const orc_appearance* A, int degree) {
    switch (A->model) {
        case 1: return degree > 0 ? 3 * ((degree + 1) * (degree + 1) - 1) : 0;
        case 2: return 7 * degree;
        case 3: return 8 * degree;
        case 4: return 9 * degree;
        case 5: return degree > 0 ? A->feature_dim : 0;
        default: return 0;
    }
}

/* ------------------------------------------------------------------------------------------------ */
/* activations in working precision (preprocess_common.cuh:51-142)                                  */

static real base_act_r(int id, real x) { return id == 1 ? DEXP(R(3.0) * x) : x; }
static real color_act_r(int id, real x) {
    switch (id) {
        case 1: return fmax(x + R(0.5), R(0.0));
        case 2: return softplus10_r(x + R(0.5));
        case 3: return R(1.0) / (R(1.0) + DEXP(-R(4.0) * x));
        case 4: return clampv_r(x + R(0.5), R(0.0), R(1.0));
        case 5: return -expm1(-x);
        default: return x + R(0.5);
    }
}
static double color_act_grad_d(int id, double y) {
    switch (id) {
        case 1: return y > 0.0 ? 1.0 : 0.0;
        case 2: return softplus10_grad_d(y);
        case 3: return 4.0 * (y - y * y);
        case 4: return (y > 0.0 && y < 1.0) ? 1.0 : 0.0;
        case 5: return 1.0 - y;
        default: return 1.0;
    }
}
static double base_act_grad_d(int id, double x) { return id == 1 ? 3.0 * exp(3.0 * x) : 1.0; }
static real sigmoid_r(real x) { return R(1.0) / (R(1.0) + DEXP(-x)); }
static real sat_r(real x) { return x > R(0.0) ? (x < R(1.0) ? x : R(1.0)) : R(0.0); }

/* ------------------------------------------------------------------------------------------------ */
/* preprocess forward                                                                                */

typedef struct { real m11, m12, m13, m21, m22, m23, m31, m32, m33; } mat3r;

static mat3r quat_to_rot_r(real r, real x, real y, real z, real* nsq) {
    const real xx = x * x, yy = y * y, zz = z * z, xy = x * y, xz = x * z, yz = y * z, rx = r * x, ry = r * y, rz = r * z;
    *nsq = r * r + xx + yy + zz;
    const real s = R(1.0) / *nsq;
    mat3r M;
    M.m11 = R(1.0) - R(2.0) * (yy + zz) * s; M.m12 = R(2.0) * (xy - rz) * s;        M.m13 = R(2.0) * (xz + ry) * s;
    M.m21 = R(2.0) * (xy + rz) * s;        M.m22 = R(1.0) - R(2.0) * (xx + zz) * s; M.m23 = R(2.0) * (yz - rx) * s;
    M.m31 = R(2.0) * (xz - ry) * s;        M.m32 = R(2.0) * (yz + rx) * s;        M.m33 = R(1.0) - R(2.0) * (xx + yy) * s;
    return M;
}

static int tile_overlaps_r(real mx, real my, real cx, real cy, real cz, uint32_t tx, uint32_t ty, real thr) {
    const real rminx = (real)(tx * TILE_W), rminy = (real)(ty * TILE_H);
    const real rmaxx = (real)((tx + 1) * TILE_W - 1), rmaxy = (real)((ty + 1) * TILE_H - 1);
    const real xmd = rminx - mx;
    const real xl = xmd >= R(0.0) ? R(1.0) : R(0.0);
    const real nx = xl + (mx > rmaxx ? R(1.0) : R(0.0));
    const real ymd = rminy - my;
    const real ya = ymd >= R(0.0) ? R(1.0) : R(0.0);
    const real ny = ya + (my > rmaxy ? R(1.0) : R(0.0));
    if (ny + nx == R(0.0)) return 1;
    /* the kernels' single-rounding operations (geometry.cuh tile_overlaps); their divisions are the GPU build's */
    const real kx = RFMA(xl, rminx - rmaxx, rmaxx);
    const real ky = RFMA(ya, rminy - rmaxy, rmaxy);
    const real dfx = mx - kx, dfy = my - ky;
    const real dx = copysign((real)(TILE_W - 1), xmd);
    const real dy = copysign((real)(TILE_H - 1), ymd);
    const real dxcx = dx * cx, dycz = dy * cz;
    const real tx_ = ny * sat_r(RFMA(dxcx, dfx, (dx * cy) * dfy) / (dxcx * dx));
    const real ty_ = nx * sat_r(RFMA(dy * cy, dfx, dycz * dfy) / (dycz * dy));
    const real px = RFMA(tx_, dx, kx), py = RFMA(ty_, dy, ky);
    const real ex = mx - px, ey = my - py;
    const real inner = RFMA(cx * ex, ex, (cz * ey) * ey);
    const real maxp = RFMA(cy * ex, ey, R(0.5) * inner);
    return maxp <= thr;
}

static uint32_t floor_clamped(real v, int hi) {
    const real c = clampv_r(v, R(-1.0), (real)hi + R(1.0));
    const int i = (int)floor(c);
    return (uint32_t)(i < 0 ? 0 : (i > hi ? hi : i));
}
static uint32_t ceil_clamped(real v, int hi) {
    const real c = clampv_r(v, R(-1.0), (real)hi + R(1.0));
    const int i = (int)ceil(c);
    return (uint32_t)(i < 0 ? 0 : (i > hi ? hi : i));
}

/* per-primitive record in working precision: mean2d, opacity, power threshold, conic, color, bounds */
typedef struct {
    real mx, my, opacity, thr, ca, cb, cc, r, g, b;
    uint32_t xmin, xmax, ymin, ymax;
} orc_rec;

static v3_r fused_color(const orc_appearance* A, const orc_view* v, int64_t i, const inreal* means, const inreal* base,
                        const inreal* residual, const inreal* mlp);

/* returns n_touched (0 = culled); fills rec and depth */
/* optional trace of the intermediate values of one primitive (debugging aid): depth, opacity, det, a, b, c, x, y,
 * mx, my, thr, xmin, xmax, ymin, ymax, nmax, count, stage reached */
static double* g_trace = 0;
#define TRACE(k, val) do { if (g_trace) g_trace[k] = (double)(val); } while (0)

static uint32_t preprocess_one(const orc_appearance* A, const orc_view* v, int64_t i, const inreal* means, const inreal* scales,
                               const inreal* rots, const inreal* opac, orc_rec* out, real* depth_out) {
    const real* w;
    real wr[16];
    for (int k = 0; k < 16; k++) wr[k] = v->w2c[k];
    w = wr;
    const real mx3 = means[3 * i], my3 = means[3 * i + 1], mz3 = means[3 * i + 2];
    const real depth = w[8] * mx3 + w[9] * my3 + w[10] * mz3 + w[11];
    *depth_out = depth;
    TRACE(0, depth);
    TRACE(17, 0);
    if (depth < (real)v->near_plane || depth > (real)v->far_plane) return 0;
    real opacity = sigmoid_r(opac[i]);
    int active = 1;
    if (opacity < R(1.0) / R(255.0)) active = 0;
    const real vx = DEXP(R(2.0) * (real)scales[3 * i]), vy = DEXP(R(2.0) * (real)scales[3 * i + 1]), vz = DEXP(R(2.0) * (real)scales[3 * i + 2]);
    real nsq;
    const mat3r Rm = quat_to_rot_r(rots[4 * i], rots[4 * i + 1], rots[4 * i + 2], rots[4 * i + 3], &nsq);
    if (nsq < R(1e-8)) active = 0;
    const mat3r RS = {Rm.m11 * vx, Rm.m12 * vy, Rm.m13 * vz, Rm.m21 * vx, Rm.m22 * vy, Rm.m23 * vz, Rm.m31 * vx, Rm.m32 * vy, Rm.m33 * vz};
    const real s11 = RS.m11 * Rm.m11 + RS.m12 * Rm.m12 + RS.m13 * Rm.m13;
    const real s12 = RS.m11 * Rm.m21 + RS.m12 * Rm.m22 + RS.m13 * Rm.m23;
    const real s13 = RS.m11 * Rm.m31 + RS.m12 * Rm.m32 + RS.m13 * Rm.m33;
    const real s22 = RS.m21 * Rm.m21 + RS.m22 * Rm.m22 + RS.m23 * Rm.m23;
    const real s23 = RS.m21 * Rm.m31 + RS.m22 * Rm.m32 + RS.m23 * Rm.m33;
    const real s33 = RS.m31 * Rm.m31 + RS.m32 * Rm.m32 + RS.m33 * Rm.m33;
    const real x = (w[0] * mx3 + w[1] * my3 + w[2] * mz3 + w[3]) / depth;
    const real y = (w[4] * mx3 + w[5] * my3 + w[6] * mz3 + w[7]) / depth;
    const real W = (real)v->width, H = (real)v->height;
    const real fx = v->fx, fy = v->fy, cx = v->cx, cy = v->cy;
    const real cl = (R(-0.15) * W - cx) / fx, cr = (R(1.15) * W - cx) / fx;
    const real ct = (R(-0.15) * H - cy) / fy, cbm = (R(1.15) * H - cy) / fy;
    const real xc = clampv_r(x, cl, cr), yc = clampv_r(y, ct, cbm);
    const real j11 = fx / depth, j13 = -j11 * xc, j22 = fy / depth, j23 = -j22 * yc;
    const v3_r a1 = mk_r(j11 * w[0] + j13 * w[8], j11 * w[1] + j13 * w[9], j11 * w[2] + j13 * w[10]);
    const v3_r a2 = mk_r(j22 * w[4] + j23 * w[8], j22 * w[5] + j23 * w[9], j22 * w[6] + j23 * w[10]);
    const v3_r b1 = mk_r(a1.x * s11 + a1.y * s12 + a1.z * s13, a1.x * s12 + a1.y * s22 + a1.z * s23, a1.x * s13 + a1.y * s23 + a1.z * s33);
    const v3_r b2 = mk_r(a2.x * s11 + a2.y * s12 + a2.z * s13, a2.x * s12 + a2.y * s22 + a2.z * s23, a2.x * s13 + a2.y * s23 + a2.z * s33);
    real a = dot_r(b1, a1);
    const real b = dot_r(b1, a2);
    real c = dot_r(b2, a2);
    const real det_raw = a * c - b * b;
    const real kd = v->proper_aa ? R(0.1) : R(0.3);
    a = a + kd;
    c = c + kd;
    const real det = a * c - b * b;
    if (det < R(1e-6)) active = 0;
    const real ca = c / det, cb = -b / det, cc = a / det;
    if (v->proper_aa) {
        opacity = opacity * sqrt(fmax(det_raw / det, R(0.0)));
        if (opacity < R(1.0) / R(255.0)) active = 0;
    }
    TRACE(1, opacity); TRACE(2, det); TRACE(3, a); TRACE(4, b); TRACE(5, c); TRACE(6, x); TRACE(7, y); TRACE(17, 1);
    if (!active) return 0;
    const real mx = x * fx + cx, my = y * fy + cy;
    const real thr = DLOG(opacity * R(255.0));
    const real cutoff = R(2.0) * thr;
    const real ex = fmax(sqrt(a * cutoff) - R(0.5), R(0.0));
    const real ey = fmax(sqrt(c * cutoff) - R(0.5), R(0.0));
    const int gw = (v->width + TILE_W - 1) / TILE_W, gh = (v->height + TILE_H - 1) / TILE_H;
    const int pw = gw * TILE_W, ph = gh * TILE_H;
    const uint32_t xmin = floor_clamped(mx - ex, pw), xmax = ceil_clamped(mx + ex, pw);
    const uint32_t ymin = floor_clamped(my - ey, ph), ymax = ceil_clamped(my + ey, ph);
    const uint32_t tx0 = xmin / TILE_W, tx1 = (xmax + TILE_W - 1) / TILE_W, ty0 = ymin / TILE_H, ty1 = (ymax + TILE_H - 1) / TILE_H;
    const uint32_t bw = tx1 - tx0, nmax = bw * (ty1 - ty0);
    TRACE(8, mx); TRACE(9, my); TRACE(10, thr); TRACE(11, xmin); TRACE(12, xmax); TRACE(13, ymin); TRACE(14, ymax); TRACE(15, nmax); TRACE(17, 2);
    if (nmax == 0) return 0;
    uint32_t count = 0;
    const real sx = mx - R(0.5), sy = my - R(0.5);
    for (uint32_t t = 0; t < nmax; t++)
        if (tile_overlaps_r(sx, sy, ca, cb, cc, tx0 + t % bw, ty0 + t / bw, thr)) count++;
    TRACE(16, count); TRACE(17, 3);
    if (count == 0) return 0;
    out->mx = mx; out->my = my; out->opacity = opacity; out->thr = thr;
    out->ca = ca; out->cb = cb; out->cc = cc;
    out->xmin = xmin; out->xmax = xmax; out->ymin = ymin; out->ymax = ymax;
    return count;
}

/* ------------------------------------------------------------------------------------------------ */
/* neural residual (fp16 MLP semantics) -- implemented in orc_neural.h                                */
#include "orc_neural.h"

static v3_r fused_color(const orc_appearance* A, const orc_view* v, int64_t i, const inreal* means, const inreal* base,
                        const inreal* residual, const inreal* mlp) {
    const v3_r cam = mk_r(v->cam[0], v->cam[1], v->cam[2]);
    const v3_r dv = sub_r(mk_r(means[3 * i], means[3 * i + 1], means[3 * i + 2]), cam);
    const real rn = R(1.0) / sqrt(fmax(dot_r(dv, dv), R(1e-24)));
    const v3_r d = scl_r(rn, dv);
    const int stride = orc_residual_stride(A);
    const inreal* rp = residual ? residual + (size_t)i * stride : 0;
    const int deg = v->degree < A->max_degree ? v->degree : A->max_degree;
    v3_r res = mk_r(R(0.0), R(0.0), R(0.0));
    switch (A->model) {
        case 1: res = sh_forward_r(rp, d, deg, A->res_act); break;
        case 2: res = sv_forward_r(rp, d, deg, A->res_act); break;
        case 3: res = lobes_forward_r(rp, d, deg, A->res_act, 0); break;
        case 4: res = lobes_forward_r(rp, d, deg, A->res_act, 1); break;
        case 5: res = neural_forward_r(A, rp, base + 3 * i, d, deg, mlp); break;
        default: break;
    }
    const v3_r bs = mk_r(base_act_r(A->base_act, base[3 * i]), base_act_r(A->base_act, base[3 * i + 1]), base_act_r(A->base_act, base[3 * i + 2]));
    const v3_r s = add_r(bs, res);
    v3_r col = mk_r(color_act_r(A->color_act, s.x), color_act_r(A->color_act, s.y), color_act_r(A->color_act, s.z));
    if (!v->render_base) {
        const v3_r bc = mk_r(color_act_r(A->color_act, bs.x), color_act_r(A->color_act, bs.y), color_act_r(A->color_act, bs.z));
        col = mk_r(fabs(col.x - bc.x), fabs(col.y - bc.y), fabs(col.z - bc.z));
    }
    return col;
}

/* Threads of the per-primitive and per-pixel loops (OpenMP). 1 (the default, used by the parity tests) runs every loop
 * in order; more threads give the same per-element results, and sums over elements (the MLP weight gradient, the
 * blend backward's per-primitive sums) are then added per thread and combined in thread order. */
static int g_threads = 1;
void orc_set_threads(int n) { g_threads = n < 1 ? 1 : n; }
int orc_threads(void) { return g_threads; }

static inline int thread_id(void) {
#ifdef _OPENMP
    return omp_get_thread_num();
#else
    return 0;
#endif
}

/* Forward preprocess of all primitives. Outputs (primitive order): n_touched[N], depth_key[N] (float bits
 * of the depth in working precision; only meaningful where n_touched > 0), rec[N*14] as doubles
 * (mx, my, opacity, thr, ca, cb, cc, r, g, b, xmin, xmax, ymin, ymax). */
int orc_preprocess(const orc_appearance* A, const orc_view* v, int64_t n, const inreal* means, const inreal* scales, const inreal* rots,
                   const inreal* opac, const inreal* precomputed, const inreal* base, const inreal* residual, const inreal* mlp,
                   uint32_t* n_touched, uint32_t* depth_key, double* rec) {
#pragma omp parallel for schedule(dynamic, 64) num_threads(g_threads) if (g_threads > 1)
    for (int64_t i = 0; i < n; i++) {
        orc_rec q;
        memset(&q, 0, sizeof(q));
        real depth;
        const uint32_t cnt = preprocess_one(A, v, i, means, scales, rots, opac, &q, &depth);
        n_touched[i] = cnt;
        const float df = (float)depth;
        depth_key[i] = bits_from_f(df);
        if (cnt > 0) {
            v3_r col;
            if (precomputed) col = mk_r(precomputed[3 * i], precomputed[3 * i + 1], precomputed[3 * i + 2]);
            else col = fused_color(A, v, i, means, base, residual, mlp);
            q.r = col.x; q.g = col.y; q.b = col.z;
        }
        double* o = rec + 14 * i;
        o[0] = q.mx; o[1] = q.my; o[2] = q.opacity; o[3] = q.thr; o[4] = q.ca; o[5] = q.cb; o[6] = q.cc;
        o[7] = q.r; o[8] = q.g; o[9] = q.b; o[10] = q.xmin; o[11] = q.xmax; o[12] = q.ymin; o[13] = q.ymax;
    }
    return 0;
}

/* ------------------------------------------------------------------------------------------------ */
/* binning                                                                                           */

static int cmp_u64(const void* a, const void* b) {
    const uint64_t x = *(const uint64_t*)a, y = *(const uint64_t*)b;
    return x < y ? -1 : (x > y ? 1 : 0);
}

/* Visible primitives sorted by (depth key, primitive index): returns V, writes sorted_idx[V]. */
int64_t orc_depth_order(int64_t n, const uint32_t* n_touched, const uint32_t* depth_key, uint32_t* sorted_idx) {
    int64_t V = 0;
    for (int64_t i = 0; i < n; i++) V += n_touched[i] > 0;
    uint64_t* tmp = (uint64_t*)malloc(sizeof(uint64_t) * (size_t)(V > 0 ? V : 1));
    int64_t k = 0;
    for (int64_t i = 0; i < n; i++)
        if (n_touched[i] > 0) tmp[k++] = ((uint64_t)depth_key[i] << 32) | (uint64_t)i;
    qsort(tmp, (size_t)V, sizeof(uint64_t), cmp_u64);
    for (int64_t r = 0; r < V; r++) sorted_idx[r] = (uint32_t)(tmp[r] & 0xffffffffu);
    free(tmp);
    return V;
}

static void rec_of(const double* rec, uint32_t i, orc_rec* q) {
    const double* o = rec + 14 * (size_t)i;
    q->mx = (real)o[0]; q->my = (real)o[1]; q->opacity = (real)o[2]; q->thr = (real)o[3];
    q->ca = (real)o[4]; q->cb = (real)o[5]; q->cc = (real)o[6]; q->r = (real)o[7]; q->g = (real)o[8]; q->b = (real)o[9];
    q->xmin = (uint32_t)o[10]; q->xmax = (uint32_t)o[11]; q->ymin = (uint32_t)o[12]; q->ymax = (uint32_t)o[13];
}

/* Instances in emission order (depth rank, then row-major tiles) and the stable tile sort.
 * Outputs: tile_keys[I], ranks[I] (sorted by tile, depth order inside a tile), ranges[2*T]. Returns I. */
int64_t orc_bin(int64_t n_visible, const uint32_t* sorted_idx, const double* rec, int width, int height, uint32_t* tile_keys,
                uint32_t* ranks, uint32_t* ranges) {
    const int gw = (width + TILE_W - 1) / TILE_W, gh = (height + TILE_H - 1) / TILE_H, T = gw * gh;
    /* emission: per depth rank the touched tiles of its primitive in row-major order (the exact tile test), ranks in
     * order; then a stable counting sort by tile keeps the emission order inside every tile list */
    int64_t* off = (int64_t*)calloc((size_t)n_visible + 1, sizeof(int64_t));
    for (int pass = 0; pass < 2; pass++) {
        uint32_t* em = pass == 1 ? (uint32_t*)malloc(sizeof(uint32_t) * ((size_t)off[n_visible] + 1)) : 0;
#pragma omp parallel for schedule(dynamic, 256) num_threads(g_threads) if (g_threads > 1)
        for (int64_t r = 0; r < n_visible; r++) {
            orc_rec q;
            rec_of(rec, sorted_idx[r], &q);
            const uint32_t tx0 = q.xmin / TILE_W, tx1 = (q.xmax + TILE_W - 1) / TILE_W, ty0 = q.ymin / TILE_H, ty1 = (q.ymax + TILE_H - 1) / TILE_H;
            const uint32_t bw = tx1 - tx0, nmax = bw * (ty1 - ty0);
            const real sx = q.mx - R(0.5), sy = q.my - R(0.5);
            int64_t k = 0;
            for (uint32_t t = 0; t < nmax; t++) {
                const uint32_t tx = tx0 + t % bw, ty = ty0 + t / bw;
                if (!tile_overlaps_r(sx, sy, q.ca, q.cb, q.cc, tx, ty, q.thr)) continue;
                if (pass == 1) em[off[r] + k] = ty * (uint32_t)gw + tx;
                k++;
            }
            if (pass == 0) off[r + 1] = k;
        }
        if (pass == 0) {
            for (int64_t r = 0; r < n_visible; r++) off[r + 1] += off[r];
            continue;
        }
        const int64_t n_inst = off[n_visible];
        int64_t* pos = (int64_t*)calloc((size_t)T + 1, sizeof(int64_t));
        for (int64_t i = 0; i < n_inst; i++) pos[em[i] + 1]++;
        for (int t = 0; t < T; t++) {
            ranges[2 * t] = pos[t + 1] ? (uint32_t)pos[t] : 0;
            pos[t + 1] += pos[t];
            ranges[2 * t + 1] = pos[t + 1] - pos[t] ? (uint32_t)pos[t + 1] : 0;
        }
        for (int64_t r = 0; r < n_visible; r++)
            for (int64_t i = off[r]; i < off[r + 1]; i++) {
                const int64_t p2 = pos[em[i]]++;
                tile_keys[p2] = em[i];
                ranks[p2] = (uint32_t)r;
            }
        free(pos);
        free(em);
    }
    const int64_t n_inst = off[n_visible];
    free(off);
    return n_inst;
}

/* number of instances, for sizing */
int64_t orc_count_instances(int64_t n_visible, const uint32_t* sorted_idx, const uint32_t* n_touched) {
    int64_t n_inst = 0;
    for (int64_t r = 0; r < n_visible; r++) n_inst += n_touched[sorted_idx[r]];
    return n_inst;
}

/* ------------------------------------------------------------------------------------------------ */
/* blending                                                                                          */

static inline int overlaps_subtile(const orc_rec* q, uint32_t sx0, uint32_t sy0) {
    return q->xmin < sx0 + SUB_W && sx0 < q->xmax && q->ymin < sy0 + SUB_H && sy0 < q->ymax;
}

/* Forward blend of one tile list per pixel. image is [3,H,W] (chw=1) or [H,W,3]; final_T and n_contrib are
 * [H,W] (may be NULL). ranks index sorted_idx; rec is in primitive order. */
int orc_blend(int64_t n_visible, const uint32_t* sorted_idx, const double* rec, const uint32_t* ranks, const uint32_t* ranges,
              const orc_view* v, real* image, real* final_T, uint32_t* n_contrib, int chw, int clamp_out) {
    (void)n_visible;
    const int W = v->width, H = v->height, gw = (W + TILE_W - 1) / TILE_W;
#pragma omp parallel for schedule(dynamic, 1) num_threads(g_threads) if (g_threads > 1)
    for (int py = 0; py < H; py++) {
        for (int px = 0; px < W; px++) {
            const int tx = px / TILE_W, ty = py / TILE_H, tile = ty * gw + tx;
            const uint32_t lx = (uint32_t)(px - tx * TILE_W), ly = (uint32_t)(py - ty * TILE_H);
            const uint32_t sx0 = (uint32_t)(tx * TILE_W) + (lx / SUB_W) * SUB_W, sy0 = (uint32_t)(ty * TILE_H) + (ly / SUB_H) * SUB_H;
            const real pxf = (real)px + R(0.5), pyf = (real)py + R(0.5);
            real cr = R(0.0), cg = R(0.0), cbl = R(0.0), tr = R(1.0);
            uint32_t last = 0;
            const uint32_t s = ranges[2 * tile], e = ranges[2 * tile + 1];
            for (uint32_t j = s; j < e; j++) {
                orc_rec q;
                rec_of(rec, sorted_idx[ranks[j]], &q);
                if (!overlaps_subtile(&q, sx0, sy0)) continue;
                const real dx = q.mx - pxf, dy = q.my - pyf;
                const real alpha = fragment_alpha_r(q.opacity, q.ca, q.cb, q.cc, dx, dy);
                if (alpha < R(0.0)) continue;
                const real w = tr * alpha;
                cr = RFMA(w, q.r, cr);
                cg = RFMA(w, q.g, cg);
                cbl = RFMA(w, q.b, cbl);
                tr = tr * (R(1.0) - alpha);
                last = j - s + 1;
                if (tr < R(1e-4)) break;
            }
            cr = RFMA(tr, (real)v->bg[0], cr);
            cg = RFMA(tr, (real)v->bg[1], cg);
            cbl = RFMA(tr, (real)v->bg[2], cbl);
            if (clamp_out) { cr = sat_r(cr); cg = sat_r(cg); cbl = sat_r(cbl); }
            const size_t pix = (size_t)py * W + px, np = (size_t)W * H;
            if (chw) { image[pix] = cr; image[np + pix] = cg; image[2 * np + pix] = cbl; }
            else { image[3 * pix] = cr; image[3 * pix + 1] = cg; image[3 * pix + 2] = cbl; }
            if (final_T) final_T[pix] = tr;
            if (n_contrib) n_contrib[pix] = last;
        }
    }
    return 0;
}

/* Backward blend in double. grad_image is [3,H,W]. The accepted fragments of a pixel are re-derived in working
 * precision exactly as in the forward (same subtile skip, same threshold), truncated at n_contrib.
 * Output per depth rank (12 doubles): d mean2d (2), d conic (3, off-diagonal halved as the kernels do),
 * d opacity-logit (sigmoid derivative folded in unless proper AA), d color (3), |d mean2d| (2), unused. */
int orc_blend_backward(int64_t n_visible, const uint32_t* sorted_idx, const double* rec, const uint32_t* ranks, const uint32_t* ranges,
                       const orc_view* v, const uint32_t* n_contrib, const float* grad_image, double* grads) {
    const int W = v->width, H = v->height, gw = (W + TILE_W - 1) / TILE_W;
    memset(grads, 0, sizeof(double) * 12 * (size_t)n_visible);
    const size_t np = (size_t)W * H;
    typedef struct { uint32_t r; double alpha, G, dx, dy; } frag;
    const int nt = g_threads;
    /* with several threads each accumulates into its own (lazily zeroed) copy and lists the depth ranks it touched, so
     * combining costs as much as the contributions, not as the whole copies */
    double* parts = nt > 1 ? (double*)calloc((size_t)nt * 12 * (size_t)n_visible, sizeof(double)) : 0;
    uint8_t* seen = nt > 1 ? (uint8_t*)calloc((size_t)nt * (size_t)n_visible, 1) : 0;
    uint32_t** touched = nt > 1 ? (uint32_t**)calloc((size_t)nt, sizeof(uint32_t*)) : 0;
    size_t* n_touched_t = nt > 1 ? (size_t*)calloc((size_t)nt, sizeof(size_t)) : 0;
#pragma omp parallel num_threads(nt) if (nt > 1)
    {
    const int tid = thread_id();
    double* acc = parts ? parts + (size_t)tid * 12 * (size_t)n_visible : grads;
    uint8_t* my_seen = seen ? seen + (size_t)tid * (size_t)n_visible : 0;
    size_t list_cap = 0;
    frag* fr = (frag*)malloc(sizeof(frag) * 1);
    size_t cap = 1;
#pragma omp for schedule(dynamic, 1)
    for (int py = 0; py < H; py++) {
        for (int px = 0; px < W; px++) {
            const int tx = px / TILE_W, ty = py / TILE_H, tile = ty * gw + tx;
            const uint32_t lx = (uint32_t)(px - tx * TILE_W), ly = (uint32_t)(py - ty * TILE_H);
            const uint32_t sx0 = (uint32_t)(tx * TILE_W) + (lx / SUB_W) * SUB_W, sy0 = (uint32_t)(ty * TILE_H) + (ly / SUB_H) * SUB_H;
            const size_t pix = (size_t)py * W + px;
            const uint32_t s = ranges[2 * tile], last = n_contrib[pix];
            size_t nf = 0;
            for (uint32_t j = s; j < s + last; j++) {
                orc_rec q;
                rec_of(rec, sorted_idx[ranks[j]], &q);
                if (!overlaps_subtile(&q, sx0, sy0)) continue;
                const real pxf = (real)px + R(0.5), pyf = (real)py + R(0.5);
                const real dxr = q.mx - pxf, dyr = q.my - pyf;
                if (fragment_alpha_r(q.opacity, q.ca, q.cb, q.cc, dxr, dyr) < R(0.0)) continue;
                const double* o = rec + 14 * (size_t)sorted_idx[ranks[j]];
                const double dx = o[0] - ((double)px + 0.5), dy = o[1] - ((double)py + 0.5);
                const double e = -0.5 * (o[4] * dx * dx + o[6] * dy * dy) - o[5] * dx * dy;
                const double G = exp(fmin(e, 0.0));
                if (nf == cap) { cap *= 2; fr = (frag*)realloc(fr, sizeof(frag) * cap); }
                fr[nf].r = ranks[j]; fr[nf].alpha = o[2] * G; fr[nf].G = G; fr[nf].dx = dx; fr[nf].dy = dy;
                nf++;
            }
            const double g[3] = {grad_image[pix], grad_image[np + pix], grad_image[2 * np + pix]};
            double T = 1.0;
            double C[3] = {0.0, 0.0, 0.0};
            for (size_t k = 0; k < nf; k++) {
                const double* o = rec + 14 * (size_t)sorted_idx[fr[k].r];
                for (int c = 0; c < 3; c++) C[c] += T * fr[k].alpha * o[7 + c];
                T *= 1.0 - fr[k].alpha;
            }
            const double Tfinal = T;
            const double gbg = -Tfinal * (g[0] * v->bg[0] + g[1] * v->bg[1] + g[2] * v->bg[2]);
            double after[3] = {C[0], C[1], C[2]};
            T = 1.0;
            for (size_t k = 0; k < nf; k++) {
                const double* o = rec + 14 * (size_t)sorted_idx[fr[k].r];
                double* gr = acc + 12 * (size_t)fr[k].r;
                if (my_seen && !my_seen[fr[k].r]) {
                    my_seen[fr[k].r] = 1;
                    if (n_touched_t[tid] == list_cap) {
                        list_cap = list_cap ? 2 * list_cap : 1024;
                        touched[tid] = (uint32_t*)realloc(touched[tid], list_cap * sizeof(uint32_t));
                    }
                    touched[tid][n_touched_t[tid]++] = fr[k].r;
                }
                const double a = fr[k].alpha, w = T * a;
                for (int c = 0; c < 3; c++) { gr[5 + c] += w * g[c]; after[c] -= w * o[7 + c]; }
                const double rcp = 1.0 / fmax(1.0 - a, 1e-6);
                double dl_da = gbg * rcp;
                for (int c = 0; c < 3; c++) dl_da += (T * o[7 + c] - after[c] * rcp) * g[c];
                gr[4 + 0] += 0.0;
                const double hlp = -a * dl_da;
                const double dx = fr[k].dx, dy = fr[k].dy;
                gr[2] += 0.5 * hlp * dx * dx;
                gr[3] += 0.5 * hlp * dx * dy;
                gr[4] += 0.5 * hlp * dy * dy;
                const double dmx = hlp * (o[4] * dx + o[5] * dy), dmy = hlp * (o[5] * dx + o[6] * dy);
                gr[0] += dmx; gr[1] += dmy;
                gr[9] += fabs(dmx); gr[10] += fabs(dmy);
                gr[11] += fr[k].G * dl_da;  /* opacity (after AA), finalised below */
                T *= 1.0 - a;
            }
        }
    }
    free(fr);
    }
    if (parts) {
        for (int t = 0; t < nt; t++) {
            const double* pt = parts + (size_t)t * 12 * (size_t)n_visible;
            for (size_t j = 0; j < n_touched_t[t]; j++) {
                const size_t r = touched[t][j];
                for (int k = 0; k < 12; k++) grads[12 * r + k] += pt[12 * r + k];
            }
            free(touched[t]);
        }
        free(parts);
        free(seen);
        free(touched);
        free(n_touched_t);
    }
    for (int64_t r = 0; r < n_visible; r++) {
        double* gr = grads + 12 * (size_t)r;
        const double o = rec[14 * (size_t)sorted_idx[r] + 2];
        const double go = gr[11];
        gr[8] = v->proper_aa ? go : (o - o * o) * go;
        gr[11] = 0.0;
    }
    return 0;
}
/* layout note: grads[r] = {mx, my, ca, cb, cc, col r, col g, col b, opacity, |mx|, |my|, 0} */

/* Pruning scores in double (rasterization/include/kernels_pruning_scores.cuh:11-173): the accepted fragments of a
 * pixel are found as in orc_blend_backward (working-precision acceptance, truncated at n_contrib); with an all-ones
 * colour gradient, scores[primitive] += (opacity * dL/dalpha)^2 for every accepted fragment. scores has one entry
 * per primitive (primitive order) and is accumulated into. */
int orc_pruning_scores(int64_t n_visible, const uint32_t* sorted_idx, const double* rec, const uint32_t* ranks, const uint32_t* ranges,
                       const orc_view* v, const uint32_t* n_contrib, double* scores) {
    (void)n_visible;
    const int W = v->width, H = v->height, gw = (W + TILE_W - 1) / TILE_W;
    uint32_t* prim = (uint32_t*)malloc(sizeof(uint32_t) * 1);
    double* alpha = (double*)malloc(sizeof(double) * 1);
    size_t cap = 1;
    const double bgsum = (double)v->bg[0] + (double)v->bg[1] + (double)v->bg[2];
    for (int py = 0; py < H; py++) {
        for (int px = 0; px < W; px++) {
            const int tx = px / TILE_W, ty = py / TILE_H, tile = ty * gw + tx;
            const uint32_t lx = (uint32_t)(px - tx * TILE_W), ly = (uint32_t)(py - ty * TILE_H);
            const uint32_t sx0 = (uint32_t)(tx * TILE_W) + (lx / SUB_W) * SUB_W, sy0 = (uint32_t)(ty * TILE_H) + (ly / SUB_H) * SUB_H;
            const size_t pix = (size_t)py * W + px;
            const uint32_t s = ranges[2 * tile], last = n_contrib[pix];
            size_t nf = 0;
            for (uint32_t j = s; j < s + last; j++) {
                orc_rec q;
                const uint32_t pi = sorted_idx[ranks[j]];
                rec_of(rec, pi, &q);
                if (!overlaps_subtile(&q, sx0, sy0)) continue;
                const real pxf = (real)px + R(0.5), pyf = (real)py + R(0.5);
                const real dxr = q.mx - pxf, dyr = q.my - pyf;
                if (fragment_alpha_r(q.opacity, q.ca, q.cb, q.cc, dxr, dyr) < R(0.0)) continue;
                const double* o = rec + 14 * (size_t)pi;
                const double dx = o[0] - ((double)px + 0.5), dy = o[1] - ((double)py + 0.5);
                const double e = -0.5 * (o[4] * dx * dx + o[6] * dy * dy) - o[5] * dx * dy;
                if (nf == cap) {
                    cap *= 2;
                    prim = (uint32_t*)realloc(prim, sizeof(uint32_t) * cap);
                    alpha = (double*)realloc(alpha, sizeof(double) * cap);
                }
                prim[nf] = pi;
                alpha[nf] = o[2] * exp(fmin(e, 0.0));
                nf++;
            }
            /* colour sum (all-ones gradient) of the blended colour without background, and the final transmittance */
            double T = 1.0, C = 0.0;
            for (size_t k = 0; k < nf; k++) {
                const double* o = rec + 14 * (size_t)prim[k];
                C += T * alpha[k] * (o[7] + o[8] + o[9]);
                T *= 1.0 - alpha[k];
            }
            const double gbg = -T * bgsum;
            double after = C;
            T = 1.0;
            for (size_t k = 0; k < nf; k++) {
                const double* o = rec + 14 * (size_t)prim[k];
                const double a = alpha[k], cs = o[7] + o[8] + o[9];
                after -= T * a * cs;
                const double rcp = 1.0 / fmax(1.0 - a, 1e-6);
                const double dl_da = T * cs - after * rcp + gbg * rcp;
                const double dl_dg = o[2] * dl_da;
                scores[prim[k]] += dl_dg * dl_dg;
                T *= 1.0 - a;
            }
        }
    }
    free(prim);
    free(alpha);
    return 0;
}

/* ------------------------------------------------------------------------------------------------ */
/* backward preprocess (double)                                                                      */

typedef struct { double m11, m12, m13, m21, m22, m23, m31, m32, m33; } mat3d;

/* gradient outputs: [N,3], [N,3], [N,4], [N], [N,3] precomputed / base, [N,R] residual, [P] mlp (may be NULL) */
int orc_preprocess_backward(const orc_appearance* A, const orc_view* v, int64_t n, const inreal* means, const inreal* scales,
                            const inreal* rots, const inreal* opac, const inreal* precomputed, const inreal* base, const inreal* residual,
                            const inreal* mlp, const uint32_t* rank_of, const double* rec_prim, const double* grads,
                            double* g_means, double* g_scales, double* g_rots, double* g_opac, double* g_pre, double* g_base,
                            double* g_res, double* g_mlp, double* densification, int dens_rows) {
    const int stride = orc_residual_stride(A);
    const double* w = 0;
    double wd[16];
    for (int k = 0; k < 16; k++) wd[k] = v->w2c[k];
    w = wd;
    const size_t n_mlp = (g_mlp && A->model == 5) ? (size_t)neural_param_count(A) : 0;
    if (n_mlp) memset(g_mlp, 0, sizeof(double) * n_mlp);
    const int nt = g_threads;
    double* mlp_parts = (nt > 1 && n_mlp) ? (double*)calloc((size_t)nt * n_mlp, sizeof(double)) : 0;
#pragma omp parallel num_threads(nt) if (nt > 1)
    {
    double* my_mlp = mlp_parts ? mlp_parts + (size_t)thread_id() * n_mlp : g_mlp;
#pragma omp for schedule(dynamic, 64)
    for (int64_t i = 0; i < n; i++) {
        const uint32_t r = rank_of[i];
        if (r == 0xffffffffu) {
            memset(g_means + 3 * i, 0, 3 * sizeof(double));
            memset(g_scales + 3 * i, 0, 3 * sizeof(double));
            memset(g_rots + 4 * i, 0, 4 * sizeof(double));
            g_opac[i] = 0.0;
            if (precomputed) memset(g_pre + 3 * i, 0, 3 * sizeof(double));
            else {
                memset(g_base + 3 * i, 0, 3 * sizeof(double));
                if (stride > 0) memset(g_res + (size_t)i * stride, 0, (size_t)stride * sizeof(double));
            }
            continue;
        }
        const double* gr = grads + 12 * (size_t)r;
        const double* q = rec_prim + 14 * (size_t)i;
        const v3_d gcol = mk_d(gr[5], gr[6], gr[7]);
        const v3_d m = mk_d(means[3 * i], means[3 * i + 1], means[3 * i + 2]);
        v3_d gmean_color = mk_d(0.0, 0.0, 0.0);
        if (precomputed) {
            g_pre[3 * i] = gcol.x; g_pre[3 * i + 1] = gcol.y; g_pre[3 * i + 2] = gcol.z;
        } else {
            const v3_d gpre = mul_d(gcol, mk_d(color_act_grad_d(A->color_act, q[7]), color_act_grad_d(A->color_act, q[8]),
                                               color_act_grad_d(A->color_act, q[9])));
            for (int c = 0; c < 3; c++)
                g_base[3 * i + c] = v->render_base ? base_act_grad_d(A->base_act, base[3 * i + c]) * (c == 0 ? gpre.x : (c == 1 ? gpre.y : gpre.z)) : 0.0;
            const v3_d dv = sub_d(m, mk_d(v->cam[0], v->cam[1], v->cam[2]));
            const double rn = 1.0 / sqrt(fmax(dot_d(dv, dv), 1e-24));
            const v3_d d = scl_d(rn, dv);
            /* the direction as the forward computed it (working precision), for the Neural inputs */
            const v3_r dv_r = sub_r(mk_r(means[3 * i], means[3 * i + 1], means[3 * i + 2]), mk_r(v->cam[0], v->cam[1], v->cam[2]));
            const v3_r d_r = scl_r(R(1.0) / sqrt(fmax(dot_r(dv_r, dv_r), R(1e-24))), dv_r);
            const int deg = v->degree < A->max_degree ? v->degree : A->max_degree;
            const inreal* rp = residual ? residual + (size_t)i * stride : 0;
            double local[128];
            memset(local, 0, sizeof(local));
            v3_d gd = mk_d(0.0, 0.0, 0.0);
            switch (A->model) {
                case 1: gd = sh_backward_d(rp, gpre, d, deg, A->res_act, local); break;
                case 2: gd = sv_backward_d(rp, gpre, d, deg, A->res_act, local); break;
                case 3: gd = lobes_backward_d(rp, gpre, d, deg, A->res_act, 0, local); break;
                case 4: gd = lobes_backward_d(rp, gpre, d, deg, A->res_act, 1, local); break;
                case 5: gd = neural_backward_d(A, rp, base + 3 * i, gpre, d, d_r, deg, mlp, local, my_mlp, g_base + 3 * i); break;
                default: break;
            }
            const int active = residual_active(A, deg);
            for (int k = 0; k < stride; k++) g_res[(size_t)i * stride + k] = k < active ? local[k] : 0.0;
            gmean_color = scl_d(rn, sub_d(gd, scl_d(dot_d(gd, d), d)));
        }
        /* geometry chain rule */
        const double depth = w[8] * m.x + w[9] * m.y + w[10] * m.z + w[11];
        const double x = (w[0] * m.x + w[1] * m.y + w[2] * m.z + w[3]) / depth;
        const double y = (w[4] * m.x + w[5] * m.y + w[6] * m.z + w[7]) / depth;
        const double vx = exp(2.0 * (double)scales[3 * i]), vy = exp(2.0 * (double)scales[3 * i + 1]), vz = exp(2.0 * (double)scales[3 * i + 2]);
        const double qr = rots[4 * i], qx = rots[4 * i + 1], qy = rots[4 * i + 2], qz = rots[4 * i + 3];
        mat3d Rm;
        {
            const double xx = qx * qx, yy = qy * qy, zz = qz * qz, xy = qx * qy, xz = qx * qz, yz = qy * qz, rx = qr * qx, ry = qr * qy, rz = qr * qz;
            const double s = 1.0 / (qr * qr + xx + yy + zz);
            Rm.m11 = 1.0 - 2.0 * (yy + zz) * s; Rm.m12 = 2.0 * (xy - rz) * s; Rm.m13 = 2.0 * (xz + ry) * s;
            Rm.m21 = 2.0 * (xy + rz) * s; Rm.m22 = 1.0 - 2.0 * (xx + zz) * s; Rm.m23 = 2.0 * (yz - rx) * s;
            Rm.m31 = 2.0 * (xz - ry) * s; Rm.m32 = 2.0 * (yz + rx) * s; Rm.m33 = 1.0 - 2.0 * (xx + yy) * s;
        }
        const mat3d RS = {Rm.m11 * vx, Rm.m12 * vy, Rm.m13 * vz, Rm.m21 * vx, Rm.m22 * vy, Rm.m23 * vz, Rm.m31 * vx, Rm.m32 * vy, Rm.m33 * vz};
        const double s11 = RS.m11 * Rm.m11 + RS.m12 * Rm.m12 + RS.m13 * Rm.m13, s12 = RS.m11 * Rm.m21 + RS.m12 * Rm.m22 + RS.m13 * Rm.m23;
        const double s13 = RS.m11 * Rm.m31 + RS.m12 * Rm.m32 + RS.m13 * Rm.m33, s22 = RS.m21 * Rm.m21 + RS.m22 * Rm.m22 + RS.m23 * Rm.m23;
        const double s23 = RS.m21 * Rm.m31 + RS.m22 * Rm.m32 + RS.m23 * Rm.m33, s33 = RS.m31 * Rm.m31 + RS.m32 * Rm.m32 + RS.m33 * Rm.m33;
        const double Wd = v->width, Hd = v->height;
        const double cl = (-0.15 * Wd - v->cx) / v->fx, cr = (1.15 * Wd - v->cx) / v->fx;
        const double ct = (-0.15 * Hd - v->cy) / v->fy, cbm = (1.15 * Hd - v->cy) / v->fy;
        const double xc = fmin(fmax(x, cl), cr), yc = fmin(fmax(y, ct), cbm);
        const double j11 = v->fx / depth, j13 = -j11 * xc, j22 = v->fy / depth, j23 = -j22 * yc;
        const v3_d a1 = mk_d(j11 * w[0] + j13 * w[8], j11 * w[1] + j13 * w[9], j11 * w[2] + j13 * w[10]);
        const v3_d a2 = mk_d(j22 * w[4] + j23 * w[8], j22 * w[5] + j23 * w[9], j22 * w[6] + j23 * w[10]);
        const v3_d b1 = mk_d(a1.x * s11 + a1.y * s12 + a1.z * s13, a1.x * s12 + a1.y * s22 + a1.z * s23, a1.x * s13 + a1.y * s23 + a1.z * s33);
        const v3_d b2 = mk_d(a2.x * s11 + a2.y * s12 + a2.z * s13, a2.x * s12 + a2.y * s22 + a2.z * s23, a2.x * s13 + a2.y * s23 + a2.z * s33);
        const double a_raw = dot_d(b1, a1), b = dot_d(b1, a2), c_raw = dot_d(b2, a2);
        const double kd = v->proper_aa ? 0.1 : 0.3;
        const double a = a_raw + kd, c = c_raw + kd;
        const double aa = a * a, bb = b * b, cc = c * c, ac = a * c, ab = a * b, bc = b * c;
        const double det = ac - bb, inv2 = 1.0 / (det * det);
        const double gca = gr[2], gcb = gr[3], gcc = gr[4];
        const double gA = inv2 * (2.0 * bc * gcb - cc * gca - bb * gcc);
        const double gB = inv2 * (bc * gca - (ac + bb) * gcb + ab * gcc);
        const double gC = inv2 * (2.0 * ab * gcb - bb * gca - aa * gcc);
        double gop = gr[8];
        if (v->proper_aa) {
            const double o = 1.0 / (1.0 + exp(-(double)opac[i]));
            gop = gop * sqrt(fmax((a_raw * c_raw - bb) / det, 0.0)) * o * (1.0 - o);
        }
        g_opac[i] = gop;
        const double d11 = a1.x * a1.x * gA + 2.0 * a1.x * a2.x * gB + a2.x * a2.x * gC;
        const double d12 = a1.x * a1.y * gA + (a1.x * a2.y + a1.y * a2.x) * gB + a2.x * a2.y * gC;
        const double d13 = a1.x * a1.z * gA + (a1.x * a2.z + a1.z * a2.x) * gB + a2.x * a2.z * gC;
        const double d22 = a1.y * a1.y * gA + 2.0 * a1.y * a2.y * gB + a2.y * a2.y * gC;
        const double d23 = a1.y * a1.z * gA + (a1.y * a2.z + a1.z * a2.y) * gB + a2.y * a2.z * gC;
        const double d33 = a1.z * a1.z * gA + 2.0 * a1.z * a2.z * gB + a2.z * a2.z * gC;
        const v3_d ga1 = scl_d(2.0, mk_d(b1.x * gA + b2.x * gB, b1.y * gA + b2.y * gB, b1.z * gA + b2.z * gB));
        const v3_d ga2 = scl_d(2.0, mk_d(b1.x * gB + b2.x * gC, b1.y * gB + b2.y * gC, b1.z * gB + b2.z * gC));
        const double gj11 = w[0] * ga1.x + w[1] * ga1.y + w[2] * ga1.z;
        const double gj22 = w[4] * ga2.x + w[5] * ga2.y + w[6] * ga2.z;
        const double gj13 = w[8] * ga1.x + w[9] * ga1.y + w[10] * ga1.z;
        const double gj23 = w[8] * ga2.x + w[9] * ga2.y + w[10] * ga2.z;
        const double gmx = gr[0], gmy = gr[1];
        if (densification) {
            densification[i] += 1.0;
            const double nx = 0.5 * gmx * Wd, ny = 0.5 * gmy * Hd;
            densification[n + i] += sqrt(nx * nx + ny * ny);
            if (dens_rows == 3) {
                const double ax = 0.5 * gr[9] * Wd, ay = 0.5 * gr[10] * Hd;
                densification[2 * n + i] += sqrt(ax * ax + ay * ay);
            }
        }
        v3_d gcam = mk_d(j11 * gmx, j22 * gmy, -j11 * x * gmx - j22 * y * gmy);
        const int vxo = x >= cl && x <= cr, vyo = y >= ct && y <= cbm;
        if (vxo) gcam.x -= j11 * gj13 / depth;
        if (vyo) gcam.y -= j22 * gj23 / depth;
        const double fxm = 1.0 + vxo, fym = 1.0 + vyo;
        gcam.z += (j11 * (fxm * xc * gj13 - gj11) + j22 * (fym * yc * gj23 - gj22)) / depth;
        const v3_d gmean = mk_d(w[0] * gcam.x + w[4] * gcam.y + w[8] * gcam.z, w[1] * gcam.x + w[5] * gcam.y + w[9] * gcam.z,
                                w[2] * gcam.x + w[6] * gcam.y + w[10] * gcam.z);
        const v3_d gm = A->dir_grad && !precomputed ? add_d(gmean, gmean_color) : gmean;
        g_means[3 * i] = gm.x; g_means[3 * i + 1] = gm.y; g_means[3 * i + 2] = gm.z;
        const double gv1 = Rm.m11 * Rm.m11 * d11 + Rm.m21 * Rm.m21 * d22 + Rm.m31 * Rm.m31 * d33 + 2.0 * (Rm.m11 * Rm.m21 * d12 + Rm.m11 * Rm.m31 * d13 + Rm.m21 * Rm.m31 * d23);
        const double gv2 = Rm.m12 * Rm.m12 * d11 + Rm.m22 * Rm.m22 * d22 + Rm.m32 * Rm.m32 * d33 + 2.0 * (Rm.m12 * Rm.m22 * d12 + Rm.m12 * Rm.m32 * d13 + Rm.m22 * Rm.m32 * d23);
        const double gv3 = Rm.m13 * Rm.m13 * d11 + Rm.m23 * Rm.m23 * d22 + Rm.m33 * Rm.m33 * d33 + 2.0 * (Rm.m13 * Rm.m23 * d12 + Rm.m13 * Rm.m33 * d13 + Rm.m23 * Rm.m33 * d23);
        g_scales[3 * i] = 2.0 * vx * gv1; g_scales[3 * i + 1] = 2.0 * vy * gv2; g_scales[3 * i + 2] = 2.0 * vz * gv3;
        const mat3d gR = {2.0 * (RS.m11 * d11 + RS.m21 * d12 + RS.m31 * d13), 2.0 * (RS.m12 * d11 + RS.m22 * d12 + RS.m32 * d13),
                          2.0 * (RS.m13 * d11 + RS.m23 * d12 + RS.m33 * d13), 2.0 * (RS.m11 * d12 + RS.m21 * d22 + RS.m31 * d23),
                          2.0 * (RS.m12 * d12 + RS.m22 * d22 + RS.m32 * d23), 2.0 * (RS.m13 * d12 + RS.m23 * d22 + RS.m33 * d23),
                          2.0 * (RS.m11 * d13 + RS.m21 * d23 + RS.m31 * d33), 2.0 * (RS.m12 * d13 + RS.m22 * d23 + RS.m32 * d33),
                          2.0 * (RS.m13 * d13 + RS.m23 * d23 + RS.m33 * d33)};
        {
            const double xx = qx * qx, yy = qy * qy, zz = qz * qz, xy = qx * qy, xz = qx * qz, yz = qy * qz, rx = qr * qx, ry = qr * qy, rz = qr * qz;
            const double t = 2.0 / (qr * qr + xx + yy + zz);
            const double g_xx = gR.m22 + gR.m33, g_yy = gR.m11 + gR.m33, g_zz = gR.m11 + gR.m22;
            const double g_rz = gR.m21 - gR.m12, g_xy = gR.m21 + gR.m12, g_ry = gR.m13 - gR.m31, g_xz = gR.m13 + gR.m31;
            const double g_rx = gR.m32 - gR.m23, g_yz = gR.m32 + gR.m23;
            const double h = t * (xy * g_xy + xz * g_xz + yz * g_yz + rx * g_rx + ry * g_ry + rz * g_rz - xx * g_xx - yy * g_yy - zz * g_zz);
            g_rots[4 * i] = t * (qx * g_rx + qy * g_ry + qz * g_rz - qr * h);
            g_rots[4 * i + 1] = t * (qr * g_rx - 2.0 * qx * g_xx + qy * g_xy + qz * g_xz - qx * h);
            g_rots[4 * i + 2] = t * (qr * g_ry + qx * g_xy - 2.0 * qy * g_yy + qz * g_yz - qy * h);
            g_rots[4 * i + 3] = t * (qr * g_rz + qx * g_xz + qy * g_yz - 2.0 * qz * g_zz - qz * h);
        }
    }
    }
    if (mlp_parts) {
        for (int t = 0; t < nt; t++)
            for (size_t k = 0; k < n_mlp; k++) g_mlp[k] += mlp_parts[(size_t)t * n_mlp + k];
        free(mlp_parts);
    }
    return 0;
}

/* ------------------------------------------------------------------------------------------------ */
/* adam (adam.cu:18-42 / :62-72): one tensor, float arithmetic with the same operation order          */

void orc_adam(int64_t n, float* param, const float* grad, float* m, float* v, int64_t step, const double* lrs, int n_lr,
              int64_t col_offset, double beta1, double beta2, double eps) {
    const double bc1 = 1.0 / (1.0 - pow(beta1, (double)step));
    const double bc2 = 1.0 / sqrt(1.0 - pow(beta2, (double)step));
    float lr[7];
    for (int k = 0; k < n_lr; k++) lr[k] = (float)(lrs[k] * bc1);
    const float b1 = (float)beta1, b2 = (float)beta2, e = (float)eps, c2 = (float)bc2;
    #pragma omp parallel for schedule(static) num_threads(g_threads) if (g_threads > 1)
    for (int64_t j = 0; j < n; j++) {
        const float g = grad[j], g2 = g * g;
        const float mm = fmaf(b1, m[j] - g, g);
        const float vv = fmaf(b2, v[j] - g2, g2);
        const float denom = sqrtf(vv) * c2 + e;
        param[j] -= lr[(col_offset + j) % n_lr] * mm / denom;
        m[j] = mm;
        v[j] = vv;
    }
}

/* exposes the deterministic functions for direct tests */
float orc_det_exp(float x) { return det_exp_f(x); }
float orc_det_exp_blend(float x) { return det_exp_blend_f(x); }
float orc_det_log(float x) { return det_log_f(x); }
void orc_det_sincos(float x, float* s, float* c) { det_sincos_f(x, s, c); }
int orc_is_double(void) {
#ifdef ORC_DOUBLE
    return 1;
#else
    return 0;
#endif
}

/* ------------------------------------------------------------------------------------------------ */
/* appearance alone (for the golden vectors of the reference's PyTorch modules)                      */

static v3_d appearance_color_d(const orc_appearance* A, int64_t i, const inreal* means, const float* cam, const inreal* base,
                               const inreal* residual, const inreal* mlp, int degree, v3_d* d_out, double* rn_out) {
    const v3_d dv = sub_d(mk_d(means[3 * i], means[3 * i + 1], means[3 * i + 2]), mk_d(cam[0], cam[1], cam[2]));
    const double rn = 1.0 / sqrt(fmax(dot_d(dv, dv), 1e-24));
    const v3_d d = scl_d(rn, dv);
    const int stride = orc_residual_stride(A);
    const inreal* rp = residual + (size_t)i * stride;
    const int deg = degree < A->max_degree ? degree : A->max_degree;
    v3_d res = mk_d(0.0, 0.0, 0.0);
    switch (A->model) {
        case 1: res = sh_forward_d(rp, d, deg, A->res_act); break;
        case 2: res = sv_forward_d(rp, d, deg, A->res_act); break;
        case 3: res = lobes_forward_d(rp, d, deg, A->res_act, 0); break;
        case 4: res = lobes_forward_d(rp, d, deg, A->res_act, 1); break;
        default: break;
    }
    double s[3];
    for (int c = 0; c < 3; c++) {
        const double b = base[3 * i + c];
        s[c] = (A->base_act == 1 ? exp(3.0 * b) : b) + (c == 0 ? res.x : (c == 1 ? res.y : res.z));
    }
    v3_d col;
    double y[3];
    for (int c = 0; c < 3; c++) {
        const double x = s[c];
        switch (A->color_act) {
            case 1: y[c] = fmax(x + 0.5, 0.0); break;
            case 2: y[c] = softplus10_d(x + 0.5); break;
            case 3: y[c] = 1.0 / (1.0 + exp(-4.0 * x)); break;
            case 4: y[c] = fmin(fmax(x + 0.5, 0.0), 1.0); break;
            case 5: y[c] = -expm1(-x); break;
            default: y[c] = x + 0.5; break;
        }
    }
    col = mk_d(y[0], y[1], y[2]);
    if (d_out) *d_out = d;
    if (rn_out) *rn_out = rn;
    return col;
}

/* colors [N,3] (double) of the fused appearance at the given degree */
int orc_appearance_eval(const orc_appearance* A, int64_t n, const inreal* means, const float* cam, const inreal* base, const inreal* residual,
                        int degree, double* colors) {
    for (int64_t i = 0; i < n; i++) {
        const v3_d c = appearance_color_d(A, i, means, cam, base, residual, 0, degree, 0, 0);
        colors[3 * i] = c.x; colors[3 * i + 1] = c.y; colors[3 * i + 2] = c.z;
    }
    return 0;
}

/* gradients of sum(colors * upstream) w.r.t. base [N,3], residual [N,R] and means [N,3] (view-direction path) */
int orc_appearance_grad(const orc_appearance* A, int64_t n, const inreal* means, const float* cam, const inreal* base, const inreal* residual,
                        int degree, const double* upstream, double* g_base, double* g_res, double* g_means) {
    const int stride = orc_residual_stride(A);
    for (int64_t i = 0; i < n; i++) {
        v3_d d;
        double rn;
        const v3_d col = appearance_color_d(A, i, means, cam, base, residual, 0, degree, &d, &rn);
        const v3_d gpre = mul_d(mk_d(upstream[3 * i], upstream[3 * i + 1], upstream[3 * i + 2]),
                                mk_d(color_act_grad_d(A->color_act, col.x), color_act_grad_d(A->color_act, col.y),
                                     color_act_grad_d(A->color_act, col.z)));
        for (int c = 0; c < 3; c++) g_base[3 * i + c] = base_act_grad_d(A->base_act, base[3 * i + c]) * (c == 0 ? gpre.x : (c == 1 ? gpre.y : gpre.z));
        const int deg = degree < A->max_degree ? degree : A->max_degree;
        const inreal* rp = residual + (size_t)i * stride;
        double local[128];
        memset(local, 0, sizeof(local));
        v3_d gd = mk_d(0.0, 0.0, 0.0);
        switch (A->model) {
            case 1: gd = sh_backward_d(rp, gpre, d, deg, A->res_act, local); break;
            case 2: gd = sv_backward_d(rp, gpre, d, deg, A->res_act, local); break;
            case 3: gd = lobes_backward_d(rp, gpre, d, deg, A->res_act, 0, local); break;
            case 4: gd = lobes_backward_d(rp, gpre, d, deg, A->res_act, 1, local); break;
            default: break;
        }
        const int active = residual_active(A, deg);
        for (int k = 0; k < stride; k++) g_res[(size_t)i * stride + k] = k < active ? local[k] : 0.0;
        const v3_d gm = scl_d(rn, sub_d(gd, scl_d(dot_d(gd, d), d)));
        g_means[3 * i] = gm.x; g_means[3 * i + 1] = gm.y; g_means[3 * i + 2] = gm.z;
    }
    return 0;
}

/* trace of the preprocess intermediates of primitive i into out[18] (debugging aid) */
int orc_preprocess_trace(const orc_appearance* A, const orc_view* v, int64_t i, const inreal* means, const inreal* scales, const inreal* rots,
                         const inreal* opac, double* out) {
    orc_rec q;
    real depth;
    for (int k = 0; k < 18; k++) out[k] = -1.0;
    g_trace = out;
    const uint32_t c = preprocess_one(A, v, i, means, scales, rots, opac, &q, &depth);
    g_trace = 0;
    return (int)c;
}
