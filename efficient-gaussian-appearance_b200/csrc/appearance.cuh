// View-dependent residual models evaluated inside the preprocess kernels: spherical harmonics (degree
// 1..3 bands), soft spherical Voronoi, NASG and NASGabor lobes. Each model has a forward that returns the
// residual for the unit view direction and a backward that writes the per-Gaussian parameter gradients
// and returns the gradient with respect to the unnormalized view vector (mean - camera position).
//
// Math follows the reference chunks FasterGSVDACudaBackend/.../rasterization/rtc/appearance_sh.cuh:30-157,
// appearance_sv.cuh:26-139, appearance_nasg.cuh:39-209, appearance_nasgabor.cuh:53-223 and the PyTorch
// twins Appearance/SH.py:34-56, SV.py:125-132, NASG.py:175-200, NASGabor.py:244-271.
#pragma once

#include "fgs_common.cuh"

namespace fgs {

// ---------------------------------------------------------------------------------------------------
// spherical harmonics: the residual is act(sum_k Y_k(d) c_k) over the bands 1..degree (15 bases max).
// Real SH normalisation constants (sqrt((2l+1)/(4 pi) (l-m)!/(l+m)!) with the usual factors folded in).
constexpr float kShC1 = 0.48860251190291987f;
constexpr float kShC2a = 1.0925484305920792f;
constexpr float kShC2b = 0.94617469575755997f;
constexpr float kShC2c = 0.31539156525251999f;
constexpr float kShC2d = 0.54627421529603959f;
constexpr float kShC3a = 0.59004358992664352f;
constexpr float kShC3b = 1.7701307697799304f;
constexpr float kShC3c = 2.8906114426405538f;
constexpr float kShC3d = 0.45704579946446572f;
constexpr float kShC3e = 2.2852289973223288f;
constexpr float kShC3f = 1.865881662950577f;
constexpr float kShC3g = 1.1195289977703462f;
constexpr float kShC3h = 1.4453057213202769f;

// basis values Y_0..Y_{n-1} of the bands 1..degree for a unit direction
__device__ inline int sh_basis(f3 d, int degree, float* Y) {
    const float x = d.x, y = d.y, z = d.z;
    Y[0] = -kShC1 * y;
    Y[1] = kShC1 * z;
    Y[2] = -kShC1 * x;
    if (degree < 2) return 3;
    const float xx = x * x, yy = y * y, zz = z * z, xy = x * y, xz = x * z, yz = y * z;
    Y[3] = kShC2a * xy;
    Y[4] = -kShC2a * yz;
    Y[5] = kShC2b * zz - kShC2c;
    Y[6] = -kShC2a * xz;
    Y[7] = kShC2d * (xx - yy);
    if (degree < 3) return 8;
    Y[8] = y * (kShC3a * yy - kShC3b * xx);
    Y[9] = kShC3c * xy * z;
    Y[10] = y * (kShC3d - kShC3e * zz);
    Y[11] = z * (kShC3f * zz - kShC3g);
    Y[12] = x * (kShC3d - kShC3e * zz);
    Y[13] = kShC3h * z * (xx - yy);
    Y[14] = x * (kShC3b * yy - kShC3a * xx);
    return 15;
}

// gradient of the basis with respect to the (unit) direction, one row per basis function
__device__ inline void sh_basis_grad(f3 d, int degree, f3* dY) {
    const float x = d.x, y = d.y, z = d.z;
    dY[0] = mk3(0.0f, -kShC1, 0.0f);
    dY[1] = mk3(0.0f, 0.0f, kShC1);
    dY[2] = mk3(-kShC1, 0.0f, 0.0f);
    if (degree < 2) return;
    const float xx = x * x, yy = y * y, zz = z * z;
    dY[3] = mk3(kShC2a * y, kShC2a * x, 0.0f);
    dY[4] = mk3(0.0f, -kShC2a * z, -kShC2a * y);
    dY[5] = mk3(0.0f, 0.0f, 2.0f * kShC2b * z);
    dY[6] = mk3(-kShC2a * z, 0.0f, -kShC2a * x);
    dY[7] = mk3(2.0f * kShC2d * x, -2.0f * kShC2d * y, 0.0f);
    if (degree < 3) return;
    dY[8] = mk3(-2.0f * kShC3b * x * y, 3.0f * kShC3a * yy - kShC3b * xx, 0.0f);
    dY[9] = mk3(kShC3c * y * z, kShC3c * x * z, kShC3c * x * y);
    dY[10] = mk3(0.0f, kShC3d - kShC3e * zz, -2.0f * kShC3e * y * z);
    dY[11] = mk3(0.0f, 0.0f, 3.0f * kShC3f * zz - kShC3g);
    dY[12] = mk3(kShC3d - kShC3e * zz, 0.0f, -2.0f * kShC3e * x * z);
    dY[13] = mk3(2.0f * kShC3h * x * z, -2.0f * kShC3h * y * z, kShC3h * (xx - yy));
    dY[14] = mk3(kShC3b * yy - 3.0f * kShC3a * xx, 2.0f * kShC3b * x * y, 0.0f);
}

// coeffs: this Gaussian's rest coefficients, laid out [n_rest][3]
__device__ inline f3 sh_forward(const float* coeffs, f3 d, int degree, int res_act) {
    if (degree <= 0) return mk3(0.0f, 0.0f, 0.0f);
    float Y[15];
    const int n = sh_basis(d, degree, Y);
    f3 s = mk3(0.0f, 0.0f, 0.0f);
    for (int k = 0; k < n; k++) s = s + Y[k] * mk3(coeffs[3 * k], coeffs[3 * k + 1], coeffs[3 * k + 2]);
    return residual_act3(res_act, s);
}

// g: gradient w.r.t. the residual; writes the active coefficient gradients; returns d/d(unit direction)
__device__ inline f3 sh_backward(const float* coeffs, f3 g, f3 d, int degree, int res_act, float* grad_coeffs) {
    if (degree <= 0) return mk3(0.0f, 0.0f, 0.0f);
    float Y[15];
    const int n = sh_basis(d, degree, Y);
    f3 s = mk3(0.0f, 0.0f, 0.0f);
    for (int k = 0; k < n; k++) s = s + Y[k] * mk3(coeffs[3 * k], coeffs[3 * k + 1], coeffs[3 * k + 2]);
    const f3 r = residual_act3(res_act, s);
    const f3 gs = g * mk3(residual_act_grad_from_y(res_act, r.x), residual_act_grad_from_y(res_act, r.y),
                          residual_act_grad_from_y(res_act, r.z));
    f3 dY[15];
    sh_basis_grad(d, degree, dY);
    f3 gd = mk3(0.0f, 0.0f, 0.0f);
    for (int k = 0; k < n; k++) {
        const f3 c = mk3(coeffs[3 * k], coeffs[3 * k + 1], coeffs[3 * k + 2]);
        grad_coeffs[3 * k] = Y[k] * gs.x;
        grad_coeffs[3 * k + 1] = Y[k] * gs.y;
        grad_coeffs[3 * k + 2] = Y[k] * gs.z;
        gd = gd + dot3(c, gs) * dY[k];
    }
    return gd;
}

// ---------------------------------------------------------------------------------------------------
// soft spherical Voronoi: site_k = normalize(raw_k), logit_k = -exp(tau_k) |site_k - d|,
// residual = sum_k softmax(logit)_k act(color_k); 7 raw values per site [xyz, tau, rgb]
constexpr int kSvStride = 7;
constexpr float kSvEps = 1e-12f;

__device__ inline f3 sv_forward(const float* p, f3 d, int n_sites, int res_act) {
    if (n_sites <= 0) return mk3(0.0f, 0.0f, 0.0f);
    float max_logit = -3.0e38f;
    for (int k = 0; k < n_sites; k++) {
        const float* s = p + kSvStride * k;
        const f3 raw = mk3(s[0], s[1], s[2]);
        const f3 site = (1.0f / fmaxf(sqrtf(dot3(raw, raw)), kSvEps)) * raw;
        const f3 diff = site - d;
        const float logit = -expf(s[3]) * sqrtf(dot3(diff, diff));
        max_logit = fmaxf(max_logit, logit);
    }
    float wsum = 0.0f;
    f3 acc = mk3(0.0f, 0.0f, 0.0f);
    for (int k = 0; k < n_sites; k++) {
        const float* s = p + kSvStride * k;
        const f3 raw = mk3(s[0], s[1], s[2]);
        const f3 site = (1.0f / fmaxf(sqrtf(dot3(raw, raw)), kSvEps)) * raw;
        const f3 diff = site - d;
        const float w = expf(-expf(s[3]) * sqrtf(dot3(diff, diff)) - max_logit);
        wsum += w;
        acc = acc + w * residual_act3(res_act, mk3(s[4], s[5], s[6]));
    }
    return (1.0f / wsum) * acc;
}

__device__ inline f3 sv_backward(const float* p, f3 g, f3 d, int n_sites, int res_act, float* gp) {
    if (n_sites <= 0) return mk3(0.0f, 0.0f, 0.0f);
    float max_logit = -3.0e38f;
    for (int k = 0; k < n_sites; k++) {
        const float* s = p + kSvStride * k;
        const f3 raw = mk3(s[0], s[1], s[2]);
        const f3 site = (1.0f / fmaxf(sqrtf(dot3(raw, raw)), kSvEps)) * raw;
        const f3 diff = site - d;
        max_logit = fmaxf(max_logit, -expf(s[3]) * sqrtf(dot3(diff, diff)));
    }
    float wsum = 0.0f;
    f3 acc = mk3(0.0f, 0.0f, 0.0f);
    for (int k = 0; k < n_sites; k++) {
        const float* s = p + kSvStride * k;
        const f3 raw = mk3(s[0], s[1], s[2]);
        const f3 site = (1.0f / fmaxf(sqrtf(dot3(raw, raw)), kSvEps)) * raw;
        const f3 diff = site - d;
        const float w = expf(-expf(s[3]) * sqrtf(dot3(diff, diff)) - max_logit);
        wsum += w;
        acc = acc + w * residual_act3(res_act, mk3(s[4], s[5], s[6]));
    }
    const float inv = 1.0f / wsum;
    const float g_mean = dot3(g, inv * acc);   // <g, residual>
    f3 gd = mk3(0.0f, 0.0f, 0.0f);
    for (int k = 0; k < n_sites; k++) {
        const float* s = p + kSvStride * k;
        float* o = gp + kSvStride * k;
        const f3 raw = mk3(s[0], s[1], s[2]);
        const float inv_len = 1.0f / fmaxf(sqrtf(dot3(raw, raw)), kSvEps);
        const f3 site = inv_len * raw;
        const f3 diff = site - d;
        const float dist = sqrtf(dot3(diff, diff));
        const float tau = expf(s[3]);
        const float w = expf(-tau * dist - max_logit) * inv;
        const f3 col = residual_act3(res_act, mk3(s[4], s[5], s[6]));
        o[4] = w * g.x * residual_act_grad_from_y(res_act, col.x);
        o[5] = w * g.y * residual_act_grad_from_y(res_act, col.y);
        o[6] = w * g.z * residual_act_grad_from_y(res_act, col.z);
        const float g_logit = w * (dot3(g, col) - g_mean);
        o[3] = -dist * tau * g_logit;
        const f3 g_diff = (-tau * g_logit / fmaxf(dist, kSvEps)) * diff;
        const f3 g_site = inv_len * (g_diff - dot3(g_diff, site) * site);
        o[0] = g_site.x;
        o[1] = g_site.y;
        o[2] = g_site.z;
        gd = gd - g_diff;
    }
    return gd;
}

// ---------------------------------------------------------------------------------------------------
// NASG / NASGabor lobes. Raw values per lobe: [0..2] frame angles (tanh -> cosines), [3] sharpness
// (exp), [4] anisotropy (exp), NASGabor only: [5] frequency (tanh -> (t + 1) * 20), then rgb weights.
constexpr float kTwoPi = 6.28318530717958647692f;
constexpr float kLobeEps = 5e-6f;
constexpr float kLobeEpsNorm = 1e-8f;
constexpr float kLobeCosLimit = 0.999999f;
constexpr float kLobePoleLimit = 0.99999988f;
constexpr float kLobeShapeLimit = 1e4f;
constexpr float kGaborScale = 20.0f;

struct Lobe {
    f3 x, z;
    float ct, cp, cu, st, sp, su;  // cos/sin of theta, phi, tau
};

__device__ inline Lobe make_lobe(float ct, float cp, float cu) {
    Lobe L;
    L.ct = ct; L.cp = cp; L.cu = cu;
    L.st = sqrtf(1.0f - ct * ct);
    L.sp = sqrtf(1.0f - cp * cp);
    L.su = sqrtf(1.0f - cu * cu);
    L.x = mk3(ct * cp * cu - L.st * L.su, L.st * cp * cu + ct * L.su, -L.sp * cu);
    L.z = mk3(ct * L.sp, L.st * L.sp, cp);
    return L;
}

template <bool kGabor>
__device__ inline f3 lobes_forward(const float* p, f3 d, int n_lobes, int res_act) {
    constexpr int stride = kGabor ? 9 : 8;
    constexpr int wofs = kGabor ? 6 : 5;
    f3 out = mk3(0.0f, 0.0f, 0.0f);
    for (int l = 0; l < n_lobes; l++) {
        const float* q = p + stride * l;
        const Lobe L = make_lobe(clampf(tanhf(q[0]), -kLobeCosLimit, kLobeCosLimit),
                                 clampf(tanhf(q[1]), -kLobeCosLimit, kLobeCosLimit),
                                 clampf(tanhf(q[2]), -kLobeCosLimit, kLobeCosLimit));
        const float lam = fminf(expf(q[3]), kLobeShapeLimit);
        const float a = fminf(expf(q[4]), kLobeShapeLimit);
        const float vz = dot3(d, L.z), vx = dot3(d, L.x);
        const float vzc = clampf(vz, -kLobePoleLimit, kLobePoleLimit);
        const float K = 0.5f * (vzc + 1.0f);
        const float Ke = kLobeEps + a * vx * vx / (1.0f - vzc * vzc);
        const float E = powf(K, Ke);
        const float Nn = lam * sqrtf(1.0f + a) / (kTwoPi * (1.0f + kLobeEpsNorm - expf(-2.0f * lam)));
        const float P = expf(2.0f * lam * (E * K - 1.0f));
        float G = 1.0f;
        if (kGabor) G = 0.5f * (1.0f + cosf((tanhf(q[5]) + 1.0f) * kGaborScale * vx));
        const float pdf = vz >= kLobePoleLimit ? 1.0f : (vz > -kLobePoleLimit ? P * E * G * Nn : 0.0f);
        out = out + pdf * residual_act3(res_act, mk3(q[wofs], q[wofs + 1], q[wofs + 2]));
    }
    return out;
}

template <bool kGabor>
__device__ inline f3 lobes_backward(const float* p, f3 g, f3 d, int n_lobes, int res_act, float* gp) {
    constexpr int stride = kGabor ? 9 : 8;
    constexpr int wofs = kGabor ? 6 : 5;
    f3 gd = mk3(0.0f, 0.0f, 0.0f);
    for (int l = 0; l < n_lobes; l++) {
        const float* q = p + stride * l;
        float* o = gp + stride * l;
        const float t0 = tanhf(q[0]), t1 = tanhf(q[1]), t2 = tanhf(q[2]);
        const Lobe L = make_lobe(clampf(t0, -kLobeCosLimit, kLobeCosLimit), clampf(t1, -kLobeCosLimit, kLobeCosLimit),
                                 clampf(t2, -kLobeCosLimit, kLobeCosLimit));
        const float lam_raw = expf(q[3]), a_raw = expf(q[4]);
        const float lam = fminf(lam_raw, kLobeShapeLimit), a = fminf(a_raw, kLobeShapeLimit);
        const f3 w = residual_act3(res_act, mk3(q[wofs], q[wofs + 1], q[wofs + 2]));
        const float vz = dot3(d, L.z), vx = dot3(d, L.x);
        const float vzc = clampf(vz, -kLobePoleLimit, kLobePoleLimit);
        const float K = 0.5f * (vzc + 1.0f);
        const float om = 1.0f - vzc * vzc;
        const float Ke = kLobeEps + a * vx * vx / om;
        const float E = powf(K, Ke);
        const float e2l = expf(-2.0f * lam);
        const float D = kTwoPi * (1.0f + kLobeEpsNorm - e2l);
        const float sq = sqrtf(1.0f + a);
        const float Nn = lam * sq / D;
        const float P = expf(2.0f * lam * (E * K - 1.0f));
        const float lnK = logf(K);
        float G = 1.0f, kf = 0.0f, tk = 0.0f, sinkx = 0.0f;
        if (kGabor) {
            tk = tanhf(q[5]);
            kf = (tk + 1.0f) * kGaborScale;
            G = 0.5f * (1.0f + cosf(kf * vx));
            sinkx = sinf(kf * vx);
        }
        const bool inside = fabsf(vz) < kLobePoleLimit;
        const float pdf = vz >= kLobePoleLimit ? 1.0f : (inside ? P * E * G * Nn : 0.0f);
        o[wofs] = g.x * pdf * residual_act_grad_from_y(res_act, w.x);
        o[wofs + 1] = g.y * pdf * residual_act_grad_from_y(res_act, w.y);
        o[wofs + 2] = g.z * pdf * residual_act_grad_from_y(res_act, w.z);
        const float gpdf = inside ? dot3(g, w) : 0.0f;
        // sharpness: through P and the normalisation
        const float dP_dlam = P * 2.0f * (E * K - 1.0f);
        const float dN_dlam = (sq * D - lam * sq * 2.0f * kTwoPi * e2l) / (D * D);
        o[3] = lam_raw >= kLobeShapeLimit ? 0.0f : gpdf * (dP_dlam * E * G * Nn + P * E * G * dN_dlam) * lam;
        // anisotropy: through K_e (E and P) and the normalisation
        const float dE_da = E * lnK * (vx * vx / om);
        const float dP_da = P * 2.0f * lam * K * dE_da;
        const float dN_da = (lam / (2.0f * sq)) / D;
        o[4] = a_raw >= kLobeShapeLimit ? 0.0f : gpdf * (dP_da * E * G * Nn + P * dE_da * G * Nn + P * E * G * dN_da) * a;
        if (kGabor) o[5] = gpdf * (P * E * (-0.5f * sinkx * vx) * Nn) * kGaborScale * (1.0f - tk * tk);
        // projections v_x = <d, x>, v_z = <d, z>
        const float dE_dvx = E * lnK * (2.0f * a * vx / om);
        const float dP_dvx = P * 2.0f * lam * K * dE_dvx;
        const float dG_dvx = kGabor ? -0.5f * sinkx * kf : 0.0f;
        const float g_vx = gpdf * (dP_dvx * E * G * Nn + P * dE_dvx * G * Nn + P * E * dG_dvx * Nn);
        const float dKe_dvz = a * vx * vx * 2.0f * vz / (om * om);
        const float dE_dvz = E * (Ke / K) * 0.5f + E * lnK * dKe_dvz;
        const float dP_dvz = P * 2.0f * lam * (K * dE_dvz + E * 0.5f);
        const float g_vz = gpdf * (dP_dvz * E * G * Nn + P * dE_dvz * G * Nn);
        gd = gd + g_vx * L.x + g_vz * L.z;
        // frame cosines through the frame construction, then tanh
        const f3 gx = g_vx * d, gz = g_vz * d;
        const float ds_t = -L.ct / L.st, ds_p = -L.cp / L.sp, ds_u = -L.cu / L.su;
        const float g_ct = gx.x * (L.cp * L.cu - ds_t * L.su) + gx.y * (ds_t * L.cp * L.cu + L.su) + gz.x * L.sp + gz.y * ds_t * L.sp;
        const float g_cp = gx.x * L.ct * L.cu + gx.y * L.st * L.cu - gx.z * ds_p * L.cu + gz.x * L.ct * ds_p + gz.y * L.st * ds_p + gz.z;
        const float g_cu = gx.x * (L.ct * L.cp - L.st * ds_u) + gx.y * (L.st * L.cp + L.ct * ds_u) - gx.z * L.sp;
        o[0] = fabsf(t0) >= kLobeCosLimit ? 0.0f : g_ct * (1.0f - t0 * t0);
        o[1] = fabsf(t1) >= kLobeCosLimit ? 0.0f : g_cp * (1.0f - t1 * t1);
        o[2] = fabsf(t2) >= kLobeCosLimit ? 0.0f : g_cu * (1.0f - t2 * t2);
    }
    return gd;
}

constexpr int kMaxResidualStride = 90;  // 10 NASGabor lobes

// number of raw residual floats per Gaussian and of those active at the given degree
__host__ __device__ inline int residual_stride(int model, int max_degree, int feature_dim) {
    switch (model) {
        case kSH: return 3 * ((max_degree + 1) * (max_degree + 1) - 1);
        case kSV: return 7 * max_degree;
        case kNASG: return 8 * max_degree;
        case kNASGabor: return 9 * max_degree;
        case kNeural: return feature_dim;
        default: return 0;
    }
}
__host__ __device__ inline int residual_active(int model, int degree, int feature_dim) {
    switch (model) {
        case kSH: return degree > 0 ? 3 * ((degree + 1) * (degree + 1) - 1) : 0;
        case kSV: return 7 * degree;
        case kNASG: return 8 * degree;
        case kNASGabor: return 9 * degree;
        case kNeural: return degree > 0 ? feature_dim : 0;
        default: return 0;
    }
}

}  // namespace fgs
