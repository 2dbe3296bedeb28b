/* Appearance residual models of the oracle, instantiated twice by fgs_oracle.c: once in the working
 * precision `real` (forward colors, same operation order as the GPU kernels) and once in double
 * (backward). Expected macros: T (scalar type), SFX (name suffix), K(x) (literal of type T).
 * Follows FasterGSVDACudaBackend/.../rasterization/rtc/appearance_sh.cuh:30-157, appearance_sv.cuh:26-139,
 * appearance_nasg.cuh:39-209, appearance_nasgabor.cuh:53-223 and rtc/preprocess_common.cuh:51-142. */

#define FN2(a, b) a##b
#define FN1(a, b) FN2(a, b)
#define FN(name) FN1(name, SFX)

typedef struct { T x, y, z; } FN(v3);

static inline FN(v3) FN(mk)(T x, T y, T z) { FN(v3) r = {x, y, z}; return r; }
static inline FN(v3) FN(add)(FN(v3) a, FN(v3) b) { return FN(mk)(a.x + b.x, a.y + b.y, a.z + b.z); }
static inline FN(v3) FN(sub)(FN(v3) a, FN(v3) b) { return FN(mk)(a.x - b.x, a.y - b.y, a.z - b.z); }
static inline FN(v3) FN(scl)(T s, FN(v3) a) { return FN(mk)(s * a.x, s * a.y, s * a.z); }
static inline FN(v3) FN(mul)(FN(v3) a, FN(v3) b) { return FN(mk)(a.x * b.x, a.y * b.y, a.z * b.z); }
static inline T FN(dot)(FN(v3) a, FN(v3) b) { return a.x * b.x + a.y * b.y + a.z * b.z; }
static inline T FN(clampv)(T x, T lo, T hi) { return fmin(fmax(x, lo), hi); }

static inline T FN(softplus10)(T x) { return (fmax(K(10.0) * x, K(0.0)) + log1p(exp(-fabs(K(10.0) * x)))) / K(10.0); }
static inline T FN(softplus10_grad)(T y) { return -expm1(-K(10.0) * y); }
static inline T FN(residual_act)(int id, T x) { return id == 1 ? tanh(x) : (id == 2 ? FN(softplus10)(x) : x); }
static inline T FN(residual_act_grad)(int id, T y) { return id == 1 ? K(1.0) - y * y : (id == 2 ? FN(softplus10_grad)(y) : K(1.0)); }
static inline FN(v3) FN(residual_act3)(int id, FN(v3) v) { return FN(mk)(FN(residual_act)(id, v.x), FN(residual_act)(id, v.y), FN(residual_act)(id, v.z)); }

/* ---- spherical harmonics, bands 1..degree ---- */
static int FN(sh_basis)(FN(v3) d, int degree, T* Y) {
    const T x = d.x, y = d.y, z = d.z;
    Y[0] = -K(0.48860251190291987) * y;
    Y[1] = K(0.48860251190291987) * z;
    Y[2] = -K(0.48860251190291987) * x;
    if (degree < 2) return 3;
    const T xx = x * x, yy = y * y, zz = z * z, xy = x * y, xz = x * z, yz = y * z;
    Y[3] = K(1.0925484305920792) * xy;
    Y[4] = -K(1.0925484305920792) * yz;
    Y[5] = K(0.94617469575755997) * zz - K(0.31539156525251999);
    Y[6] = -K(1.0925484305920792) * xz;
    Y[7] = K(0.54627421529603959) * (xx - yy);
    if (degree < 3) return 8;
    Y[8] = y * (K(0.59004358992664352) * yy - K(1.7701307697799304) * xx);
    Y[9] = K(2.8906114426405538) * xy * z;
    Y[10] = y * (K(0.45704579946446572) - K(2.2852289973223288) * zz);
    Y[11] = z * (K(1.865881662950577) * zz - K(1.1195289977703462));
    Y[12] = x * (K(0.45704579946446572) - K(2.2852289973223288) * zz);
    Y[13] = K(1.4453057213202769) * z * (xx - yy);
    Y[14] = x * (K(1.7701307697799304) * yy - K(0.59004358992664352) * xx);
    return 15;
}

static void FN(sh_basis_grad)(FN(v3) d, int degree, FN(v3)* dY) {
    const T x = d.x, y = d.y, z = d.z;
    const T c1 = K(0.48860251190291987), c2a = K(1.0925484305920792), c2b = K(0.94617469575755997), c2d = K(0.54627421529603959);
    const T c3a = K(0.59004358992664352), c3b = K(1.7701307697799304), c3c = K(2.8906114426405538), c3d = K(0.45704579946446572);
    const T c3e = K(2.2852289973223288), c3f = K(1.865881662950577), c3g = K(1.1195289977703462), c3h = K(1.4453057213202769);
    dY[0] = FN(mk)(K(0.0), -c1, K(0.0));
    dY[1] = FN(mk)(K(0.0), K(0.0), c1);
    dY[2] = FN(mk)(-c1, K(0.0), K(0.0));
    if (degree < 2) return;
    const T xx = x * x, yy = y * y, zz = z * z;
    dY[3] = FN(mk)(c2a * y, c2a * x, K(0.0));
    dY[4] = FN(mk)(K(0.0), -c2a * z, -c2a * y);
    dY[5] = FN(mk)(K(0.0), K(0.0), K(2.0) * c2b * z);
    dY[6] = FN(mk)(-c2a * z, K(0.0), -c2a * x);
    dY[7] = FN(mk)(K(2.0) * c2d * x, -K(2.0) * c2d * y, K(0.0));
    if (degree < 3) return;
    dY[8] = FN(mk)(-K(2.0) * c3b * x * y, K(3.0) * c3a * yy - c3b * xx, K(0.0));
    dY[9] = FN(mk)(c3c * y * z, c3c * x * z, c3c * x * y);
    dY[10] = FN(mk)(K(0.0), c3d - c3e * zz, -K(2.0) * c3e * y * z);
    dY[11] = FN(mk)(K(0.0), K(0.0), K(3.0) * c3f * zz - c3g);
    dY[12] = FN(mk)(c3d - c3e * zz, K(0.0), -K(2.0) * c3e * x * z);
    dY[13] = FN(mk)(K(2.0) * c3h * x * z, -K(2.0) * c3h * y * z, c3h * (xx - yy));
    dY[14] = FN(mk)(c3b * yy - K(3.0) * c3a * xx, K(2.0) * c3b * x * y, K(0.0));
}

static FN(v3) FN(sh_forward)(const inreal* c, FN(v3) d, int degree, int act) {
    if (degree <= 0) return FN(mk)(K(0.0), K(0.0), K(0.0));
    T Y[15];
    const int n = FN(sh_basis)(d, degree, Y);
    FN(v3) s = FN(mk)(K(0.0), K(0.0), K(0.0));
    for (int k = 0; k < n; k++) s = FN(add)(s, FN(scl)(Y[k], FN(mk)(c[3 * k], c[3 * k + 1], c[3 * k + 2])));
    return FN(residual_act3)(act, s);
}

static FN(v3) FN(sh_backward)(const inreal* c, FN(v3) g, FN(v3) d, int degree, int act, T* gc) {
    if (degree <= 0) return FN(mk)(K(0.0), K(0.0), K(0.0));
    T Y[15];
    FN(v3) dY[15];
    const int n = FN(sh_basis)(d, degree, Y);
    FN(sh_basis_grad)(d, degree, dY);
    FN(v3) s = FN(mk)(K(0.0), K(0.0), K(0.0));
    for (int k = 0; k < n; k++) s = FN(add)(s, FN(scl)(Y[k], FN(mk)(c[3 * k], c[3 * k + 1], c[3 * k + 2])));
    const FN(v3) r = FN(residual_act3)(act, s);
    const FN(v3) gs = FN(mul)(g, FN(mk)(FN(residual_act_grad)(act, r.x), FN(residual_act_grad)(act, r.y), FN(residual_act_grad)(act, r.z)));
    FN(v3) gd = FN(mk)(K(0.0), K(0.0), K(0.0));
    for (int k = 0; k < n; k++) {
        gc[3 * k] = Y[k] * gs.x;
        gc[3 * k + 1] = Y[k] * gs.y;
        gc[3 * k + 2] = Y[k] * gs.z;
        gd = FN(add)(gd, FN(scl)(FN(dot)(FN(mk)(c[3 * k], c[3 * k + 1], c[3 * k + 2]), gs), dY[k]));
    }
    return gd;
}

/* ---- soft spherical Voronoi (7 values per site: xyz, log tau, rgb) ---- */
static FN(v3) FN(sv_eval)(const inreal* p, FN(v3) d, int n, int act, T* max_out, T* wsum_out, FN(v3)* acc_out) {
    T mx = K(-3.0e38);
    for (int k = 0; k < n; k++) {
        const inreal* s = p + 7 * k;
        const FN(v3) raw = FN(mk)(s[0], s[1], s[2]);
        const FN(v3) site = FN(scl)(K(1.0) / fmax(sqrt(FN(dot)(raw, raw)), K(1e-12)), raw);
        const FN(v3) df = FN(sub)(site, d);
        const T logit = -exp((T)s[3]) * sqrt(FN(dot)(df, df));
        mx = fmax(mx, logit);
    }
    T ws = K(0.0);
    FN(v3) acc = FN(mk)(K(0.0), K(0.0), K(0.0));
    for (int k = 0; k < n; k++) {
        const inreal* s = p + 7 * k;
        const FN(v3) raw = FN(mk)(s[0], s[1], s[2]);
        const FN(v3) site = FN(scl)(K(1.0) / fmax(sqrt(FN(dot)(raw, raw)), K(1e-12)), raw);
        const FN(v3) df = FN(sub)(site, d);
        const T w = exp(-exp((T)s[3]) * sqrt(FN(dot)(df, df)) - mx);
        ws += w;
        acc = FN(add)(acc, FN(scl)(w, FN(residual_act3)(act, FN(mk)(s[4], s[5], s[6]))));
    }
    if (max_out) *max_out = mx;
    if (wsum_out) *wsum_out = ws;
    if (acc_out) *acc_out = acc;
    return FN(scl)(K(1.0) / ws, acc);
}

static FN(v3) FN(sv_forward)(const inreal* p, FN(v3) d, int n, int act) {
    if (n <= 0) return FN(mk)(K(0.0), K(0.0), K(0.0));
    return FN(sv_eval)(p, d, n, act, 0, 0, 0);
}

static FN(v3) FN(sv_backward)(const inreal* p, FN(v3) g, FN(v3) d, int n, int act, T* gp) {
    if (n <= 0) return FN(mk)(K(0.0), K(0.0), K(0.0));
    T mx, ws;
    FN(v3) acc;
    FN(sv_eval)(p, d, n, act, &mx, &ws, &acc);
    const T inv = K(1.0) / ws;
    const T gmean = FN(dot)(g, FN(scl)(inv, acc));
    FN(v3) gd = FN(mk)(K(0.0), K(0.0), K(0.0));
    for (int k = 0; k < n; k++) {
        const inreal* s = p + 7 * k;
        T* o = gp + 7 * k;
        const FN(v3) raw = FN(mk)(s[0], s[1], s[2]);
        const T il = K(1.0) / fmax(sqrt(FN(dot)(raw, raw)), K(1e-12));
        const FN(v3) site = FN(scl)(il, raw);
        const FN(v3) df = FN(sub)(site, d);
        const T dist = sqrt(FN(dot)(df, df));
        const T tau = exp((T)s[3]);
        const T w = exp(-tau * dist - mx) * inv;
        const FN(v3) col = FN(residual_act3)(act, FN(mk)(s[4], s[5], s[6]));
        o[4] = w * g.x * FN(residual_act_grad)(act, col.x);
        o[5] = w * g.y * FN(residual_act_grad)(act, col.y);
        o[6] = w * g.z * FN(residual_act_grad)(act, col.z);
        const T gl = w * (FN(dot)(g, col) - gmean);
        o[3] = -dist * tau * gl;
        const FN(v3) gdf = FN(scl)(-tau * gl / fmax(dist, K(1e-12)), df);
        const FN(v3) gs = FN(scl)(il, FN(sub)(gdf, FN(scl)(FN(dot)(gdf, site), site)));
        o[0] = gs.x; o[1] = gs.y; o[2] = gs.z;
        gd = FN(sub)(gd, gdf);
    }
    return gd;
}

/* ---- NASG / NASGabor lobes ---- */
static FN(v3) FN(lobes_forward)(const inreal* p, FN(v3) d, int n, int act, int gabor) {
    const int stride = gabor ? 9 : 8, wo = gabor ? 6 : 5;
    FN(v3) out = FN(mk)(K(0.0), K(0.0), K(0.0));
    for (int l = 0; l < n; l++) {
        const inreal* q = p + stride * l;
        const T ct = FN(clampv)(tanh((T)q[0]), -K(0.999999), K(0.999999));
        const T cp = FN(clampv)(tanh((T)q[1]), -K(0.999999), K(0.999999));
        const T cu = FN(clampv)(tanh((T)q[2]), -K(0.999999), K(0.999999));
        const T st = sqrt(K(1.0) - ct * ct), sp = sqrt(K(1.0) - cp * cp), su = sqrt(K(1.0) - cu * cu);
        const FN(v3) fx = FN(mk)(ct * cp * cu - st * su, st * cp * cu + ct * su, -sp * cu);
        const FN(v3) fz = FN(mk)(ct * sp, st * sp, cp);
        const T lam = fmin(exp((T)q[3]), K(1e4)), a = fmin(exp((T)q[4]), K(1e4));
        const T vz = FN(dot)(d, fz), vx = FN(dot)(d, fx);
        const T vzc = FN(clampv)(vz, -K(0.99999988), K(0.99999988));
        const T Kk = K(0.5) * (vzc + K(1.0));
        const T Ke = K(5e-6) + a * vx * vx / (K(1.0) - vzc * vzc);
        const T E = pow(Kk, Ke);
        const T N = lam * sqrt(K(1.0) + a) / (K(6.28318530717958647692) * (K(1.0) + K(1e-8) - exp(-K(2.0) * lam)));
        const T P = exp(K(2.0) * lam * (E * Kk - K(1.0)));
        T G = K(1.0);
        if (gabor) G = K(0.5) * (K(1.0) + cos((tanh((T)q[5]) + K(1.0)) * K(20.0) * vx));
        const T pdf = vz >= K(0.99999988) ? K(1.0) : (vz > -K(0.99999988) ? P * E * G * N : K(0.0));
        out = FN(add)(out, FN(scl)(pdf, FN(residual_act3)(act, FN(mk)(q[wo], q[wo + 1], q[wo + 2]))));
    }
    return out;
}

static FN(v3) FN(lobes_backward)(const inreal* p, FN(v3) g, FN(v3) d, int n, int act, int gabor, T* gp) {
    const int stride = gabor ? 9 : 8, wo = gabor ? 6 : 5;
    FN(v3) gd = FN(mk)(K(0.0), K(0.0), K(0.0));
    for (int l = 0; l < n; l++) {
        const inreal* q = p + stride * l;
        T* o = gp + stride * l;
        const T t0 = tanh((T)q[0]), t1 = tanh((T)q[1]), t2 = tanh((T)q[2]);
        const T ct = FN(clampv)(t0, -K(0.999999), K(0.999999)), cp = FN(clampv)(t1, -K(0.999999), K(0.999999));
        const T cu = FN(clampv)(t2, -K(0.999999), K(0.999999));
        const T st = sqrt(K(1.0) - ct * ct), sp = sqrt(K(1.0) - cp * cp), su = sqrt(K(1.0) - cu * cu);
        const FN(v3) fx = FN(mk)(ct * cp * cu - st * su, st * cp * cu + ct * su, -sp * cu);
        const FN(v3) fz = FN(mk)(ct * sp, st * sp, cp);
        const T lr = exp((T)q[3]), ar = exp((T)q[4]);
        const T lam = fmin(lr, K(1e4)), a = fmin(ar, K(1e4));
        const FN(v3) w = FN(residual_act3)(act, FN(mk)(q[wo], q[wo + 1], q[wo + 2]));
        const T vz = FN(dot)(d, fz), vx = FN(dot)(d, fx);
        const T vzc = FN(clampv)(vz, -K(0.99999988), K(0.99999988));
        const T Kk = K(0.5) * (vzc + K(1.0));
        const T om = K(1.0) - vzc * vzc;
        const T Ke = K(5e-6) + a * vx * vx / om;
        const T E = pow(Kk, Ke);
        const T e2l = exp(-K(2.0) * lam);
        const T D = K(6.28318530717958647692) * (K(1.0) + K(1e-8) - e2l);
        const T sq = sqrt(K(1.0) + a);
        const T N = lam * sq / D;
        const T P = exp(K(2.0) * lam * (E * Kk - K(1.0)));
        const T lnK = log(Kk);
        T G = K(1.0), kf = K(0.0), tk = K(0.0), skx = K(0.0);
        if (gabor) {
            tk = tanh((T)q[5]);
            kf = (tk + K(1.0)) * K(20.0);
            G = K(0.5) * (K(1.0) + cos(kf * vx));
            skx = sin(kf * vx);
        }
        const int inside = fabs(vz) < K(0.99999988);
        const T pdf = vz >= K(0.99999988) ? K(1.0) : (inside ? P * E * G * N : K(0.0));
        o[wo] = g.x * pdf * FN(residual_act_grad)(act, w.x);
        o[wo + 1] = g.y * pdf * FN(residual_act_grad)(act, w.y);
        o[wo + 2] = g.z * pdf * FN(residual_act_grad)(act, w.z);
        const T gpdf = inside ? FN(dot)(g, w) : K(0.0);
        const T dP_dl = P * K(2.0) * (E * Kk - K(1.0));
        const T dN_dl = (sq * D - lam * sq * K(2.0) * K(6.28318530717958647692) * e2l) / (D * D);
        o[3] = lr >= K(1e4) ? K(0.0) : gpdf * (dP_dl * E * G * N + P * E * G * dN_dl) * lam;
        const T dE_da = E * lnK * (vx * vx / om);
        const T dP_da = P * K(2.0) * lam * Kk * dE_da;
        const T dN_da = (lam / (K(2.0) * sq)) / D;
        o[4] = ar >= K(1e4) ? K(0.0) : gpdf * (dP_da * E * G * N + P * dE_da * G * N + P * E * G * dN_da) * a;
        if (gabor) o[5] = gpdf * (P * E * (-K(0.5) * skx * vx) * N) * K(20.0) * (K(1.0) - tk * tk);
        const T dE_dvx = E * lnK * (K(2.0) * a * vx / om);
        const T dP_dvx = P * K(2.0) * lam * Kk * dE_dvx;
        const T dG_dvx = gabor ? -K(0.5) * skx * kf : K(0.0);
        const T gvx = gpdf * (dP_dvx * E * G * N + P * dE_dvx * G * N + P * E * dG_dvx * N);
        const T dKe_dvz = a * vx * vx * K(2.0) * vz / (om * om);
        const T dE_dvz = E * (Ke / Kk) * K(0.5) + E * lnK * dKe_dvz;
        const T dP_dvz = P * K(2.0) * lam * (Kk * dE_dvz + E * K(0.5));
        const T gvz = gpdf * (dP_dvz * E * G * N + P * dE_dvz * G * N);
        gd = FN(add)(gd, FN(add)(FN(scl)(gvx, fx), FN(scl)(gvz, fz)));
        const FN(v3) gx = FN(scl)(gvx, d), gz = FN(scl)(gvz, d);
        const T dst = -ct / st, dsp = -cp / sp, dsu = -cu / su;
        const T gct = gx.x * (cp * cu - dst * su) + gx.y * (dst * cp * cu + su) + gz.x * sp + gz.y * dst * sp;
        const T gcp = gx.x * ct * cu + gx.y * st * cu - gx.z * dsp * cu + gz.x * ct * dsp + gz.y * st * dsp + gz.z;
        const T gcu = gx.x * (ct * cp - st * dsu) + gx.y * (st * cp + ct * dsu) - gx.z * sp;
        o[0] = fabs(t0) >= K(0.999999) ? K(0.0) : gct * (K(1.0) - t0 * t0);
        o[1] = fabs(t1) >= K(0.999999) ? K(0.0) : gcp * (K(1.0) - t1 * t1);
        o[2] = fabs(t2) >= K(0.999999) ? K(0.0) : gcu * (K(1.0) - t2 * t2);
    }
    return gd;
}

#undef FN
#undef FN1
#undef FN2
