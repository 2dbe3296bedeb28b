/* Neural residual of the oracle (included by fgs_oracle.c).
 *
 * Semantics restated from FasterGSVDACudaBackend/.../rasterization/rtc/appearance_neural.cuh:10-407 and
 * Appearance/Neural.py:40-111 / Appearance/utils.py:254-348. The MLP itself is tiny-cuda-nn's FullyFusedMLP,
 * whose sources are absent from the reference checkout (submodule not populated, version unpinned); its
 * published behaviour is restated: Identity encoding with inputs padded to a multiple of 16 (padding value 1),
 * fp16 weights and activations with fp32 accumulation, hidden layers with ReLU (or none), a linear output layer
 * padded to 16 rows, no biases. Weight layout of the flat parameter vector: input layer [n_neurons, n_input_pad],
 * (n_hidden - 1) hidden layers [n_neurons, n_neurons], output layer [16, n_neurons], each row-major.
 * In the float build every layer input and output is rounded to fp16 (matching the kernels); the double build
 * keeps full precision so that finite differences are meaningful. */

#ifndef ORC_DOUBLE
static inline real h16(real x) { return (real)(_Float16)x; }

/* One fp32-accumulating tensor-core instruction over n <= 16 products of fp16 operands, as the B200 tensor cores
 * evaluate it (tcgen05.mma kind::f16 and mma.sync m16n8k16 with an fp32 accumulator give identical results). The
 * rule was measured on the hardware with random operands (exact on every output, fp16 subnormals included): every
 * nonzero product a*b is aligned to E = max over the products of (exponent(a) + exponent(b)) and over the incoming
 * accumulator of its exponent, where exponent(x) = floor(log2|x|) and an fp16 subnormal counts as -14; each product
 * and the accumulator are truncated toward zero to a multiple of 2^(E - 25); the truncated values are added exactly
 * and the sum is rounded toward zero to fp32. */
static inline int h16_exponent(float x) { const int e = ilogbf(x); return e < -14 ? -14 : e; }
static float tc_accumulate(float acc, const float* a, const float* b, int n) {
    int emax = -100000;
    for (int k = 0; k < n; k++)
        if (a[k] != 0.0f && b[k] != 0.0f) {
            const int e = h16_exponent(a[k]) + h16_exponent(b[k]);
            if (e > emax) emax = e;
        }
    if (acc != 0.0f) {
        const int e = ilogbf(acc);
        if (e > emax) emax = e;
    }
    if (emax == -100000) return 0.0f;
    int64_t sum = (int64_t)trunc(ldexp((double)acc, 25 - emax));
    for (int k = 0; k < n; k++) sum += (int64_t)trunc(ldexp((double)a[k] * (double)b[k], 25 - emax));
    const double v = ldexp((double)sum, emax - 25);
    float f = (float)v;
    if (fabs((double)f) > fabs(v)) f = nextafterf(f, 0.0f);
    return f;
}

/* dot product of n (a multiple of 16) fp16 pairs, 16 at a time in ascending order, as the MLP kernels issue it */
static float tc_dot(const float* a, const float* b, int n) {
    float acc = 0.0f;
    for (int k0 = 0; k0 < n; k0 += 16) acc = tc_accumulate(acc, a + k0, b + k0, 16);
    return acc;
}
#else
static inline real h16(real x) { return x; }
#endif

static int64_t neural_param_count(const orc_appearance* A) {
    return (int64_t)A->n_neurons * A->n_input_pad + (int64_t)(A->n_hidden - 1) * A->n_neurons * A->n_neurons + 16LL * A->n_neurons;
}

static const double SH_C0 = 0.28209479177387814;

/* SH values of the configured bands (ascending), band 0 never gated, the i-th band >= 1 zeroed unless i < deg */
static int sh_degree_values(const orc_appearance* A, double x, double y, double z, int deg, double* out) {
    const double xy = x * y, xz = x * z, yz = y * z, x2 = x * x, y2 = y * y, z2 = z * z;
    const double x4 = x2 * x2, y4 = y2 * y2, z4 = z2 * z2, x6 = x4 * x2, y6 = y4 * y2, z6 = z4 * z2;
    int o = 0, rank = 0;
    if (A->sh_mask & 1) out[o++] = SH_C0;
    for (int l = 1; l <= 6; l++) {
        if (!(A->sh_mask & (1 << l))) continue;
        const double m = rank++ < deg ? 1.0 : 0.0;
        double v[13];
        int n = 0;
        switch (l) {
            case 1: v[0] = -0.48860251190291987 * y; v[1] = 0.48860251190291987 * z; v[2] = -0.48860251190291987 * x; n = 3; break;
            case 2:
                v[0] = 1.0925484305920792 * xy; v[1] = -1.0925484305920792 * yz; v[2] = 0.94617469575755997 * z2 - 0.31539156525251999;
                v[3] = -1.0925484305920792 * xz; v[4] = 0.54627421529603959 * x2 - 0.54627421529603959 * y2; n = 5; break;
            case 3:
                v[0] = 0.59004358992664352 * y * (-3.0 * x2 + y2); v[1] = 2.8906114426405538 * xy * z;
                v[2] = 0.45704579946446572 * y * (1.0 - 5.0 * z2); v[3] = 0.3731763325901154 * z * (5.0 * z2 - 3.0);
                v[4] = 0.45704579946446572 * x * (1.0 - 5.0 * z2); v[5] = 1.4453057213202769 * z * (x2 - y2);
                v[6] = 0.59004358992664352 * x * (-x2 + 3.0 * y2); n = 7; break;
            case 4:
                v[0] = 2.5033429417967046 * xy * (x2 - y2); v[1] = 1.7701307697799304 * yz * (-3.0 * x2 + y2);
                v[2] = 0.94617469575756008 * xy * (7.0 * z2 - 1.0); v[3] = 0.66904654355728921 * yz * (3.0 - 7.0 * z2);
                v[4] = -3.1735664074561294 * z2 + 3.7024941420321507 * z4 + 0.31735664074561293;
                v[5] = 0.66904654355728921 * xz * (3.0 - 7.0 * z2); v[6] = 0.47308734787878004 * (x2 - y2) * (7.0 * z2 - 1.0);
                v[7] = 1.7701307697799304 * xz * (-x2 + 3.0 * y2);
                v[8] = -3.7550144126950569 * x2 * y2 + 0.62583573544917614 * x4 + 0.62583573544917614 * y4; n = 9; break;
            case 5:
                v[0] = 0.65638205684017015 * y * (10.0 * x2 * y2 - 5.0 * x4 - y4); v[1] = 8.3026492595241645 * xy * z * (x2 - y2);
                v[2] = -0.48923829943525038 * y * (3.0 * x2 - y2) * (9.0 * z2 - 1.0); v[3] = 4.7935367849733241 * xy * z * (3.0 * z2 - 1.0);
                v[4] = 0.45294665119569694 * y * (14.0 * z2 - 21.0 * z4 - 1.0); v[5] = 0.1169503224534236 * z * (-70.0 * z2 + 63.0 * z4 + 15.0);
                v[6] = 0.45294665119569694 * x * (14.0 * z2 - 21.0 * z4 - 1.0); v[7] = 2.3967683924866621 * z * (x2 - y2) * (3.0 * z2 - 1.0);
                v[8] = -0.48923829943525038 * x * (x2 - 3.0 * y2) * (9.0 * z2 - 1.0); v[9] = 2.0756623148810411 * z * (-6.0 * x2 * y2 + x4 + y4);
                v[10] = 0.65638205684017015 * x * (10.0 * x2 * y2 - x4 - 5.0 * y4); n = 11; break;
            default:
                v[0] = 1.3663682103838286 * xy * (-10.0 * x2 * y2 + 3.0 * x4 + 3.0 * y4);
                v[1] = 2.3666191622317521 * yz * (10.0 * x2 * y2 - 5.0 * x4 - y4);
                v[2] = 2.0182596029148963 * xy * (x2 - y2) * (11.0 * z2 - 1.0);
                v[3] = -0.92120525951492349 * yz * (3.0 * x2 - y2) * (11.0 * z2 - 3.0);
                v[4] = 0.92120525951492349 * xy * (-18.0 * z2 + 33.0 * z4 + 1.0);
                v[5] = 0.58262136251873131 * yz * (30.0 * z2 - 33.0 * z4 - 5.0);
                v[6] = 6.6747662381009842 * z2 - 20.024298714302954 * z4 + 14.684485723822165 * z6 - 0.31784601133814211;
                v[7] = 0.58262136251873131 * xz * (30.0 * z2 - 33.0 * z4 - 5.0);
                v[8] = 0.46060262975746175 * (x2 - y2) * (11.0 * z2 * (3.0 * z2 - 1.0) - 7.0 * z2 + 1.0);
                v[9] = -0.92120525951492349 * xz * (x2 - 3.0 * y2) * (11.0 * z2 - 3.0);
                v[10] = 0.50456490072872406 * (11.0 * z2 - 1.0) * (-6.0 * x2 * y2 + x4 + y4);
                v[11] = 2.3666191622317521 * xz * (10.0 * x2 * y2 - x4 - 5.0 * y4);
                v[12] = 10.247761577878714 * x2 * y4 - 10.247761577878714 * x4 * y2 + 0.6831841051919143 * x6 - 0.6831841051919143 * y6;
                n = 13; break;
        }
        for (int k = 0; k < n; k++) out[o++] = m * v[k];
    }
    return o;
}

#ifndef ORC_DOUBLE
/* SH inputs of bands 0..3 in float, every product and sum rounded as written (the kernels evaluate the same
 * operations in the same order, neural_common.cuh sh_band_values); returns the number written */
static int sh_band_values_f(int mask, int deg, float x, float y, float z, double* out) {
    const float c1 = 0.48860251190291987f, c2a = 1.0925484305920792f, c2b = 0.94617469575755997f, c2c = 0.31539156525251999f;
    const float c2d = 0.54627421529603959f, c3a = 0.59004358992664352f, c3b = 2.8906114426405538f, c3c = 0.45704579946446572f;
    const float c3d = 0.3731763325901154f, c3e = 1.4453057213202769f;
    const float xx = x * x, yy = y * y, zz = z * z, xy = x * y, xz = x * z, yz = y * z;
    int o = 0, rank = 0;
    if (mask & 1) out[o++] = 0.28209479177387814f;
    if (mask & 2) {
        const float m = rank++ < deg ? 1.0f : 0.0f;
        out[o++] = m * (-c1 * y);
        out[o++] = m * (c1 * z);
        out[o++] = m * (-c1 * x);
    }
    if (mask & 4) {
        const float m = rank++ < deg ? 1.0f : 0.0f;
        out[o++] = m * (c2a * xy);
        out[o++] = m * (-c2a * yz);
        out[o++] = m * (c2b * zz - c2c);
        out[o++] = m * (-c2a * xz);
        out[o++] = m * (c2d * xx - c2d * yy);
    }
    if (mask & 8) {
        const float m = rank++ < deg ? 1.0f : 0.0f;
        out[o++] = m * ((c3a * y) * (-3.0f * xx + yy));
        out[o++] = m * ((c3b * xy) * z);
        out[o++] = m * ((c3c * y) * (1.0f - 5.0f * zz));
        out[o++] = m * ((c3d * z) * (5.0f * zz - 3.0f));
        out[o++] = m * ((c3c * x) * (1.0f - 5.0f * zz));
        out[o++] = m * ((c3e * z) * (xx - yy));
        out[o++] = m * ((c3a * x) * (-xx + 3.0f * yy));
    }
    return o;
}
#endif

/* builds the encoder input vector (before padding); returns its length */
static int neural_inputs(const orc_appearance* A, const inreal* feat, const inreal* base, double dx, double dy, double dz, int deg, double* x) {
    const int nraw = A->feature_dim + (A->base_input ? 3 : 0);
    int o = 0;
    for (int i = 0; i < nraw; i++) {
        const double val = i < A->feature_dim ? feat[i] : base[i - A->feature_dim];
        if (A->n_freq == 0) { x[o++] = val; continue; }
        for (int f = 0; f < A->n_freq; f++) {
            const double s = ldexp(val, f);
#ifndef ORC_DOUBLE
            float sn, cs;
            det_sincos_f((float)s, &sn, &cs);
            x[o++] = sn;
            x[o++] = cs;
#else
            x[o++] = sin(s);
            x[o++] = cos(s);
#endif
        }
    }
#ifndef ORC_DOUBLE
    if (A->sh_mask <= 15) {
        o += sh_band_values_f(A->sh_mask, deg, (float)dx, (float)dy, (float)dz, x + o);
        return o;
    }
#endif
    o += sh_degree_values(A, dx, dy, dz, deg, x + o);
    return o;
}

/* forward through the MLP; acts[l] holds the (rounded) input of layer l, out receives 16 outputs */
static void neural_mlp(const orc_appearance* A, const inreal* W, const double* x0, double* acts, double* out) {
    const int nin = A->n_input_pad, nn = A->n_neurons, L = A->n_hidden + 1;
    double* cur = acts;
    for (int i = 0; i < nin; i++) cur[i] = h16((real)x0[i]);
    int cur_w = nin;
    size_t off = 0;
    for (int l = 0; l < L; l++) {
        const int out_w = l == L - 1 ? 16 : nn;
        double* nxt = l == L - 1 ? out : acts + (size_t)nin + (size_t)l * nn;
        for (int o = 0; o < out_w; o++) {
#ifndef ORC_DOUBLE
            float av[128], bv[128];
            for (int k = 0; k < cur_w; k++) {
                av[k] = (float)cur[k];
                bv[k] = h16(W[off + (size_t)o * cur_w + k]);
            }
            double val = tc_dot(av, bv, cur_w);
#else
            real acc = 0;
            for (int k = 0; k < cur_w; k++) acc += (real)(h16(W[off + (size_t)o * cur_w + k]) * (real)cur[k]);
            double val = acc;
#endif
            if (l < L - 1 && A->hidden_act == 1 && val < 0.0) val = 0.0;
            nxt[o] = h16((real)val);
        }
        off += (size_t)out_w * cur_w;
        cur = nxt;
        cur_w = out_w;
    }
}

static v3_r neural_forward_r(const orc_appearance* A, const inreal* feat, const inreal* base, v3_r d, int deg, const inreal* W) {
    if (deg <= 0) return mk_r(R(0.0), R(0.0), R(0.0));
    double x[160];
    const int n = neural_inputs(A, feat, base, d.x, d.y, d.z, deg, x);
    for (int i = n; i < A->n_input_pad; i++) x[i] = 1.0;
    double acts[128 + 8 * 128];
    double out[16];
    neural_mlp(A, W, x, acts, out);
    return mk_r(residual_act_r(A->res_act, (real)out[0]), residual_act_r(A->res_act, (real)out[1]), residual_act_r(A->res_act, (real)out[2]));
}

/* backward in double; g = gradient w.r.t. the residual. Writes the feature gradients into gfeat, accumulates the
 * weight gradients into gW (may be NULL), adds base gradients (base_input) into gbase, and returns the gradient
 * w.r.t. the unit direction. */
static v3_d neural_backward_d(const orc_appearance* A, const inreal* feat, const inreal* base, v3_d g, v3_d d, v3_r d_in, int deg,
                              const inreal* W, double* gfeat, double* gW, double* gbase) {
    if (deg <= 0) return mk_d(0.0, 0.0, 0.0);
    double x[160];
    /* the network's inputs from the direction the forward used (working precision), so the recomputed activations are
     * the forward's */
    const int n = neural_inputs(A, feat, base, d_in.x, d_in.y, d_in.z, deg, x);
    for (int i = n; i < A->n_input_pad; i++) x[i] = 1.0;
    const int nin = A->n_input_pad, nn = A->n_neurons, L = A->n_hidden + 1;
    double acts[128 + 8 * 128];
    double out[16];
    neural_mlp(A, W, x, acts, out);
    /* dL/dy through the residual activation (recovered from the rounded output) */
    double gy[16] = {0};
    const double gv[3] = {g.x, g.y, g.z};
    for (int c = 0; c < 3; c++) gy[c] = gv[c] * residual_act_grad_d(A->res_act, residual_act_d(A->res_act, out[c]));
    /* walk the layers backwards */
    size_t offs[10];
    int win[10], wout[10];
    size_t off = 0;
    for (int l = 0; l < L; l++) {
        win[l] = l == 0 ? nin : nn;
        wout[l] = l == L - 1 ? 16 : nn;
        offs[l] = off;
        off += (size_t)win[l] * wout[l];
    }
    double gcur[128];
    double gin[128];
#ifndef ORC_DOUBLE
    /* fp16 semantics of the network's backward (tiny-cuda-nn's __half network, appearance_neural.cuh:370-380, with the
     * loss scale of rasterization_config.h:17): the output gradient is scaled by 128 and rounded to fp16, every layer's
     * data gradient accumulates fp16 products on the tensor cores (tc_dot, 16 rows of the layer at a time), hidden
     * gradients are masked by the ReLU of the stored activation and rounded to fp16, the input gradient stays fp32;
     * weight gradients are sums of products of the fp16 gradients and activations; everything is unscaled at the end */
    const double inv_scale = 1.0 / 128.0;
    for (int o = 0; o < 16; o++) gcur[o] = h16(128.0f * (float)gy[o]);
    for (int l = L - 1; l >= 0; l--) {
        const double* inp = l == 0 ? acts : acts + (size_t)nin + (size_t)(l - 1) * nn;
        float gv16[128];
        for (int o = 0; o < wout[l]; o++) gv16[o] = (float)gcur[o];
        for (int k = 0; k < win[l]; k++) {
            float wcol[128];
            for (int o = 0; o < wout[l]; o++) wcol[o] = h16(W[offs[l] + (size_t)o * win[l] + k]);
            gin[k] = tc_dot(gv16, wcol, wout[l]);
        }
        if (gW)
            for (int o = 0; o < wout[l]; o++)
                for (int k = 0; k < win[l]; k++) gW[offs[l] + (size_t)o * win[l] + k] += gcur[o] * inp[k] * inv_scale;
        if (l > 0)
            for (int k = 0; k < win[l]; k++) gcur[k] = (A->hidden_act == 1 && !(inp[k] > 0.0)) ? 0.0 : h16((float)gin[k]);
    }
    for (int k = 0; k < nin; k++) gin[k] *= inv_scale;
#else
    for (int o = 0; o < 16; o++) gcur[o] = gy[o];
    for (int l = L - 1; l >= 0; l--) {
        const double* inp = l == 0 ? acts : acts + (size_t)nin + (size_t)(l - 1) * nn;
        for (int k = 0; k < win[l]; k++) {
            double s = 0.0;
            for (int o = 0; o < wout[l]; o++) s += (double)(float)h16(W[offs[l] + (size_t)o * win[l] + k]) * gcur[o];
            gin[k] = s;
        }
        if (gW)
            for (int o = 0; o < wout[l]; o++)
                for (int k = 0; k < win[l]; k++) gW[offs[l] + (size_t)o * win[l] + k] += gcur[o] * inp[k];
        if (l > 0) {
            /* hidden activation derivative from the layer input (which is the previous layer's output) */
            for (int k = 0; k < win[l]; k++) gcur[k] = (A->hidden_act == 1 && inp[k] <= 0.0) ? 0.0 : gin[k];
        }
    }
#endif
    /* gin = dL/dx (encoder output); features through the frequency encoding */
    const int nraw = A->feature_dim + (A->base_input ? 3 : 0);
    const int per = A->n_freq == 0 ? 1 : 2 * A->n_freq;
    for (int i = 0; i < nraw; i++) {
        const double val = i < A->feature_dim ? feat[i] : base[i - A->feature_dim];
        double gval = 0.0;
        if (A->n_freq == 0) gval = gin[i];
        else
            for (int f = 0; f < A->n_freq; f++) {
                const double s = ldexp(val, f);
                gval += ldexp(1.0, f) * (cos(s) * gin[i * per + 2 * f] - sin(s) * gin[i * per + 2 * f + 1]);
            }
        if (i < A->feature_dim) gfeat[i] = gval;
        else gbase[i - A->feature_dim] += gval;
    }
    /* direction through the SH values: central differences of the band polynomials (degree <= 6, step 1e-6, so the
     * truncation error is O(1e-12) relative) */
    const int sh0 = nraw * per;
    double gd[3] = {0.0, 0.0, 0.0};
    const double h = 1e-6;
    for (int c = 0; c < 3; c++) {
        double dp[3] = {d.x, d.y, d.z}, dm[3] = {d.x, d.y, d.z};
        dp[c] += h;
        dm[c] -= h;
        double vp[64], vm[64];
        const int m = sh_degree_values(A, dp[0], dp[1], dp[2], deg, vp);
        sh_degree_values(A, dm[0], dm[1], dm[2], deg, vm);
        double s = 0.0;
        for (int k = 0; k < m; k++) s += gin[sh0 + k] * (vp[k] - vm[k]) / (2.0 * h);
        gd[c] = s;
    }
    return mk_d(gd[0], gd[1], gd[2]);
}
