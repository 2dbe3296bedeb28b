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
            real acc = 0;
            for (int k = 0; k < cur_w; k++) acc += (real)(h16(W[off + (size_t)o * cur_w + k]) * (real)cur[k]);
            double val = acc;
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
static v3_d neural_backward_d(const orc_appearance* A, const inreal* feat, const inreal* base, v3_d g, v3_d d, int deg, const inreal* W,
                              double* gfeat, double* gW, double* gbase) {
    if (deg <= 0) return mk_d(0.0, 0.0, 0.0);
    double x[160];
    const int n = neural_inputs(A, feat, base, d.x, d.y, d.z, deg, x);
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
    for (int o = 0; o < 16; o++) gcur[o] = gy[o];
    double gin[128];
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
