"""GPU parity of the Neural appearance (latent features -> frequency encoding + SH bands of the view direction ->
fp16 MLP on tensor cores) against the oracle's fp16-semantics restatement, for the reference's default
configuration (8 features, 1 octave, bands 0-3, 2x16 hidden), the c2 configuration (32 features, 2x64 hidden,
80 inputs), raw features with 1 and 3 hidden layers, and base colors as extra inputs.

The oracle's float build restates the network bit for bit: the encoding's sine and cosine and the SH inputs are the
kernels' single-rounding operations, and every tensor-core instruction's fp32 accumulation of fp16 products follows
the rule measured on the hardware (orc_neural.h tc_accumulate), so the fp16 activations and raw outputs agree exactly
and the colours to the last rounding of the activation functions (asserted within 1e-5 per colour channel). The image
is these colours blended by the reference's own kernels bit for bit (blend_matches_reference), so it is within 1e-5 of
the restatement's colours blended with the reference's decisions; against the IEEE restatement of the whole pipeline
it agrees within fgs_testutil.compare_forward's bounds (decisions at a threshold can flip). Every gradient is compared
at 1e-3 relative L2: the oracle's backward follows the kernels' fp16 semantics (loss-scaled output gradient
and hidden gradients rounded to fp16, data gradients on the restated tensor-core accumulation) and differs in the
order of the weight-gradient sums only."""
import ctypes

import numpy as np
import pytest
import torch

import synthetic as S
from oracle import oracle as O
from fgs_testutil import to_dev, settings_for, gpu_forward_stages, rel_err, compare_forward

pytestmark = pytest.mark.gpu


def blend_matches_reference(g, dev, settings):
    """The reference's own kernels, given this run's Neural colours as precomputed colours, reproduce the forward
    stages and the image bit for bit (the reference's Neural path itself needs tiny-cuda-nn, which is absent)."""
    from oracle import reference as REF
    from fgs_testutil import gpu_colors_by_primitive, assert_matches_reference
    if not REF.available():
        return
    n = dev['means'].shape[0]
    colors = torch.from_numpy(gpu_colors_by_primitive(g, n)).to(dev['means'].device)
    geo = {'means': dev['means'], 'scales': dev['scales'], 'rotations': dev['rotations'], 'opacities': dev['opacities'], 'precomputed_colors': colors}
    ref = REF.Reference('precomputed')
    img_ref = ref.forward(geo, settings)
    assert_matches_reference(g, ref.buffers(), img_ref, exact_image=True)
    ref.close()

CONFIGS = [
    # feature_dim, n_freq, neurons, hidden, base_input, res_act
    (8, 1, 16, 2, False, 'tanh'),
    (32, 1, 64, 2, False, 'tanh'),
    (16, 0, 32, 1, False, 'none'),
    (16, 0, 32, 3, False, 'softplus'),
    (8, 1, 16, 2, True, 'tanh'),
    # 64-wide networks run on the tcgen05 kernels: one hidden layer and raw features, two octaves with base inputs and
    # three hidden layers, and a feature count that is not a multiple of 8 (generic encoding path)
    (16, 0, 64, 1, False, 'none'),
    (8, 2, 64, 3, True, 'softplus'),
    (12, 1, 64, 2, False, 'tanh'),
]


def _setup(F, feat, nf, nn, nh, base_input, res_act):
    n_enc = (feat + (3 if base_input else 0)) * (2 * nf if nf else 1)
    n_in = n_enc + 16
    F.initialize_appearance('neural', 0, 'none', res_act, 'relu', True)
    F.initialize_residual_mlp(n_in, 3, {'otype': 'Identity'}, {'otype': 'FullyFusedMLP', 'activation': 'ReLU', 'output_activation': 'None',
                                                                'n_neurons': nn, 'n_hidden_layers': nh}, base_input, nf, [0, 1, 2, 3])
    pad = (n_in + 15) // 16 * 16
    neural = dict(feature_dim=feat, base_input=int(base_input), n_freq=nf, sh_mask=15, n_input=n_in, n_input_pad=pad, n_neurons=nn,
                  n_hidden=nh, hidden_act=1)
    return neural, S.mlp_layer_shapes(pad, nn, nh)


@pytest.mark.parametrize('cfg', CONFIGS, ids=[f'f{c[0]}x{c[1]}-n{c[2]}x{c[3]}{"-base" if c[4] else ""}-{c[5]}' for c in CONFIGS])
def test_neural_parity(cuda, cfg):
    import FasterGSVDACudaBackend as F
    feat, nf, nn, nh, base_input, res_act = cfg
    neural, shapes = _setup(F, feat, nf, nn, nh, base_input, res_act)
    n, W, H = 12000, 192, 128
    geo = S.geometry(n)
    geo['scales'] = geo['scales'] + 1.0
    app = S.neural_appearance(n, feature_dim=feat, layer_shapes=shapes)
    prims = {**geo, **app}
    cam = S.ring_cameras(3, W, H)[2]
    settings = settings_for(F, cam, 3, cuda)
    dev = to_dev(prims, cuda)
    g = gpu_forward_stages(F, dev, settings)
    a = O.make_appearance('neural', 0, 0, {'none': 0, 'tanh': 1, 'softplus': 2}[res_act], 1, True, neural=neural)
    grad_image = torch.randn(3, H, W, generator=torch.Generator().manual_seed(2)) * 0.01
    o = O.run(a, O.make_view(cam, 3), prims, grad_image=grad_image)
    compare_forward(g, o)
    both = (g['n_touched'] > 0) & (o['n_touched'] > 0)
    col_err = np.abs(g['records'][g['rank_of'][both], 8:11].astype(np.float64) - o['records'][both, 7:10])
    img_err = np.abs(g['image'] - o['image'])
    print(f'[neural {cfg}] colours of {int(both.sum())} primitives max-abs {col_err.max():.3e}; image max-abs {img_err.max():.3e} '
          f'mean-abs {img_err.mean():.3e}')
    assert col_err.max() <= 1e-5
    blend_matches_reference(g, dev, settings)

    leaves = {k: v.clone().requires_grad_(True) for k, v in dev.items()}
    img = F.diff_rasterize(leaves['means'], leaves['scales'], leaves['rotations'], leaves['opacities'], torch.empty(0, device=cuda), settings,
                           base_colors=leaves['base_colors'], residual_params=leaves['residual_params'], mlp_weights=leaves['mlp_weights'])
    img.backward(grad_image.to(cuda))
    for k, t in leaves.items():
        ref = o['grads'][k]
        err = rel_err(t.grad.cpu().numpy().reshape(ref.shape), ref)
        print(f'[neural {cfg}] grad {k} rel {err:.3e}')
        assert err <= 1e-3, f'{k}: relative error {err:.2e}'


def test_neural_tensor_core_many_tiles(cuda):
    """Enough visible rows that CTAs process several 128-row tiles and carry the weight gradient across them."""
    import FasterGSVDACudaBackend as F
    neural, shapes = _setup(F, 32, 1, 64, 2, False, 'tanh')
    n, W, H = 160000, 256, 192
    geo = S.geometry(n, seed=3)
    prims = {**geo, **S.neural_appearance(n, feature_dim=32, layer_shapes=shapes, seed=4)}
    cam = S.ring_cameras(4, W, H)[1]
    settings = settings_for(F, cam, 3, cuda)
    dev = to_dev(prims, cuda)
    a = O.make_appearance('neural', 0, 0, 1, 1, True, neural=neural)
    grad_image = torch.randn(3, H, W, generator=torch.Generator().manual_seed(6)) * 0.01
    o = O.run(a, O.make_view(cam, 3), prims, grad_image=grad_image)
    assert o['n_visible'] > 2 * 148 * 128, o['n_visible']
    leaves = {k: v.clone().requires_grad_(True) for k, v in dev.items()}
    img = F.diff_rasterize(leaves['means'], leaves['scales'], leaves['rotations'], leaves['opacities'], torch.empty(0, device=cuda), settings,
                           base_colors=leaves['base_colors'], residual_params=leaves['residual_params'], mlp_weights=leaves['mlp_weights'])
    img_err = np.abs(img.detach().cpu().numpy() - o['image'])
    print(f'\n[neural many tiles] image max-abs {img_err.max():.3e} mean-abs {img_err.mean():.3e}')
    assert img_err.mean() <= 5e-6 and (img_err.max(0) > 1e-4).mean() <= 1e-3, (img_err.max(), img_err.mean())
    img.backward(grad_image.to(cuda))
    torch.cuda.synchronize()
    from FasterGSVDACudaBackend import _lib
    flag = ctypes.c_int(-1)
    _lib.check(_lib.lib.fgs_tc_timeout(ctypes.byref(flag), 0))
    assert flag.value == 0, 'a tensor-core kernel gave up a bounded wait'
    for k, t in (('means', 1e-3), ('opacities', 1e-3), ('base_colors', 1e-3), ('residual_params', 1e-3), ('mlp_weights', 1e-3)):
        ref = o['grads'][k]
        err = rel_err(leaves[k].grad.cpu().numpy().reshape(ref.shape), ref)
        print(f'[neural many tiles] grad {k} rel {err:.3e}')
        assert err <= t, f'{k}: relative error {err:.2e}'


def test_neural_accumulate_two_views(cuda):
    """accumulate=True adds a second view's gradients to the first's (the data-parallel trainer's mode)."""
    import FasterGSVDACudaBackend as F
    from FasterGSVDACudaBackend import rasterization as R, _lib
    neural, shapes = _setup(F, 32, 1, 64, 2, False, 'tanh')
    n, W, H = 30000, 192, 128
    prims = {**S.geometry(n, seed=8), **S.neural_appearance(n, feature_dim=32, layer_shapes=shapes, seed=9)}
    dev = to_dev(prims, cuda)
    cams = S.ring_cameras(4, W, H)
    gimgs = [torch.randn(3, H, W, generator=torch.Generator().manual_seed(10 + k)).to(cuda) * 0.01 for k in range(2)]
    cp = R._c_primitives(dev['means'], dev['scales'], dev['rotations'], dev['opacities'], None, dev['base_colors'], dev['residual_params'],
                         dev['mlp_weights'])

    def grads_of(views, accumulate_second):
        out = {k: torch.zeros_like(v) for k, v in dev.items()}
        cg = _lib.Gradients(*[out[k].data_ptr() if k in out else None for k in
                              ('means', 'scales', 'rotations', 'opacities', 'precomputed_colors', 'base_colors', 'residual_params', 'mlp_weights')])
        for j, (cam, gi) in enumerate(views):
            st = R.ForwardState(R._rasterizer, cp, settings_for(F, cam, 3, cuda), cuda)
            st.preprocess(cp)
            image = torch.empty(3, H, W, device=cuda)
            st.render_train(image)
            st.backward(cp, image, gi, cg, None, accumulate=accumulate_second and j > 0)
        torch.cuda.synchronize()
        return out

    both = grads_of([(cams[0], gimgs[0]), (cams[1], gimgs[1])], True)
    g0 = grads_of([(cams[0], gimgs[0])], False)
    g1 = grads_of([(cams[1], gimgs[1])], False)
    for k in both:
        ref = (g0[k] + g1[k]).cpu().numpy()
        err = rel_err(both[k].cpu().numpy(), ref)
        assert err <= 1e-5, f'{k}: relative error {err:.2e}'


@pytest.mark.parametrize('cfg', [(16, 0, 64, 1, False, 'none'), (32, 1, 64, 2, False, 'tanh'), (8, 2, 64, 3, True, 'softplus'),
                                 (16, 1, 64, 1, False, 'none'), (8, 1, 64, 2, False, 'softplus')],
                         ids=['1-hidden', '2-hidden', '3-hidden-base', 'f16-1-hidden', 'f8-2-hidden'])
def test_neural_stored_activations_match_recompute(cuda, cfg):
    """A training forward keeps the tensor-core MLP's activations for the backward (frame.mlp_activations); a forward
    whose workspace excludes the store (training=False) leaves the backward to recompute them. Both give the same
    image and the same gradients (up to the order of the fp32 atomics), over enough rows that every CTA fetches
    several tiles' activations. In the cases with one octave and no base input ('2-hidden', 'f16-1-hidden',
    'f8-2-hidden') the stored path runs the warp-specialised backward, so these also check it against the other kernel."""
    import FasterGSVDACudaBackend as F
    from FasterGSVDACudaBackend import rasterization as R, _lib
    feat, nf, nn, nh, base_input, res_act = cfg
    neural, shapes = _setup(F, feat, nf, nn, nh, base_input, res_act)
    n, W, H = 160000, 256, 192
    prims = {**S.geometry(n, seed=3), **S.neural_appearance(n, feature_dim=feat, layer_shapes=shapes, seed=4)}
    dev = to_dev(prims, cuda)
    cam = S.ring_cameras(4, W, H)[1]
    gi = (torch.randn(3, H, W, generator=torch.Generator().manual_seed(6)) * 0.01).to(cuda)
    cp = R._c_primitives(dev['means'], dev['scales'], dev['rotations'], dev['opacities'], None, dev['base_colors'], dev['residual_params'],
                         dev['mlp_weights'])
    names = ('means', 'scales', 'rotations', 'opacities', 'precomputed_colors', 'base_colors', 'residual_params', 'mlp_weights')

    def run(training):
        out = {k: torch.zeros_like(v) for k, v in dev.items()}
        cg = _lib.Gradients(*[out[k].data_ptr() if k in out else None for k in names])
        st = R.ForwardState(R._rasterizer, cp, settings_for(F, cam, 3, cuda), cuda, training=training)
        st.preprocess(cp)
        image = torch.empty(3, H, W, device=cuda)
        st.render_train(image)
        st.backward(cp, image, gi, cg, None)
        torch.cuda.synchronize()
        return st.frame, image.cpu().numpy(), out

    f1, img1, g1 = run(True)
    f0, img0, g0 = run(False)
    assert f1.mlp_activations == 1 and f0.mlp_activations == 0
    assert f1.n_visible > 2 * 148 * 128, f1.n_visible
    np.testing.assert_array_equal(img1, img0)
    for k in g1:
        err = rel_err(g1[k].cpu().numpy(), g0[k].cpu().numpy())
        assert err <= 1e-5, f'{k}: relative error {err:.2e}'
    flag = ctypes.c_int(-1)
    _lib.check(_lib.lib.fgs_tc_timeout(ctypes.byref(flag), 0))
    assert flag.value == 0


def test_neural_degree_zero_backward(cuda):
    """A view rendered at degree 0 skips the MLP: only base colours and geometry receive gradients."""
    import FasterGSVDACudaBackend as F
    neural, shapes = _setup(F, 32, 1, 64, 2, False, 'tanh')
    n, W, H = 10000, 160, 120
    geo = S.geometry(n, seed=11)
    geo['scales'] = geo['scales'] + 1.0
    prims = {**geo, **S.neural_appearance(n, feature_dim=32, layer_shapes=shapes, seed=12)}
    cam = S.ring_cameras(2, W, H)[1]
    dev = to_dev(prims, cuda)
    a = O.make_appearance('neural', 0, 0, 1, 1, True, neural=neural)
    grad_image = torch.randn(3, H, W, generator=torch.Generator().manual_seed(13)) * 0.01
    o = O.run(a, O.make_view(cam, 0), prims, grad_image=grad_image)
    leaves = {k: v.clone().requires_grad_(True) for k, v in dev.items()}
    img = F.diff_rasterize(leaves['means'], leaves['scales'], leaves['rotations'], leaves['opacities'], torch.empty(0, device=cuda),
                           settings_for(F, cam, 0, cuda), base_colors=leaves['base_colors'], residual_params=leaves['residual_params'],
                           mlp_weights=leaves['mlp_weights'])
    d = np.abs(img.detach().cpu().numpy() - o['image'])
    assert d.mean() <= 5e-6 and (d.max(0) > 1e-4).mean() <= 1e-3, (d.max(), d.mean())
    img.backward(grad_image.to(cuda))
    for k in ('means', 'opacities', 'base_colors'):
        ref = o['grads'][k]
        assert rel_err(leaves[k].grad.cpu().numpy().reshape(ref.shape), ref) <= 1e-3, k
    assert float(leaves['residual_params'].grad.abs().max()) == 0.0
    assert leaves['mlp_weights'].grad is None or float(leaves['mlp_weights'].grad.abs().max()) == 0.0


def test_neural_degree_zero_and_inference(cuda):
    import FasterGSVDACudaBackend as F
    neural, shapes = _setup(F, 8, 1, 16, 2, False, 'tanh')
    n, W, H = 8000, 160, 120
    geo = S.geometry(n, seed=5)
    geo['scales'] = geo['scales'] + 1.0
    prims = {**geo, **S.neural_appearance(n, feature_dim=8, layer_shapes=shapes)}
    cam = S.ring_cameras(2, W, H)[0]
    dev = to_dev(prims, cuda)
    a = O.make_appearance('neural', 0, 0, 1, 1, True, neural=neural)
    for degree in (0, 2):
        settings = settings_for(F, cam, degree, cuda)
        img = F.rasterize(dev['means'], dev['scales'], dev['rotations'], dev['opacities'], settings, True, False,
                          base_colors=dev['base_colors'], residual_params=dev['residual_params'], mlp_weights=dev['mlp_weights'])
        o = O.run(a, O.make_view(cam, degree), prims)
        err = np.abs(img.cpu().numpy() - o['image'])
        assert err.mean() <= 5e-6 and (err.max(0) > 1e-4).mean() <= 1e-3, (degree, err.max(), err.mean())
