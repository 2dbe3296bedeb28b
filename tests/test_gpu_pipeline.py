"""GPU parity: every stage of the training forward and the backward against the CPU oracle, for all appearance
models. Integer stages (culling, depth keys, depth order, instance offsets, tile keys, tile lists, ranges,
contributor counts) and the transmittance are compared bit for bit; images bit for bit where the colors are
(precomputed, SH with identity / ReLU activations) and within 1e-4 max-abs otherwise; gradients within 1e-3
relative (L2 over each tensor, against the double-precision oracle backward)."""
import numpy as np
import pytest
import torch

import synthetic as S
from oracle import oracle as O
from fgs_testutil import ACT, scene, to_dev, settings_for, gpu_forward_stages, rel_err, oracle_records_in_rank_order

pytestmark = pytest.mark.gpu

CASES = [
    # model, degree, base, residual, color, exact_image
    ('precomputed', 0, 'none', 'none', 'relu', True),
    ('sh', 3, 'none', 'none', 'relu', True),
    ('sh', 1, 'none', 'none', 'none', True),
    ('sh', 2, 'exp', 'tanh', 'satexp', False),
    ('sv', 8, 'none', 'none', 'relu', False),
    ('nasg', 8, 'none', 'tanh', 'relu', False),
    ('nasgabor', 4, 'none', 'tanh', 'sigmoid', False),
]


def _configure(F, model, degree, base, res, col):
    if model != 'precomputed':
        F.initialize_appearance(model, degree, base, res, col, True)
    else:
        F.initialize_appearance('sh', 3, 'none', 'none', 'relu', True)


def _compare_forward(g, o, exact_image):
    assert g['n_visible'] == o['n_visible']
    assert g['n_instances'] == o['n_instances']
    np.testing.assert_array_equal(g['n_touched'], o['n_touched'])
    vis = o['n_touched'] > 0
    np.testing.assert_array_equal(g['depth_key'][vis], o['depth_key'][vis])
    np.testing.assert_array_equal(g['sorted_idx'], o['sorted_idx'])
    np.testing.assert_array_equal(g['instance_offsets'], o['instance_offsets'])
    np.testing.assert_array_equal(g['tile_keys'], o['tile_keys'])
    np.testing.assert_array_equal(g['ranks'], o['ranks'])
    np.testing.assert_array_equal(g['ranges'], o['ranges'])
    # bucket offsets: inclusive scan of ceil(tile list length / 32) (kernels_forward.cuh:14-24, forward.cu:204-219)
    lengths = o['ranges'][:, 1].astype(np.int64) - o['ranges'][:, 0].astype(np.int64)
    np.testing.assert_array_equal(g['bucket_off'], np.cumsum((lengths + 31) // 32).astype(np.uint32))
    rec_o = oracle_records_in_rank_order(o)
    rec_g = g['records']
    # geometry fields bit-exact: mean2d, opacity, power threshold, conic, bounds
    for gi, oi in ((0, 0), (1, 1), (2, 2), (3, 3), (4, 4), (5, 5), (6, 6)):
        np.testing.assert_array_equal(rec_g[:, gi], rec_o[:, oi].astype(np.float32))
    bx = rec_g[:, 7].view(np.uint32)
    by = rec_g[:, 11].view(np.uint32)
    np.testing.assert_array_equal(bx & 0xffff, rec_o[:, 10].astype(np.uint32))
    np.testing.assert_array_equal(bx >> 16, rec_o[:, 11].astype(np.uint32))
    np.testing.assert_array_equal(by & 0xffff, rec_o[:, 12].astype(np.uint32))
    np.testing.assert_array_equal(by >> 16, rec_o[:, 13].astype(np.uint32))
    np.testing.assert_array_equal(g['n_contrib'], o['n_contrib'])
    colors_g = rec_g[:, 8:11]
    colors_o = rec_o[:, 7:10].astype(np.float32)
    if exact_image:
        np.testing.assert_array_equal(colors_g, colors_o)
        np.testing.assert_array_equal(g['image'], o['image'])
        np.testing.assert_array_equal(g['final_T'], o['final_T'])
    else:
        assert np.abs(colors_g - colors_o).max() <= 1e-5 * max(1.0, np.abs(colors_o).max())
        assert np.abs(g['image'] - o['image']).max() <= 1e-4
        assert np.abs(g['final_T'] - o['final_T']).max() <= 1e-6


@pytest.mark.parametrize('case', CASES, ids=[f'{c[0]}{c[1]}-{c[2]}-{c[3]}-{c[4]}' for c in CASES])
def test_forward_backward_parity(cuda, case):
    import FasterGSVDACudaBackend as F
    model, degree, base, res, col, exact = case
    _configure(F, model, degree, base, res, col)
    n, W, H = 20000, 256, 192
    prims = scene(model, n, degree, seed=0, scale_shift=1.0)
    cam = S.ring_cameras(3, W, H)[1]
    settings = settings_for(F, cam, degree, cuda)
    dev = to_dev(prims, cuda)
    g = gpu_forward_stages(F, dev, settings)
    a = O.make_appearance(model if model != 'precomputed' else 'sh', degree if model != 'precomputed' else 3, ACT['base'][base],
                          ACT['res'][res], ACT['color'][col], True)
    grad_image = torch.randn(3, H, W, generator=torch.Generator().manual_seed(2)) * 0.01
    o = O.run(a, O.make_view(cam, degree), prims, grad_image=grad_image)
    assert o['n_visible'] > 1000 and o['n_instances'] > o['n_visible']
    _compare_forward(g, o, exact)

    # backward through autograd
    leaves = {k: v.clone().requires_grad_(True) for k, v in dev.items()}
    img = F.diff_rasterize(leaves['means'], leaves['scales'], leaves['rotations'], leaves['opacities'], torch.empty(0, device=cuda), settings,
                           precomputed_colors=leaves.get('precomputed_colors'), base_colors=leaves.get('base_colors'),
                           residual_params=leaves.get('residual_params'))
    if exact:
        np.testing.assert_array_equal(img.detach().cpu().numpy(), o['image'])
    img.backward(grad_image.to(cuda))
    for k, t in leaves.items():
        ref = o['grads'][k]
        got = t.grad.detach().cpu().numpy().reshape(ref.shape)
        err = rel_err(got, ref)
        assert err <= 1e-3, f'{k}: relative error {err:.2e}'
        scale = np.abs(ref).max()
        assert np.allclose(got, ref, rtol=1e-2, atol=1e-4 * scale), f'{k}: elementwise mismatch'


def test_variants_proper_aa_render_base_densification(cuda):
    import FasterGSVDACudaBackend as F
    F.initialize_appearance('sh', 3, 'none', 'none', 'relu', True)
    n, W, H = 15000, 200, 150
    prims = scene('sh', n, 3, seed=4, scale_shift=1.0)
    cam = S.ring_cameras(5, W, H)[2]
    for proper_aa, render_base in ((True, True), (False, False)):
        settings = settings_for(F, cam, 3, cuda, proper_aa=proper_aa, render_base=render_base)
        dev = to_dev(prims, cuda)
        g = gpu_forward_stages(F, dev, settings)
        a = O.make_appearance('sh', 3, 0, 0, 1, True)
        grad_image = torch.randn(3, H, W, generator=torch.Generator().manual_seed(2)) * 0.01
        o = O.run(a, O.make_view(cam, 3, proper_aa=proper_aa, render_base=render_base), prims, grad_image=grad_image, densification_rows=3)
        _compare_forward(g, o, exact_image=True)
        leaves = {k: v.clone().requires_grad_(True) for k, v in dev.items()}
        dens = torch.zeros(3, n, device=cuda)
        img = F.diff_rasterize(leaves['means'], leaves['scales'], leaves['rotations'], leaves['opacities'], dens, settings,
                               base_colors=leaves['base_colors'], residual_params=leaves['residual_params'])
        img.backward(grad_image.to(cuda))
        for k, t in leaves.items():
            ref = o['grads'][k]
            err = rel_err(t.grad.cpu().numpy().reshape(ref.shape), ref)
            assert err <= 1e-3, f'{k} (aa={proper_aa}, base={render_base}): {err:.2e}'
        d = dens.cpu().numpy()
        np.testing.assert_array_equal(d[0], o['densification'][0].astype(np.float32))
        assert rel_err(d[1], o['densification'][1]) <= 1e-3
        assert rel_err(d[2], o['densification'][2]) <= 1e-3


@pytest.mark.parametrize('to_chw,clamp', [(False, True), (True, False)])
def test_inference_matches_oracle(cuda, to_chw, clamp):
    import FasterGSVDACudaBackend as F
    F.initialize_appearance('sh', 3, 'none', 'none', 'relu', True)
    n, W, H = 20000, 250, 130
    prims = scene('sh', n, 3, seed=9, scale_shift=1.0)
    cam = S.ring_cameras(4, W, H)[3]
    settings = settings_for(F, cam, 3, cuda)
    dev = to_dev(prims, cuda)
    img = F.rasterize(dev['means'], dev['scales'], dev['rotations'], dev['opacities'], settings, to_chw, clamp,
                      base_colors=dev['base_colors'], residual_params=dev['residual_params'])
    o = O.run(O.make_appearance('sh', 3, 0, 0, 1, True), O.make_view(cam, 3), prims)
    ref = o['image']
    if clamp:
        ref = np.clip(ref, 0.0, 1.0)
    if not to_chw:
        ref = ref.transpose(1, 2, 0)
    np.testing.assert_array_equal(img.cpu().numpy(), ref)
