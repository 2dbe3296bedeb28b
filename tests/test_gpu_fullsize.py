"""Parity at the benchmark configurations' full sizes (one view each), where the small cases of the other tests cannot
reach: tile lists thousands of instances long, 20- to 23-bit depth ranks, instance counts in the millions, radix sorts
over several 4096-key tiles per digit, hundreds of tensor-core tiles per CTA.

- c1 (SH-3, 1,000,000 Gaussians, 1280x720, view 0 of the training ring): every forward stage bit for bit against the
  oracle (all integer stages, records, image, transmittance, contributor counts), and the backward through the public
  autograd API within 1e-3 relative L2 per gradient tensor against the oracle's double-precision backward.
- c3 (NASG-8 inference, 3,000,000 Gaussians, 1920x1080): integer stages bit for bit, colors within 1e-5 relative, the
  clamped HWC inference image within 1e-4 of the oracle; and, with the GPU's own colors given to the oracle as
  precomputed colors, the blended image bit for bit.
- c2 (Neural 80-64-64-3, 1,000,000 Gaussians, 1264x832): against the full oracle run, integer stages bit for bit, the
  image within 1e-3 max / 1e-5 mean, gradients within 1e-3 (geometry) / 1e-2 (base colours, features, weights).
- c4 (Neural 80-64-64-3, 6,000,000 Gaussians, 1920x1080, view 0 of the training batch): culling, depth order, binning,
  records and the blended image bit for bit against the oracle fed the GPU's colors; the colors themselves against the
  oracle's fp16-semantics MLP on a seeded sample of 20,000 Gaussians (1e-3 max abs, 2e-5 mean abs: the tensor cores
  sum in another order, which moves an fp16 rounding by one unit now and then); determinism of the whole forward; and
  linearity of the backward in the upstream gradient (twice the gradient gives twice every parameter gradient, within
  1e-4 relative L2: only the order of the fp32 atomics and an fp16 rounding they tip differ).

The oracle runs on all host cores here (its per-primitive and per-pixel loops give the same results on any thread
count; the backward's per-thread sums differ only in double-precision rounding)."""
import os

import numpy as np
import pytest
import torch

import synthetic as S
from oracle import oracle as O
from fgs_testutil import settings_for, gpu_forward_stages, rel_err, compare_forward, gpu_colors_by_primitive

pytestmark = pytest.mark.gpu


@pytest.fixture
def oracle_threads():
    O.set_threads(os.cpu_count() or 1)
    yield
    O.set_threads(1)


def _geometry_only(prims: dict, colors: np.ndarray) -> dict:
    return {'means': prims['means'], 'scales': prims['scales'], 'rotations': prims['rotations'], 'opacities': prims['opacities'],
            'precomputed_colors': torch.from_numpy(colors)}


def _assert_blend_of_gpu_colors(g, prims, cam, degree):
    """The oracle, given the GPU's blended colors as precomputed colors, reproduces the GPU forward bit for bit."""
    a = O.make_appearance('sh', 3, 0, 0, 1, True)
    o = O.run(a, O.make_view(cam, degree), _geometry_only(prims, gpu_colors_by_primitive(g, prims['means'].shape[0])))
    compare_forward(g, o, exact_image=True)
    return o


def test_c1_full_size_forward_bit_exact_and_backward(cuda, oracle_threads):
    import FasterGSVDACudaBackend as F
    n, W, H = 1_000_000, 1280, 720
    F.initialize_appearance('sh', 3, 'none', 'none', 'relu', True)
    prims = {**S.geometry(n), **S.sh_appearance(n, 3)}
    cam = S.ring_cameras(8, W, H)[0]
    settings = settings_for(F, cam, 3, cuda)
    dev = {k: v.to(cuda).contiguous() for k, v in prims.items()}
    g = gpu_forward_stages(F, dev, settings)
    grad_image = torch.randn(3, H, W, generator=torch.Generator().manual_seed(2)) * 0.01
    o = O.run(O.make_appearance('sh', 3, 0, 0, 1, True), O.make_view(cam, 3), prims, grad_image=grad_image)
    assert o['n_visible'] > 400_000 and o['n_instances'] > 1_000_000
    assert (o['ranges'][:, 1].astype(np.int64) - o['ranges'][:, 0]).max() > 1000
    compare_forward(g, o, exact_image=True)

    leaves = {k: v.clone().requires_grad_(True) for k, v in dev.items()}
    img = F.diff_rasterize(leaves['means'], leaves['scales'], leaves['rotations'], leaves['opacities'], torch.empty(0, device=cuda), settings,
                           base_colors=leaves['base_colors'], residual_params=leaves['residual_params'])
    np.testing.assert_array_equal(img.detach().cpu().numpy(), o['image'])
    img.backward(grad_image.to(cuda))
    for k, t in leaves.items():
        ref = o['grads'][k]
        err = rel_err(t.grad.cpu().numpy().reshape(ref.shape), ref)
        assert err <= 1e-3, f'{k}: relative error {err:.2e}'


def test_c3_full_size_nasg_inference(cuda, oracle_threads):
    import FasterGSVDACudaBackend as F
    n, W, H, lobes = 3_000_000, 1920, 1080, 8
    F.initialize_appearance('nasg', lobes, 'none', 'none', 'relu', True)
    prims = {**S.geometry(n), **S.nasg_appearance(n, lobes)}
    cam = S.ring_cameras(64, W, H)[0]
    settings = settings_for(F, cam, lobes, cuda)
    dev = {k: v.to(cuda).contiguous() for k, v in prims.items()}
    img = F.rasterize(dev['means'], dev['scales'], dev['rotations'], dev['opacities'], settings, False, True,
                      base_colors=dev['base_colors'], residual_params=dev['residual_params']).cpu().numpy()
    g = gpu_forward_stages(F, dev, settings)
    o = O.run(O.make_appearance('nasg', lobes, 0, 0, 1, True), O.make_view(cam, lobes), prims)
    assert o['n_visible'] > 1_000_000 and o['n_instances'] > 4_000_000
    compare_forward(g, o, exact_image=False)
    assert np.abs(img - np.clip(o['image'], 0.0, 1.0).transpose(1, 2, 0)).max() <= 1e-4
    _assert_blend_of_gpu_colors(g, prims, cam, lobes)


def _neural_c4(F):
    feat, n_freq, neurons, hidden = 32, 1, 64, 2
    n_in = feat * 2 * n_freq + 16
    pad = (n_in + 15) // 16 * 16
    F.initialize_appearance('neural', 0, 'none', 'tanh', 'relu', True)
    F.initialize_residual_mlp(n_in, 3, {'otype': 'Identity'}, {'otype': 'FullyFusedMLP', 'activation': 'ReLU', 'output_activation': 'None',
                                                               'n_neurons': neurons, 'n_hidden_layers': hidden}, False, n_freq, [0, 1, 2, 3])
    neural = dict(feature_dim=feat, base_input=0, n_freq=n_freq, sh_mask=15, n_input=n_in, n_input_pad=pad, n_neurons=neurons, n_hidden=hidden,
                  hidden_act=1)
    return neural, S.mlp_layer_shapes(pad, neurons, hidden)


def test_c2_full_size_neural_forward_backward(cuda, oracle_threads):
    """c2: Neural appearance (32 latent features, 80 inputs, 2x64 hidden), 1,000,000 Gaussians at 1264x832, compared
    with the full oracle run (no sampling): integer stages bit for bit, image within the Neural tolerances, gradients
    within 1e-3 (geometry) / 1e-2 (base colours, features, MLP weights) relative L2."""
    import FasterGSVDACudaBackend as F
    n, W, H = 1_000_000, 1264, 832
    neural, shapes = _neural_c4(F)
    prims = {**S.geometry(n), **S.neural_appearance(n, 32, layer_shapes=shapes)}
    cam = S.ring_cameras(1, W, H)[0]
    settings = settings_for(F, cam, 3, cuda)
    dev = {k: v.to(cuda).contiguous() for k, v in prims.items()}
    g = gpu_forward_stages(F, dev, settings)
    grad_image = torch.randn(3, H, W, generator=torch.Generator().manual_seed(2)) * 0.01
    o = O.run(O.make_appearance('neural', 0, 0, 1, 1, True, neural=neural), O.make_view(cam, 3), prims, grad_image=grad_image)
    assert o['n_visible'] > 500_000 and o['n_instances'] > 1_200_000
    assert g['n_visible'] == o['n_visible'] and g['n_instances'] == o['n_instances']
    for k in ('n_touched', 'sorted_idx', 'tile_keys', 'ranks', 'ranges', 'n_contrib'):
        np.testing.assert_array_equal(g[k], o[k], err_msg=k)
    err = np.abs(g['image'] - o['image'])
    assert err.max() <= 1e-3 and err.mean() <= 1e-5, (err.max(), err.mean())
    del g

    leaves = {k: v.clone().requires_grad_(True) for k, v in dev.items()}
    img = F.diff_rasterize(leaves['means'], leaves['scales'], leaves['rotations'], leaves['opacities'], torch.empty(0, device=cuda), settings,
                           base_colors=leaves['base_colors'], residual_params=leaves['residual_params'], mlp_weights=leaves['mlp_weights'])
    img.backward(grad_image.to(cuda))
    tol = {'means': 1e-3, 'scales': 1e-3, 'rotations': 1e-3, 'opacities': 1e-3, 'base_colors': 1e-2, 'residual_params': 1e-2, 'mlp_weights': 1e-2}
    for k, t in leaves.items():
        ref = o['grads'][k]
        e = rel_err(t.grad.cpu().numpy().reshape(ref.shape), ref)
        assert e <= tol[k], f'{k}: relative error {e:.2e}'


def test_c4_full_size_neural_view(cuda, oracle_threads):
    import FasterGSVDACudaBackend as F
    n, W, H = 6_000_000, 1920, 1080
    neural, shapes = _neural_c4(F)
    prims = {**S.geometry(n), **S.neural_appearance(n, 32, layer_shapes=shapes)}
    cam = S.ring_cameras(8, W, H)[0]
    settings = settings_for(F, cam, 3, cuda)
    dev = {k: v.to(cuda).contiguous() for k, v in prims.items()}

    g = gpu_forward_stages(F, dev, settings)
    o = _assert_blend_of_gpu_colors(g, prims, cam, 3)
    assert o['n_visible'] > 2_000_000 and o['n_instances'] > 8_000_000

    # the colors: the oracle's MLP on a seeded sample of Gaussians (colors are per primitive, so a subset scene gives
    # the same colors as the full one)
    idx = torch.randperm(n, generator=torch.Generator().manual_seed(11))[:20000].sort().values
    sub = {k: (v if k == 'mlp_weights' else v[idx]) for k, v in prims.items()}
    a = O.make_appearance('neural', 0, 0, 1, 1, True, neural=neural)
    os_ = O.run(a, O.make_view(cam, 3), sub)
    np.testing.assert_array_equal(os_['n_touched'], g['n_touched'][idx.numpy()])
    vis = os_['n_touched'] > 0
    assert vis.sum() > 5000
    rank = g['rank_of'][idx.numpy()[vis]]
    err = np.abs(g['records'][rank, 8:11] - os_['records'][vis, 7:10].astype(np.float32))
    assert err.max() <= 1e-3 and err.mean() <= 2e-5, (err.max(), err.mean())

    # determinism of the forward: a second run reproduces every stage and the image bit for bit
    g2 = gpu_forward_stages(F, dev, settings)
    for k in ('n_touched', 'sorted_idx', 'instance_offsets', 'tile_keys', 'ranks', 'ranges', 'bucket_off', 'records', 'image', 'final_T',
              'n_contrib'):
        np.testing.assert_array_equal(g2[k], g[k], err_msg=k)
    del g, g2, o

    # linearity of the backward in the upstream gradient
    up = torch.randn(3, H, W, generator=torch.Generator().manual_seed(2)).mul_(0.01).to(cuda)
    grads = []
    for scale in (1.0, 2.0):
        leaves = {k: v.clone().requires_grad_(True) for k, v in dev.items()}
        img = F.diff_rasterize(leaves['means'], leaves['scales'], leaves['rotations'], leaves['opacities'], torch.empty(0, device=cuda), settings,
                               base_colors=leaves['base_colors'], residual_params=leaves['residual_params'], mlp_weights=leaves['mlp_weights'])
        img.backward(up * scale)
        grads.append({k: t.grad.double() for k, t in leaves.items()})
        del leaves, img
    for k in grads[0]:
        a1, a2 = grads[0][k], grads[1][k]
        assert float(a1.norm()) > 0, k
        err = float((a2 - 2.0 * a1).norm() / (2.0 * a1).norm())
        assert err <= 1e-4, f'{k}: {err:.2e}'
