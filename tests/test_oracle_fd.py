"""Finite-difference check of the oracle backward (double-precision build) for every appearance model, the
precomputed-colors path and proper antialiasing: the analytic gradient of L = <image, G> must match central
differences (step 1e-6) to 1e-3 relative."""
import numpy as np
import pytest
import torch

import synthetic as S
from oracle import oracle as O
from fgs_testutil import scene

CASES = [('sh', 3, 0, 1, False), ('sh', 2, 1, 5, False), ('sv', 4, 1, 1, False), ('nasg', 3, 1, 1, False), ('nasgabor', 3, 2, 3, False),
         ('precomputed', 0, 0, 1, False), ('sh', 3, 0, 1, True)]


@pytest.mark.parametrize('model,deg,res_act,col_act,aa', CASES)
def test_backward_matches_finite_differences(model, deg, res_act, col_act, aa):
    n, W, H = 300, 64, 48
    prims = {k: v.double().numpy() for k, v in scene(model, n, deg, seed=0, scale_shift=2.5).items()}
    cam = S.look_at(torch.tensor([0.0, 0.0, 12.0]), W, H)
    v = O.make_view(cam, deg, proper_aa=aa)
    a = O.make_appearance(model if model != 'precomputed' else 'sh', deg if model != 'precomputed' else 3, 0, res_act, col_act, True)
    G = torch.randn(3, H, W, generator=torch.Generator().manual_seed(2)).numpy()
    out = O.run(a, v, prims, grad_image=G, double=True)

    def loss(pr):
        return float((O.run(a, v, pr, double=True)['image'] * G).sum())

    rng = np.random.default_rng(1)
    vis = np.where(out['rank_of'] != 0xffffffff)[0]
    assert len(vis) > 50
    keys = [k for k in ('means', 'scales', 'rotations', 'opacities', 'base_colors', 'residual_params', 'precomputed_colors') if k in prims]
    if aa:
        # with proper antialiasing the opacity compensation factor is detached from the 2D covariance by design
        # (rasterization_config.h:12), so only the opacity and color gradients are exact derivatives
        keys = [k for k in keys if k in ('opacities', 'base_colors', 'residual_params')]
    bad = []
    for key in keys:
        ana = out['grads'][key].reshape(n, -1)
        for _ in range(4):
            i, j = rng.choice(vis), rng.integers(ana.shape[1])
            h = 1e-6
            p1 = {k: x.copy() for k, x in prims.items()}
            p2 = {k: x.copy() for k, x in prims.items()}
            p1[key].reshape(n, -1)[i, j] += h
            p2[key].reshape(n, -1)[i, j] -= h
            fd = (loss(p1) - loss(p2)) / (2 * h)
            if abs(ana[i, j] - fd) > 1e-3 * max(abs(fd), 1e-3) + 1e-6:
                bad.append((key, int(i), int(j), float(ana[i, j]), fd))
    assert not bad, bad


@pytest.mark.parametrize('base_input', [False, True])
def test_neural_backward_matches_finite_differences(base_input):
    feat, nf, nn, nh = 8, 1, 16, 2
    n_in = (feat + (3 if base_input else 0)) * 2 * nf + 16
    pad = (n_in + 15) // 16 * 16
    shapes = S.mlp_layer_shapes(pad, nn, nh)
    neural = dict(feature_dim=feat, base_input=int(base_input), n_freq=nf, sh_mask=15, n_input=n_in, n_input_pad=pad, n_neurons=nn,
                  n_hidden=nh, hidden_act=1)
    n, W, H = 300, 64, 48
    geo = S.geometry(n)
    geo['scales'] = geo['scales'] + 2.5
    prims = {k: v.double().numpy() for k, v in {**geo, **S.neural_appearance(n, feature_dim=feat, layer_shapes=shapes)}.items()}
    cam = S.look_at(torch.tensor([0.0, 0.0, 12.0]), W, H)
    v = O.make_view(cam, 3)
    a = O.make_appearance('neural', 0, 0, 1, 1, True, neural=neural)
    G = torch.randn(3, H, W, generator=torch.Generator().manual_seed(2)).numpy()
    out = O.run(a, v, prims, grad_image=G, double=True)

    def loss(pr):
        return float((O.run(a, v, pr, double=True)['image'] * G).sum())

    rng = np.random.default_rng(0)
    vis = np.where(out['rank_of'] != 0xffffffff)[0]
    bad = []
    for key in ('means', 'residual_params', 'mlp_weights', 'base_colors'):
        for _ in range(5):
            p1 = {k: x.copy() for k, x in prims.items()}
            p2 = {k: x.copy() for k, x in prims.items()}
            h = 1e-6
            if key == 'mlp_weights':
                i = int(rng.integers(prims[key].size))
                p1[key][i] += h
                p2[key][i] -= h
                ana = out['grads'][key][i]
            else:
                i, j = rng.choice(vis), rng.integers(prims[key].reshape(n, -1).shape[1])
                p1[key].reshape(n, -1)[i, j] += h
                p2[key].reshape(n, -1)[i, j] -= h
                ana = out['grads'][key].reshape(n, -1)[i, j]
            fd = (loss(p1) - loss(p2)) / (2 * h)
            if abs(ana - fd) > 1e-3 * max(abs(fd), 1e-3) + 1e-6:
                bad.append((key, fd, ana))
    assert not bad, bad
