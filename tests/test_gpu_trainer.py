"""The training step's view pipeline (trainer.Trainer.backward_views with overlap_views): consecutive views alternate
between two streams with their own workspaces while the backward passes stay chained in view order. The loss is
bit-identical to the sequential order; the accumulated gradients agree to float rounding (the blend backward adds
per-warp sums with atomics, whose order varies from run to run in either mode), for SH and the Neural appearance."""
import pytest
import torch

import synthetic as S
from fgs_testutil import scene, settings_for

pytestmark = pytest.mark.gpu

LRS = {'means': 1e-3, 'scales': 5e-3, 'rotations': 1e-3, 'opacities': 5e-2, 'base_colors': 2.5e-3, 'residual_params': 1e-3,
       'mlp_weights': 1e-3}


def _prims(model: str) -> dict:
    if model == 'sh':
        return scene('sh', 60000, 3, seed=2, scale_shift=1.0)
    geo = S.geometry(60000)
    geo['scales'] = geo['scales'] + 1.0
    shapes = S.mlp_layer_shapes(80, 64, 2)
    return {**geo, **S.neural_appearance(60000, feature_dim=32, layer_shapes=shapes)}


@pytest.mark.parametrize('model', ['sh', 'neural'])
def test_view_overlap_matches_sequential(cuda, model):
    import FasterGSVDACudaBackend as F
    from trainer import Trainer
    if model == 'sh':
        F.initialize_appearance('sh', 3, 'none', 'none', 'relu', True)
    else:
        F.initialize_appearance('neural', 0, 'none', 'tanh', 'relu', True)
        F.initialize_residual_mlp(80, 3, {'otype': 'Identity'}, {'otype': 'FullyFusedMLP', 'activation': 'ReLU', 'output_activation': 'None',
                                                                 'n_neurons': 64, 'n_hidden_layers': 2}, False, 1, [0, 1, 2, 3])
    prims = {k: v.to(cuda) for k, v in _prims(model).items()}
    cams = S.ring_cameras(5, 320, 240)
    settings = [settings_for(F, c, 3, cuda) for c in cams]
    g = torch.Generator().manual_seed(4)
    targets = [torch.rand(3, 240, 320, generator=g).to(cuda) for _ in cams]
    out = {}
    for overlap in (False, True):
        tr = Trainer(prims, LRS, cuda, overlap_views=overlap)
        tr.grads.zero_()
        loss = tr.backward_views(settings, targets)
        torch.cuda.synchronize()
        out[overlap] = (loss.item(), tr.grads.clone())
    assert out[True][0] == out[False][0]
    a, b = out[True][1].double(), out[False][1].double()
    assert b.abs().sum().item() > 0
    assert ((a - b).norm() / b.norm()).item() <= 1e-5
    assert torch.allclose(a, b, rtol=1e-3, atol=1e-6 * b.abs().max().item())
