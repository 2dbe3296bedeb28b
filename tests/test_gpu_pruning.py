"""GPU parity of update_pruning_scores (Speedy-Splat scores, rasterization/include/kernels_pruning_scores.cuh:11-173)
against the oracle (oracle/fgs_oracle.c orc_pruning_scores, float acceptance as the GPU, double arithmetic):
within 1e-3 relative (L2 over all primitives) and elementwise to 1e-2 relative; the scores are added into the
caller's tensor, primitives that contribute to no pixel keep their value."""
import numpy as np
import pytest
import torch

import synthetic as S
from oracle import oracle as O
from fgs_testutil import scene, to_dev, settings_for, rel_err

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize('model,proper_aa,bg', [('sh', False, (0.0, 0.0, 0.0)), ('sh', True, (0.2, 0.5, 0.9)), ('precomputed', False, (1.0, 1.0, 1.0))])
def test_pruning_scores_match_oracle(cuda, model, proper_aa, bg):
    import FasterGSVDACudaBackend as F
    F.initialize_appearance('sh', 3, 'none', 'none', 'relu', True)
    n, W, H = 20000, 256, 192
    prims = scene(model, n, 3, seed=3, scale_shift=1.0)
    cam = S.ring_cameras(3, W, H)[2]
    cam.bg = torch.tensor(bg, dtype=torch.float32)
    settings = settings_for(F, cam, 3, cuda, proper_aa=proper_aa)
    dev = to_dev(prims, cuda)
    v = O.make_view(cam, 3, proper_aa=proper_aa)
    o = O.run(O.make_appearance('sh', 3, 0, 0, 1, True), v, prims, pruning=True)
    ref = o['pruning_scores']
    assert (ref > 0).sum() > 1000

    base = torch.rand(n, generator=torch.Generator().manual_seed(5)).to(cuda)
    scores = base.clone()
    kw = dict(precomputed_colors=dev.get('precomputed_colors'), base_colors=dev.get('base_colors'), residual_params=dev.get('residual_params'))
    assert F.update_pruning_scores(scores, dev['means'], dev['scales'], dev['rotations'], dev['opacities'], settings, **kw) is None
    got = (scores - base).cpu().numpy().astype(np.float64)
    assert rel_err(got, ref) <= 1e-3
    assert np.allclose(got, ref, rtol=1e-2, atol=1e-5 * ref.max())
    untouched = ref == 0
    np.testing.assert_array_equal(scores.cpu().numpy()[untouched], base.cpu().numpy()[untouched])
    # a second view accumulates
    F.update_pruning_scores(scores, dev['means'], dev['scales'], dev['rotations'], dev['opacities'], settings, **kw)
    assert rel_err((scores - base).cpu().numpy(), 2 * ref) <= 1e-3


def test_pruning_scores_reject_bad_scores(cuda):
    import FasterGSVDACudaBackend as F
    F.initialize_appearance('sh', 3, 'none', 'none', 'relu', True)
    prims = to_dev(scene('sh', 100, 3, seed=1), cuda)
    cam = S.ring_cameras(3, 64, 48)[0]
    settings = settings_for(F, cam, 3, cuda)
    with pytest.raises(RuntimeError):
        F.update_pruning_scores(torch.zeros(99, device=cuda), prims['means'], prims['scales'], prims['rotations'], prims['opacities'], settings,
                                base_colors=prims['base_colors'], residual_params=prims['residual_params'])
