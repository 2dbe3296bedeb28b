"""GPU edge cases of the reference's input space: empty and tiny inputs, everything culled, footprints larger than
the warp-cooperative threshold (screen-filling Gaussians), image sizes that are not tile multiples, and 32-bit tile
keys (more than 2^16 tiles). Each rendered case is checked stage by stage against the reference's own kernels
(oracle/_ref, fgs_testutil.assert_matches_reference) and against the C restatement within its tolerances; the empty
and all-culled scenes, which the reference's host code cannot launch (zero-sized grids), against their exact
expected results."""
import numpy as np
import pytest
import torch

import synthetic as S
from oracle import oracle as O
from oracle import reference as REF
from fgs_testutil import scene, to_dev, settings_for, gpu_forward_stages, compare_forward, assert_matches_reference

pytestmark = pytest.mark.gpu


def _check(F, cuda, prims, cam, degree=3):
    settings = settings_for(F, cam, degree, cuda)
    dev = to_dev(prims, cuda)
    g = gpu_forward_stages(F, dev, settings)
    o = O.run(O.make_appearance('sh', 3, 0, 0, 1, True), O.make_view(cam, degree), prims)
    compare_forward(g, o)
    if REF.available() and g['n_visible'] > 0:
        ref = REF.Reference('sh3_none_none_relu')
        img_ref = ref.forward(dev, settings)
        assert_matches_reference(g, ref.buffers(), img_ref)
        ref.close()
    return g, o


def test_empty_and_single(cuda):
    import FasterGSVDACudaBackend as F
    F.initialize_appearance('sh', 3, 'none', 'none', 'relu', True)
    cam = S.ring_cameras(1, 64, 48)[0]
    settings = settings_for(F, cam, 3, cuda)
    empty = {k: v[:0] for k, v in scene('sh', 4, 3).items()}
    dev = to_dev(empty, cuda)
    img = F.rasterize(dev['means'], dev['scales'], dev['rotations'], dev['opacities'], settings, True, False,
                      base_colors=dev['base_colors'], residual_params=dev['residual_params'])
    assert img.shape == (3, 48, 64) and torch.all(img == 0)
    one = scene('sh', 1, 3)
    one['means'][:] = torch.tensor([0.0, 0.0, 0.0])
    one['scales'][:] = -1.0
    one['opacities'][:] = 3.0
    g, o = _check(F, cuda, one, cam)
    assert g['n_visible'] == 1


def test_all_culled(cuda):
    import FasterGSVDACudaBackend as F
    F.initialize_appearance('sh', 3, 'none', 'none', 'relu', True)
    cam = S.ring_cameras(1, 80, 60)[0]
    p = scene('sh', 5000, 3)
    p['opacities'][:] = -10.0  # sigmoid < 1/255 everywhere
    g, o = _check(F, cuda, p, cam)
    assert g['n_visible'] == 0 and g['n_instances'] == 0
    assert np.all(g['image'] == 0)


def test_screen_filling_and_ragged_sizes(cuda):
    import FasterGSVDACudaBackend as F
    F.initialize_appearance('sh', 3, 'none', 'none', 'relu', True)
    p = scene('sh', 3000, 3, seed=3)
    p['scales'][:50] = 0.5  # huge footprints: many tiles, warp-cooperative counting and emission
    for W, H in ((101, 37), (16, 12), (17, 13), (333, 250)):
        cam = S.ring_cameras(2, W, H)[1]
        _check(F, cuda, p, cam)


def test_wide_tile_keys(cuda):
    import FasterGSVDACudaBackend as F
    F.initialize_appearance('sh', 3, 'none', 'none', 'relu', True)
    W, H = 4112, 3084  # 257 x 257 tiles > 2^16 -> 32-bit keys
    p = scene('sh', 4000, 3, seed=5, scale_shift=2.0)
    cam = S.ring_cameras(1, W, H)[0]
    g, o = _check(F, cuda, p, cam)
    assert g['state'].frame.wide_keys == 1
