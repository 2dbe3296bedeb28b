"""The allocation-free inference entry point (fgs_inference_noalloc) renders the same image as the regular
inference path, on two calls in a row (the second call must not see stale state from the first).

Callers of that entry point are render hooks that cannot allocate device memory mid-frame (a host application
owns the device-memory budget); the entry point keeps its workspaces in a static device array instead. Covered:
SH from raw parameters, precomputed colours, and the Neural model on both MLP paths (a 64-wide network on the
tensor-core kernels, which then run without an activation store, and the paper's 16-wide network). This file is
collected last so that a failure here does not hide the other tests in a run that stops at the first failure."""
import ctypes

import numpy as np
import pytest
import torch

import synthetic as S
from fgs_testutil import scene, to_dev, settings_for

pytestmark = pytest.mark.gpu


def _noalloc(F, dev_prims, settings, to_chw, clamp):
    from FasterGSVDACudaBackend import rasterization as R, _lib
    device = dev_prims['means'].device
    get = lambda k: dev_prims.get(k)
    cp = R._c_primitives(dev_prims['means'], dev_prims['scales'], dev_prims['rotations'], dev_prims['opacities'], get('precomputed_colors'),
                         get('base_colors'), get('residual_params'), get('mlp_weights'))
    cs, keep = R._c_settings(settings, device)
    h, w = settings.height, settings.width
    image = torch.full((3, h, w) if to_chw else (h, w, 3), float('nan'), device=device)
    nv, ni = ctypes.c_int64(0), ctypes.c_int64(0)
    _lib.check(_lib.lib.fgs_inference_noalloc(R._rasterizer.handle, ctypes.byref(cp), ctypes.byref(cs), image.data_ptr(), int(to_chw),
                                              int(clamp), torch.cuda.current_stream().cuda_stream, ctypes.byref(nv), ctypes.byref(ni)))
    torch.cuda.synchronize()
    return image, nv.value, ni.value


def _regular(F, p, settings, to_chw, clamp):
    return F.rasterize(p['means'], p['scales'], p['rotations'], p['opacities'], settings, to_chw, clamp,
                       precomputed_colors=p.get('precomputed_colors'), base_colors=p.get('base_colors'),
                       residual_params=p.get('residual_params'), mlp_weights=p.get('mlp_weights'))


def test_noalloc_matches_inference_twice(cuda):
    import FasterGSVDACudaBackend as F
    F.initialize_appearance('sh', 3, 'none', 'none', 'relu', True)
    for k, (n, W, H, to_chw, clamp) in enumerate(((20000, 256, 192, False, True), (12000, 200, 130, True, False))):
        prims = to_dev(scene('sh', n, 3, seed=11 + k, scale_shift=1.0), cuda)
        cam = S.ring_cameras(4, W, H)[k]
        settings = settings_for(F, cam, 3, cuda)
        ref = _regular(F, prims, settings, to_chw, clamp)
        got, nv, ni = _noalloc(F, prims, settings, to_chw, clamp)
        assert nv > 0 and ni > 0
        np.testing.assert_array_equal(got.cpu().numpy(), ref.cpu().numpy())


def test_noalloc_precomputed_colors_twice(cuda):
    import FasterGSVDACudaBackend as F
    F.initialize_appearance('sh', 3, 'none', 'none', 'relu', True)
    for k, (to_chw, clamp) in enumerate(((False, True), (True, False))):
        prims = to_dev(scene('precomputed', 15000, 3, seed=21 + k, scale_shift=1.0), cuda)
        settings = settings_for(F, S.ring_cameras(3, 224, 160)[k], 3, cuda)
        ref = _regular(F, prims, settings, to_chw, clamp)
        got, nv, ni = _noalloc(F, prims, settings, to_chw, clamp)
        assert nv > 0 and ni > 0
        np.testing.assert_array_equal(got.cpu().numpy(), ref.cpu().numpy())


@pytest.mark.parametrize('neurons,feat', [(64, 32), (16, 8)], ids=['tcgen05-64', 'mma-16'])
def test_noalloc_neural_twice(cuda, neurons, feat):
    """The Neural colour pass inside the static array (no activation store) matches the regular inference path, and
    the entry point reports no tensor-core timeout (it reads and clears the kernels' flag after the colour pass)."""
    import FasterGSVDACudaBackend as F
    from FasterGSVDACudaBackend._lib import lib
    n_in = feat * 2 + 16
    F.initialize_appearance('neural', 0, 'none', 'tanh', 'relu', True)
    F.initialize_residual_mlp(n_in, 3, {'otype': 'Identity'}, {'otype': 'FullyFusedMLP', 'activation': 'ReLU', 'output_activation': 'None',
                                                                'n_neurons': neurons, 'n_hidden_layers': 2}, False, 1, [0, 1, 2, 3])
    shapes = S.mlp_layer_shapes((n_in + 15) // 16 * 16, neurons, 2)
    for k, (to_chw, clamp) in enumerate(((False, True), (True, False))):
        n = 16000
        prims = {**S.geometry(n, seed=31 + k), **S.neural_appearance(n, feature_dim=feat, layer_shapes=shapes, seed=33 + k)}
        prims['scales'] = prims['scales'] + 1.0
        dev = to_dev(prims, cuda)
        settings = settings_for(F, S.ring_cameras(4, 240, 176)[k + 1], 3, cuda)
        ref = _regular(F, dev, settings, to_chw, clamp)
        got, nv, ni = _noalloc(F, dev, settings, to_chw, clamp)
        assert nv > 2 * 128 and ni > 0
        np.testing.assert_array_equal(got.cpu().numpy(), ref.cpu().numpy())
    flag = ctypes.c_int(7)
    assert lib.fgs_tc_timeout(ctypes.byref(flag), 0) == 0 and flag.value == 0


def test_noalloc_rejects_oversized_scene(cuda):
    import FasterGSVDACudaBackend as F
    F.initialize_appearance('sh', 3, 'none', 'none', 'relu', True)
    prims = to_dev(scene('sh', 400000, 3, seed=1), cuda)
    cam = S.ring_cameras(1, 640, 480)[0]
    with pytest.raises(RuntimeError, match='static maximum'):
        _noalloc(F, prims, settings_for(F, cam, 3, cuda), False, True)
