"""The allocation-free inference entry point (fgs_inference_noalloc) renders the same image as the regular
inference path, on two calls in a row (the second call must not see stale state from the first).

Callers of that entry point are render hooks that cannot allocate device memory mid-frame (a host application
owns the device-memory budget); the entry point keeps its workspaces in a static device array instead. This file
is collected last so that a failure here does not hide the other tests in a run that stops at the first failure."""
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
    cp = R._c_primitives(dev_prims['means'], dev_prims['scales'], dev_prims['rotations'], dev_prims['opacities'], None,
                         dev_prims['base_colors'], dev_prims['residual_params'], None)
    cs, keep = R._c_settings(settings, device)
    h, w = settings.height, settings.width
    image = torch.full((3, h, w) if to_chw else (h, w, 3), float('nan'), device=device)
    nv, ni = ctypes.c_int64(0), ctypes.c_int64(0)
    _lib.check(_lib.lib.fgs_inference_noalloc(R._rasterizer.handle, ctypes.byref(cp), ctypes.byref(cs), image.data_ptr(), int(to_chw),
                                              int(clamp), torch.cuda.current_stream().cuda_stream, ctypes.byref(nv), ctypes.byref(ni)))
    torch.cuda.synchronize()
    return image, nv.value, ni.value


def test_noalloc_matches_inference_twice(cuda):
    import FasterGSVDACudaBackend as F
    F.initialize_appearance('sh', 3, 'none', 'none', 'relu', True)
    for k, (n, W, H, to_chw, clamp) in enumerate(((20000, 256, 192, False, True), (12000, 200, 130, True, False))):
        prims = to_dev(scene('sh', n, 3, seed=11 + k, scale_shift=1.0), cuda)
        cam = S.ring_cameras(4, W, H)[k]
        settings = settings_for(F, cam, 3, cuda)
        ref = F.rasterize(prims['means'], prims['scales'], prims['rotations'], prims['opacities'], settings, to_chw, clamp,
                          base_colors=prims['base_colors'], residual_params=prims['residual_params'])
        got, nv, ni = _noalloc(F, prims, settings, to_chw, clamp)
        assert nv > 0 and ni > 0
        np.testing.assert_array_equal(got.cpu().numpy(), ref.cpu().numpy())


def test_noalloc_rejects_oversized_scene(cuda):
    import FasterGSVDACudaBackend as F
    F.initialize_appearance('sh', 3, 'none', 'none', 'relu', True)
    prims = to_dev(scene('sh', 400000, 3, seed=1), cuda)
    cam = S.ring_cameras(1, 640, 480)[0]
    with pytest.raises(RuntimeError, match='static maximum'):
        _noalloc(F, prims, settings_for(F, cam, 3, cuda), False, True)
