"""The deterministic exp / log used on both sides of the parity checks stay within a few ulp of the exact
functions, and the oracle's binning invariants hold (ranges partition the instance list, lists sorted by tile,
depth order inside a tile)."""
import numpy as np
import torch

import synthetic as S
from oracle import oracle as O
from fgs_testutil import scene


def test_det_exp_log_accuracy():
    lib = O.load(False)
    xs = np.concatenate([np.linspace(-86, 87, 20001), np.linspace(-6, 0, 5001)]).astype(np.float32)
    e = np.array([lib.orc_det_exp(float(x)) for x in xs], np.float64)
    ref = np.exp(xs.astype(np.float64))
    assert np.max(np.abs(e - ref) / ref) < 3e-7
    xb = np.linspace(-6, 0, 5001).astype(np.float32)
    eb = np.array([lib.orc_det_exp_blend(float(x)) for x in xb], np.float64)
    assert np.max(np.abs(eb - np.exp(xb.astype(np.float64))) / np.exp(xb.astype(np.float64))) < 5e-7
    ys = np.concatenate([np.geomspace(1e-30, 1e30, 20001), np.linspace(0.9, 300, 5001)]).astype(np.float32)
    lg = np.array([lib.orc_det_log(float(y)) for y in ys], np.float64)
    ref = np.log(ys.astype(np.float64))
    assert np.max(np.abs(lg - ref) / np.maximum(np.abs(ref), 1.0)) < 3e-7


def test_binning_invariants():
    n, W, H = 5000, 160, 120
    prims = scene('sh', n, 3, seed=2, scale_shift=1.0)
    cam = S.ring_cameras(2, W, H)[0]
    o = O.run(O.make_appearance('sh', 3, 0, 0, 1, True), O.make_view(cam, 3), prims)
    keys, ranks, ranges = o['tile_keys'], o['ranks'], o['ranges']
    assert np.all(np.diff(keys.astype(np.int64)) >= 0)
    for t in np.unique(keys):
        s, e = ranges[t]
        assert np.all(keys[s:e] == t)
        assert np.all(np.diff(ranks[s:e].astype(np.int64)) > 0)
    assert ranges[:, 1].max() == len(keys)
    assert o['n_instances'] == int(o['n_touched'].sum())
    d = o['depth_key'][o['sorted_idx']].view(np.float32)
    assert np.all(np.diff(d) >= 0)


def test_det_sincos_error_bound():
    """The oracle's deterministic sine / cosine of the Neural encoding (Cody-Waite reduction + Taylor series) against
    double-precision libm: at most 2.5e-7 absolute error on [-8192, 8192] and at the quadrant boundaries; arguments
    beyond are clamped to +-8192 (as the kernels do)."""
    import ctypes
    lib = O.load(False)
    rng = np.random.default_rng(0)
    xs = np.concatenate([rng.normal(0, 0.1, 20000), rng.uniform(-10, 10, 20000), rng.uniform(-8192, 8192, 20000),
                         (np.arange(-64, 65) * np.pi / 4), [0.0, -0.0, 1e-30, 8192.0, -8192.0]]).astype(np.float32)
    s, c = ctypes.c_float(), ctypes.c_float()
    worst = 0.0
    for x in xs:
        lib.orc_det_sincos(ctypes.c_float(x), ctypes.byref(s), ctypes.byref(c))
        worst = max(worst, abs(s.value - np.sin(np.float64(x))), abs(c.value - np.cos(np.float64(x))))
    assert worst <= 2.5e-7, worst
    s2, c2 = ctypes.c_float(), ctypes.c_float()
    lib.orc_det_sincos(ctypes.c_float(9000.0), ctypes.byref(s), ctypes.byref(c))
    lib.orc_det_sincos(ctypes.c_float(8192.0), ctypes.byref(s2), ctypes.byref(c2))
    assert (s.value, c.value) == (s2.value, c2.value)
