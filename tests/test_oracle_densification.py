"""Invariants of the oracle's training-loop helpers (oracle/densification.py): the MCMC relocation keeps the
composite opacity of the N copies and leaves a single copy unchanged (kernels_mcmc.cuh:10-54), the restated
Philox4x32-10 bits and Box-Muller normals have the moments of uniform bits and standard normals, and the 3D filter
update takes min(filter, distance2filter * depth) exactly for the points inside the widened frustum."""
import numpy as np

from oracle import densification as D


def test_relocation_keeps_composite_opacity():
    rng = np.random.default_rng(0)
    o = rng.uniform(0.01, 0.99, 400)
    sc = np.exp(rng.normal(-3.0, 0.5, (400, 3)))
    n = rng.integers(1, 12, 400)
    p, s = D.relocation(o, sc, n)
    np.testing.assert_allclose(1.0 - (1.0 - p) ** n, o, rtol=1e-12)
    one = n == 1
    np.testing.assert_allclose(p[one], o[one], rtol=1e-14)
    np.testing.assert_allclose(s[one], sc[one], rtol=1e-12)
    assert np.all(s[~one] > 0) and np.all(np.isfinite(s))
    # counts above the maximum behave as the maximum
    p60, s60 = D.relocation(o[:5], sc[:5], np.full(5, 60))
    p50, s50 = D.relocation(o[:5], sc[:5], np.full(5, 50))
    np.testing.assert_array_equal(p60, p50)
    np.testing.assert_array_equal(s60, s50)


def test_philox_bits_and_normals_have_the_expected_moments():
    n = 200000
    idx = np.arange(n, dtype=np.uint64)
    zero = np.zeros(n, np.uint64)
    bits = D.philox4x32_10([zero + 7, zero, idx, zero], (0x1234ABCD, 0x0BADF00D))
    for b in bits:
        u = b.astype(np.float64) / 2.0 ** 32
        assert abs(u.mean() - 0.5) < 0.005 and abs(u.var() - 1.0 / 12.0) < 0.002
    assert len(np.unique(bits[0])) > n * 0.99  # distinct counters give distinct words
    z0, z1 = D.box_muller(bits[0], bits[1])
    for z in (z0, z1):
        assert abs(z.mean()) < 0.01 and abs(z.var() - 1.0) < 0.02
    assert abs(np.mean(z0 * z1)) < 0.01


def test_filter3d_takes_the_minimum_inside_the_frustum():
    rng = np.random.default_rng(1)
    P = rng.normal(0.0, 4.0, (5000, 3)).astype(np.float32)
    w2c = np.eye(4, dtype=np.float32)
    w2c[2, 3] = 10.0
    flt0 = np.full(5000, 0.01, np.float32)
    flt0[::3] = 1e9
    vis0 = np.zeros(5000, bool)
    flt, vis = D.filter3d(P, w2c, flt0, vis0, 640, 480, 500.0, 500.0, 320.0, 240.0, 0.2, 1e4, 0.15, 0.002)
    z = P[:, 2] + 10.0
    inside = (np.abs(P[:, 0] / z) <= 0.65 * 640 / 500) & (np.abs(P[:, 1] / z) <= 0.65 * 480 / 500) & (z > 0.2)
    strict = inside & (np.abs(np.abs(P[:, 0] / z) - 0.65 * 640 / 500) > 1e-4) & (np.abs(np.abs(P[:, 1] / z) - 0.65 * 480 / 500) > 1e-4)
    want = np.where(inside & (0.002 * z <= flt0), 0.002 * z, flt0)
    np.testing.assert_allclose(flt[strict], want[strict], rtol=1e-6)
    assert vis[strict].tolist() == (inside & (0.002 * z <= flt0))[strict].tolist()
    assert vis.sum() > 100 and (~vis).sum() > 100
