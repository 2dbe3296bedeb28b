"""CPU restatement of the training-loop helpers around the rasterizer (TEST INFRASTRUCTURE ONLY: imported by tests/,
never by the product path): 3DGS-MCMC relocation and position noise, and the 3D filter update.

Follows FasterGSVDACudaBackend/FasterGSVDACudaBackend/densification/include/kernels_mcmc.cuh (relocation :10-54,
Box-Muller :74-80, noise :82-146) and filter3d/src/filter3d.cu:11-73. The relocation and the noise are evaluated in
double; the 3D filter in float32 with the kernel's operation order, so it matches bit for bit. The noise draws its
normals from Philox4x32-10 (Salmon, Moraes, Dror, Shaw, "Parallel random numbers: as easy as 1, 2, 3", SC 2011),
restated here from the published algorithm: ten rounds of two 32x32->64-bit multiplies whose high halves are mixed
into the other words with the round key, the key advancing by the Weyl constants between rounds.
"""
from __future__ import annotations

import math

import numpy as np

MAX_SAMPLES = 50
_M0, _M1 = np.uint64(0xD2511F53), np.uint64(0xCD9E8D57)
_W0, _W1 = np.uint64(0x9E3779B9), np.uint64(0xBB67AE85)
_MASK = np.uint64(0xFFFFFFFF)


def relocation(old_opacity: np.ndarray, old_scale: np.ndarray, n_samples: np.ndarray) -> tuple[np.ndarray, np.ndarray]:
    """(new opacity [M], new scales [M,3]) in double: p = 1 - (1 - o)^(1/N), scales * o / sum_{n<N} sum_{k<=n}
    C(n,k) (-1)^k p^(k+1) / sqrt(k+1), with N clamped to [1, 50] (kernels_mcmc.cuh:10-54)."""
    o = np.asarray(old_opacity, np.float64).reshape(-1)
    sc = np.asarray(old_scale, np.float64).reshape(-1, 3)
    N = np.clip(np.asarray(n_samples).reshape(-1), 1, MAX_SAMPLES).astype(np.int64)
    p = 1.0 - np.power(1.0 - o, 1.0 / N)
    denom = np.zeros_like(o)
    for i in range(o.size):
        acc = 0.0
        for n in range(int(N[i])):
            for k in range(n + 1):
                acc += math.comb(n, k) * (-1.0) ** k / math.sqrt(k + 1) * p[i] ** (k + 1)
        denom[i] = acc
    return p, sc * (o / denom)[:, None]


def philox4x32_10(c: list[np.ndarray], key: tuple[int, int]) -> list[np.ndarray]:
    """Philox4x32-10 of counters c = [c0, c1, c2, c3] (uint32 arrays) under key (k0, k1); returns four uint32 arrays."""
    c = [np.asarray(x, np.uint64) & _MASK for x in c]
    k0, k1 = np.uint64(key[0]) & _MASK, np.uint64(key[1]) & _MASK
    for r in range(10):
        if r > 0:
            k0, k1 = (k0 + _W0) & _MASK, (k1 + _W1) & _MASK
        p0, p1 = _M0 * c[0], _M1 * c[2]
        hi0, lo0 = p0 >> np.uint64(32), p0 & _MASK
        hi1, lo1 = p1 >> np.uint64(32), p1 & _MASK
        c = [hi1 ^ c[1] ^ k0, lo1, hi0 ^ c[3] ^ k1, lo0]
    return [x.astype(np.uint32) for x in c]


def box_muller(bu: np.ndarray, bv: np.ndarray) -> tuple[np.ndarray, np.ndarray]:
    """Two standard normals from two uint32 arrays: u = (bu + 1/2) / 2^32 in (0, 1], angle = bv * 2 pi / 2^32."""
    u = (bu.astype(np.float64) + 0.5) / 4294967296.0
    radius = np.sqrt(-2.0 * np.log(u))
    ang = bv.astype(np.float64) * (2.0 * math.pi / 4294967296.0)
    return radius * np.cos(ang), radius * np.sin(ang)


def add_noise(raw_scales, raw_rotations, raw_opacities, means, lr: float, seed: int, offset: int) -> np.ndarray:
    """Means [N,3] after the MCMC noise step in double (kernels_mcmc.cuh:82-146); degenerate quaternions unchanged."""
    s = np.asarray(raw_scales, np.float64).reshape(-1, 3)
    q = np.asarray(raw_rotations, np.float64).reshape(-1, 4)
    op = np.asarray(raw_opacities, np.float64).reshape(-1)
    m = np.asarray(means, np.float64).reshape(-1, 3).copy()
    n = m.shape[0]
    ctr = offset // 4
    idx = np.arange(n, dtype=np.uint64)
    bits = philox4x32_10([np.full(n, ctr & 0xFFFFFFFF, np.uint64), np.full(n, ctr >> 32, np.uint64), idx, np.zeros(n, np.uint64)],
                         (seed & 0xFFFFFFFF, (seed >> 32) & 0xFFFFFFFF))
    z0, z1 = box_muller(bits[0], bits[1])
    z2, _ = box_muller(bits[2], bits[3])
    z = np.stack([z0, z1, z2], axis=1)
    r, x, y, w = q[:, 0], q[:, 1], q[:, 2], q[:, 3]
    nsq = r * r + x * x + y * y + w * w
    ok = nsq >= 1e-8
    inv = np.where(ok, 1.0 / np.where(ok, nsq, 1.0), 0.0)
    R = np.empty((n, 3, 3))
    R[:, 0, 0] = 1 - 2 * (y * y + w * w) * inv; R[:, 0, 1] = 2 * (x * y - r * w) * inv; R[:, 0, 2] = 2 * (x * w + r * y) * inv
    R[:, 1, 0] = 2 * (x * y + r * w) * inv; R[:, 1, 1] = 1 - 2 * (x * x + w * w) * inv; R[:, 1, 2] = 2 * (y * w - r * x) * inv
    R[:, 2, 0] = 2 * (x * w - r * y) * inv; R[:, 2, 1] = 2 * (y * w + r * x) * inv; R[:, 2, 2] = 1 - 2 * (x * x + y * y) * inv
    cov = np.einsum('nij,nj,nkj->nik', R, np.exp(2.0 * s), R)
    o = 1.0 / (1.0 + np.exp(-op))
    factor = lr / (1.0 + np.exp(100.0 * o - 0.5))
    m[ok] += (factor[:, None] * np.einsum('nij,nj->ni', cov, z))[ok]
    return m


def filter3d(positions, w2c, filter_3d, visible, width: int, height: int, fx: float, fy: float, cx: float, cy: float, near: float,
             far: float, clipping_tolerance: float, distance2filter: float) -> tuple[np.ndarray, np.ndarray]:
    """(filter, visibility) after one view's update, float32 in the kernel's operation order (filter3d.cu:11-73)."""
    f32 = np.float32
    P = np.asarray(positions, f32).reshape(-1, 3)
    M = np.asarray(w2c, f32).reshape(4, 4)
    flt = np.asarray(filter_3d, f32).copy()
    vis = np.asarray(visible, bool).copy()
    b = f32(clipping_tolerance) + f32(0.5)
    w, h = f32(width), f32(height)
    ox, oy = f32(cx) - f32(0.5) * w, f32(cy) - f32(0.5) * h
    left, right = (-(b * w) - ox) / f32(fx), (b * w - ox) / f32(fx)
    top, bottom = (-(b * h) - oy) / f32(fy), (b * h - oy) / f32(fy)

    def row(i):
        return ((M[i, 0] * P[:, 0] + M[i, 1] * P[:, 1]) + M[i, 2] * P[:, 2]) + M[i, 3]

    z, xc, yc = row(2), row(0), row(1)
    inside = (z >= f32(near)) & (z <= f32(far)) & (xc >= left * z) & (xc <= right * z) & (yc >= top * z) & (yc <= bottom * z)
    new = f32(distance2filter) * z
    upd = inside & ~(flt < new)
    flt[upd] = new[upd]
    vis[upd] = True
    return flt, vis
