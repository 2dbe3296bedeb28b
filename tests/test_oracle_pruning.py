"""Pins the oracle's pruning scores (oracle/fgs_oracle.c orc_pruning_scores, following
rasterization/include/kernels_pruning_scores.cuh:11-173) against an independent derivation: for every pixel, the
accepted fragments' alphas become autograd leaves of the composited colour sum (background included), and the
score of a primitive is the sum over its fragments of (opacity * dL/dalpha)^2."""
import numpy as np
import torch

import synthetic as S
from oracle import oracle as O
from fgs_testutil import scene


def test_pruning_scores_match_autograd_of_the_blend():
    n, W, H = 200, 48, 36
    prims = {k: v.double().numpy() for k, v in scene('sh', n, 3, seed=0, scale_shift=2.5).items()}
    cam = S.look_at(torch.tensor([0.0, 0.0, 12.0]), W, H)
    v = O.make_view(cam, 3)
    v.bg[0], v.bg[1], v.bg[2] = 0.25, 0.5, 0.75
    a = O.make_appearance('sh', 3, 0, 0, 1, True)
    out = O.run(a, v, prims, double=True, pruning=True)
    rec, ranks, ranges, sidx, ncon = out['records'], out['ranks'], out['ranges'], out['sorted_idx'], out['n_contrib']
    bg = torch.tensor([0.25, 0.5, 0.75], dtype=torch.float64)
    gw = (W + 15) // 16
    ref = np.zeros(n)
    for py in range(H):
        for px in range(W):
            tile = (py // 12) * gw + px // 16
            sx0 = (px // 16) * 16 + ((px % 16) // 8) * 8
            sy0 = (py // 12) * 12 + ((py % 12) // 4) * 4
            s = int(ranges[tile, 0])
            frags = []
            for j in range(s, s + int(ncon[py, px])):
                pi = int(sidx[ranks[j]])
                o = rec[pi]
                if not (o[10] < sx0 + 8 and sx0 < o[11] and o[12] < sy0 + 4 and sy0 < o[13]):
                    continue
                dx, dy = o[0] - (px + 0.5), o[1] - (py + 0.5)
                e = -0.5 * (o[4] * dx * dx + o[6] * dy * dy) - o[5] * dx * dy
                if e < -o[3]:
                    continue
                frags.append((pi, o[2] * np.exp(min(e, 0.0))))
            if not frags:
                continue
            alphas = torch.tensor([f[1] for f in frags], dtype=torch.float64, requires_grad=True)
            T = torch.ones((), dtype=torch.float64)
            C = torch.zeros(3, dtype=torch.float64)
            for k, (pi, _) in enumerate(frags):
                C = C + T * alphas[k] * torch.from_numpy(rec[pi, 7:10])
                T = T * (1.0 - alphas[k])
            L = (C + T * bg).sum()
            (g,) = torch.autograd.grad(L, alphas)
            for k, (pi, _) in enumerate(frags):
                ref[pi] += (rec[pi, 2] * float(g[k])) ** 2
    got = out['pruning_scores']
    assert (ref > 0).sum() > 50
    np.testing.assert_allclose(got, ref, rtol=1e-9, atol=1e-12)
