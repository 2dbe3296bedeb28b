"""GPU parity of the training-loop helpers against the oracle (oracle/densification.py): MCMC relocation
(relocation_adjustment, kernels_mcmc.cuh:10-54) within 1e-5 relative on opacities and 1e-4 on scales, MCMC position
noise (add_noise, kernels_mcmc.cuh:64-146) with the same Philox seed and offset within 1e-4 relative on the
increments beyond the float32 rounding of the means (the generator offset advances by 4, degenerate quaternions stay unchanged), and the 3D filter update
(update_3d_filter, filter3d.cu:11-90) bit for bit."""
import numpy as np
import pytest
import torch

import synthetic as S
from oracle import densification as D

pytestmark = pytest.mark.gpu


def test_relocation_matches_oracle(cuda):
    import FasterGSVDACudaBackend as F
    g = torch.Generator().manual_seed(0)
    m = 5000
    o = torch.rand(m, 1, generator=g) * 0.98 + 0.01
    sc = torch.exp(torch.randn(m, 3, generator=g) * 0.5 - 3.0)
    n = torch.randint(1, 13, (m,), generator=g, dtype=torch.int64)
    po, ps = F.relocation_adjustment(o.to(cuda), sc.to(cuda), n.to(cuda))
    ro, rs = D.relocation(o.numpy(), sc.numpy(), n.numpy())
    np.testing.assert_allclose(po.cpu().numpy().reshape(-1), ro, rtol=1e-5, atol=1e-7)
    np.testing.assert_allclose(ps.cpu().numpy(), rs, rtol=1e-4)
    # counts are clamped to 1..50
    big = F.relocation_adjustment(o[:64].to(cuda), sc[:64].to(cuda), torch.full((64,), 80, dtype=torch.int64, device=cuda))
    cap = F.relocation_adjustment(o[:64].to(cuda), sc[:64].to(cuda), torch.full((64,), 50, dtype=torch.int64, device=cuda))
    zero = F.relocation_adjustment(o[:64].to(cuda), sc[:64].to(cuda), torch.zeros(64, dtype=torch.int64, device=cuda))
    assert torch.equal(big[0], cap[0]) and torch.equal(big[1], cap[1])
    # a count of 0 acts as 1: a single copy keeps its opacity (up to the rounding of 1 - (1 - o)) and its scales
    assert torch.allclose(zero[0].cpu(), o[:64], rtol=0, atol=1e-7) and torch.allclose(zero[1].cpu(), sc[:64], rtol=1e-6)


def test_add_noise_matches_oracle(cuda):
    import FasterGSVDACudaBackend as F
    g = torch.Generator().manual_seed(1)
    n = 20000
    raw_s = torch.randn(n, 3, generator=g) * 0.5 - 3.0
    raw_r = torch.randn(n, 4, generator=g)
    raw_r[:50] = 0.0  # degenerate quaternions: left unchanged
    raw_o = torch.randn(n, 1, generator=g) - 6.0
    means = torch.randn(n, 3, generator=g) * 3.0
    dev = {k: v.to(cuda).contiguous() for k, v in dict(s=raw_s, r=raw_r, o=raw_o, m=means).items()}
    torch.cuda.manual_seed(1234)
    gen = torch.cuda.default_generators[cuda.index if cuda.index is not None else torch.cuda.current_device()]
    seed, offset = gen.initial_seed(), gen.get_offset()
    F.add_noise(dev['s'], dev['r'], dev['o'], dev['m'], 0.02)
    assert gen.get_offset() == offset + 4
    got = dev['m'].cpu().numpy().astype(np.float64)
    ref = D.add_noise(raw_s.numpy(), raw_r.numpy(), raw_o.numpy(), means.numpy(), 0.02, seed, offset)
    np.testing.assert_array_equal(got[:50], means.numpy()[:50])
    d_got, d_ref = got - means.numpy(), ref - means.numpy()
    assert np.abs(d_ref).max() > 1e-4
    # the float32 means round the sum to a few ulp of the mean; beyond that the increments agree to 1e-4
    eps = np.finfo(np.float32).eps
    assert np.all(np.abs(got - ref) <= 2 * eps * np.abs(ref) + 1e-4 * np.abs(d_ref) + 1e-12)
    assert abs(np.linalg.norm(d_got) - np.linalg.norm(d_ref)) / np.linalg.norm(d_ref) <= 1e-4
    # a second call draws new numbers
    F.add_noise(dev['s'], dev['r'], dev['o'], dev['m'], 0.02)
    assert not np.allclose(dev['m'].cpu().numpy() - got, d_got)


def test_update_3d_filter_matches_oracle_bitwise(cuda):
    import FasterGSVDACudaBackend as F
    g = torch.Generator().manual_seed(2)
    n = 30000
    pos = torch.randn(n, 3, generator=g) * 5.0
    flt = torch.rand(n, generator=g) * 0.05
    flt[::4] = float('inf')
    vis = torch.zeros(n, dtype=torch.bool)
    cam = S.ring_cameras(4, 640, 480)[1]
    flt_d, vis_d = flt.to(cuda), vis.to(cuda)
    F.update_3d_filter(pos.to(cuda), cam.w2c.to(cuda), flt_d, vis_d, cam.width, cam.height, cam.focal_x, cam.focal_y, cam.center_x,
                       cam.center_y, cam.near_plane, cam.far_plane, 0.15, 0.001)
    rf, rv = D.filter3d(pos.numpy(), cam.w2c.numpy(), flt.numpy(), vis.numpy(), cam.width, cam.height, cam.focal_x, cam.focal_y,
                        cam.center_x, cam.center_y, cam.near_plane, cam.far_plane, 0.15, 0.001)
    np.testing.assert_array_equal(flt_d.cpu().numpy(), rf)
    np.testing.assert_array_equal(vis_d.cpu().numpy(), rv)
    assert rv.sum() > 1000


def _spread3(x):
    out = np.zeros_like(x, dtype=np.uint64)
    for b in range(21):
        out |= ((x >> np.uint64(b)) & np.uint64(1)) << np.uint64(3 * b)
    return out


def test_morton_codes_and_reordering(cuda):
    import FasterGSVDACudaBackend as F
    from trainer import morton_order, Trainer
    g = torch.Generator().manual_seed(3)
    n = 50000
    means = torch.randn(n, 3, generator=g) * torch.tensor([4.0, 1.0, 9.0])
    order = morton_order(means.to(cuda)).cpu().numpy()
    # codes restated: 21 bits per axis over the bounding box (float32 as the kernel), interleaved x lowest
    m = means.numpy()
    lo, hi = m.min(0), m.max(0)
    q = np.empty((n, 3), np.uint64)
    for a in range(3):
        scale = np.float32(2097152.0) / (np.float32(hi[a]) - np.float32(lo[a]))
        v = (m[:, a].astype(np.float32) - np.float32(lo[a])) * scale
        q[:, a] = np.clip(np.floor(v), 0, 2097151).astype(np.uint64)
    codes = _spread3(q[:, 0]) | (_spread3(q[:, 1]) << np.uint64(1)) | (_spread3(q[:, 2]) << np.uint64(2))
    np.testing.assert_array_equal(order, np.argsort(codes, kind='stable'))
    # the trainer permutes every per-Gaussian group (and its moments) by that order; the MLP weights stay
    F.initialize_appearance('sh', 3, 'none', 'none', 'relu', True)
    prims = {'means': means, 'scales': torch.randn(n, 3, generator=g) - 4.0, 'rotations': torch.randn(n, 4, generator=g),
             'opacities': torch.randn(n, 1, generator=g), 'base_colors': torch.randn(n, 3, generator=g),
             'residual_params': torch.randn(n, 45, generator=g)}
    lrs = {k: 1e-3 for k in prims}
    tr = Trainer({k: v.to(cuda) for k, v in prims.items()}, lrs, cuda)
    tr.exp_avg.copy_(torch.arange(tr.shard, dtype=torch.float32, device=cuda))
    before = tr.exp_avg.clone()
    tr.apply_morton_ordering()
    for k, v in prims.items():
        assert torch.equal(tr.view(tr.params, k).cpu(), v[order])
        gi = next(x for x in tr.groups if x.name == k)
        moved = before[gi.offset:gi.offset + gi.numel].view(n, -1)[torch.from_numpy(order).to(cuda)]
        assert torch.equal(tr.exp_avg[gi.offset:gi.offset + gi.numel].view(n, -1), moved)
