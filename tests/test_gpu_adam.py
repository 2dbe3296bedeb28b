"""FusedAdam on the GPU against the oracle restatement of adam.cu (bit-exact: same float operations), including the
per-column learning-rate cycle of the spherical Voronoi layout and per-group betas."""
import numpy as np
import pytest
import torch

from oracle import oracle as O

pytestmark = pytest.mark.gpu


def test_fused_adam_bit_exact(cuda):
    import FasterGSVDACudaBackend as F
    g = torch.Generator().manual_seed(0)
    shapes = [(1000, 3), (1000, 4), (1000, 1), (500, 8, 7), (2384,)]
    params = [torch.randn(*s, generator=g) for s in shapes]
    lrs = [1.6e-4, 0.001, 0.05, [0.002] * 3 + [0.006] + [0.0008] * 3, 0.003]
    betas = [(0.9, 0.999)] * 4 + [(0.9, 0.99)]
    dev = [torch.nn.Parameter(p.clone().to(cuda)) for p in params]
    opt = F.FusedAdam([{'params': [p], 'lr': lr, 'betas': b} for p, lr, b in zip(dev, lrs, betas)], lr=0.0, eps=1e-15)
    ref = [p.numpy().copy() for p in params]
    m = [np.zeros_like(r) for r in ref]
    v = [np.zeros_like(r) for r in ref]
    for step in range(1, 4):
        grads = [torch.randn(*s, generator=g) for s in shapes]
        for p, gr in zip(dev, grads):
            p.grad = gr.to(cuda)
        opt.step()
        for i in range(len(ref)):
            O.adam(ref[i].reshape(-1), grads[i].numpy().reshape(-1).copy(), m[i].reshape(-1), v[i].reshape(-1), step, lrs[i], betas[i], 1e-15)
    for p, r in zip(dev, ref):
        np.testing.assert_array_equal(p.detach().cpu().numpy(), r)
