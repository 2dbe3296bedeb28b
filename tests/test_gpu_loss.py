"""Fused L1 + DSSIM loss (fgs_l1_dssim) against its PyTorch fp32 definition (trainer.loss_and_grad_reference)."""
import pytest
import torch

from trainer import FusedLoss, loss_and_grad_reference, blur


@pytest.mark.gpu
@pytest.mark.parametrize('shape', [(3, 64, 64), (3, 97, 131), (1, 5, 7), (3, 270, 480)])
def test_fused_loss_matches_torch(cuda, shape):
    g = torch.Generator().manual_seed(7)
    img = torch.rand(shape, generator=g)
    tgt = blur(torch.rand(shape, generator=g), 9, 2.0).contiguous() if min(shape[1:]) >= 9 else torch.rand(shape, generator=g)
    ref_loss, ref_grad = loss_and_grad_reference(img.double(), tgt.double())
    loss, grad = FusedLoss()(img.to(cuda), tgt.to(cuda))
    torch.cuda.synchronize()
    # tolerance: fp32 sums in a different order than the float64 evaluation of the same definition
    assert abs(float(loss) - float(ref_loss)) <= 1e-5 * max(1.0, abs(float(ref_loss)))
    grad = grad.cpu().double()
    rel = (grad - ref_grad).norm() / ref_grad.norm()
    assert rel < 1e-4, float(rel)
    assert (grad - ref_grad).abs().max() <= 1e-3 * ref_grad.abs().max()


@pytest.mark.gpu
def test_fused_loss_deterministic_and_identical_inputs(cuda):
    g = torch.Generator().manual_seed(8)
    img = torch.rand((3, 120, 200), generator=g).to(cuda)
    fl = FusedLoss()
    l1, g1 = fl(img, img.clone())
    assert abs(float(l1)) < 1e-6  # SSIM(x, x) = 1 and L1 = 0
    tgt = torch.rand((3, 120, 200), generator=g).to(cuda)
    a, ga = fl(img, tgt)
    b, gb = fl(img, tgt)
    assert float(a) == float(b) and torch.equal(ga, gb)


def test_fused_loss_rejects_cpu_tensors():
    with pytest.raises(RuntimeError):
        FusedLoss()(torch.zeros(3, 8, 8), torch.zeros(3, 8, 8))
