"""3DGS-MCMC helpers, drop-in for FasterGSVDACudaBackend/FasterGSVDACudaBackend/torch_bindings/densification.py:6-21
(kernels: densification/include/kernels_mcmc.cuh; here csrc/densification.cu behind fgs_relocation_adjustment and
fgs_add_noise)."""
import torch

from ._lib import lib, check


def _need(t: torch.Tensor, name: str, dtype=torch.float32) -> None:
    if not t.is_cuda or t.dtype != dtype or not t.is_contiguous():
        raise RuntimeError(f'{name} must be a contiguous CUDA {dtype} tensor')


def relocation_adjustment(
    old_opacities: torch.Tensor,
    old_scales: torch.Tensor,
    n_samples_per_primitive: torch.Tensor,
) -> tuple[torch.Tensor, torch.Tensor]:
    """Opacities [M,1] and scales [M,3] (activated) of primitives duplicated into n_samples_per_primitive[i] copies
    (int64, clamped to 1..50): returns the adjusted (new_opacities [M,1], new_scales [M,3])."""
    old_opacities = old_opacities.contiguous()
    old_scales = old_scales.contiguous()
    n_samples = n_samples_per_primitive.contiguous()
    _need(old_opacities, 'old_opacities')
    _need(old_scales, 'old_scales')
    _need(n_samples, 'n_samples_per_primitive', torch.int64)
    m = old_opacities.shape[0]
    if old_opacities.numel() != m or old_scales.numel() != 3 * m or n_samples.numel() != m:
        raise ValueError('expected opacities [M,1], scales [M,3] and sample counts [M]')
    new_opacities = torch.empty((m, 1), dtype=torch.float32, device=old_opacities.device)
    new_scales = torch.empty((m, 3), dtype=torch.float32, device=old_opacities.device)
    check(lib.fgs_relocation_adjustment(old_opacities.data_ptr(), old_scales.data_ptr(), n_samples.data_ptr(), new_opacities.data_ptr(),
                                        new_scales.data_ptr(), m, torch.cuda.current_stream(old_opacities.device).cuda_stream))
    return new_opacities, new_scales


def add_noise(
    raw_scales: torch.Tensor,
    raw_rotations: torch.Tensor,
    raw_opacities: torch.Tensor,
    means: torch.Tensor,
    current_lr: float,
) -> None:
    """Adds the MCMC position noise to `means` [N,3] in place. Like the reference, the Philox seed and offset come from
    torch's default CUDA generator of the device, whose offset advances by 4 per call."""
    for t, name in ((raw_scales, 'raw_scales'), (raw_rotations, 'raw_rotations'), (raw_opacities, 'raw_opacities'), (means, 'means')):
        _need(t, name)
    n = means.shape[0]
    if raw_scales.numel() != 3 * n or raw_rotations.numel() != 4 * n or raw_opacities.numel() != n or means.numel() != 3 * n:
        raise ValueError('expected scales [N,3], rotations [N,4], opacities [N,1] and means [N,3]')
    index = means.device.index if means.device.index is not None else torch.cuda.current_device()
    gen = torch.cuda.default_generators[index]
    seed, offset = gen.initial_seed(), gen.get_offset()
    gen.set_offset(offset + 4)
    check(lib.fgs_add_noise(raw_scales.data_ptr(), raw_rotations.data_ptr(), raw_opacities.data_ptr(), means.data_ptr(), n, float(current_lr),
                            seed & 0xFFFFFFFFFFFFFFFF, offset, torch.cuda.current_stream(means.device).cuda_stream))
