"""3D filter update, drop-in for FasterGSVDACudaBackend/FasterGSVDACudaBackend/torch_bindings/filter3d.py:6-40
(kernel: filter3d/src/filter3d.cu; here csrc/densification.cu behind fgs_update_3d_filter)."""
import torch

from ._lib import lib, check


def update_3d_filter(
    positions: torch.Tensor,
    w2c: torch.Tensor,
    filter_3d: torch.Tensor,
    visibility_mask: torch.Tensor,
    width: int,
    height: int,
    focal_x: float,
    focal_y: float,
    center_x: float,
    center_y: float,
    near_plane: float,
    far_plane: float,
    clipping_tolerance: float,
    distance2filter: float,
) -> None:
    """For the points [N,3] inside the view's frustum (widened by clipping_tolerance), filter_3d [N] becomes
    min(filter_3d, distance2filter * depth) and visibility_mask [N] (bool) is set; both updated in place."""
    n = positions.shape[0]
    for t, name, dt in ((positions, 'positions', torch.float32), (filter_3d, 'filter_3d', torch.float32), (visibility_mask, 'visibility_mask', torch.bool)):
        if not t.is_cuda or t.dtype != dt or not t.is_contiguous():
            raise RuntimeError(f'{name} must be a contiguous CUDA {dt} tensor')
    if positions.numel() != 3 * n or filter_3d.numel() != n or visibility_mask.numel() != n:
        raise ValueError('expected positions [N,3], filter_3d [N] and visibility_mask [N]')
    m = w2c.to(device=positions.device, dtype=torch.float32).contiguous()
    if m.numel() != 16:
        raise ValueError('w2c must hold a 4x4 matrix')
    if m.data_ptr() % 16 != 0:
        m = m.clone()
    check(lib.fgs_update_3d_filter(positions.data_ptr(), m.data_ptr(), filter_3d.data_ptr(), visibility_mask.data_ptr(), n, int(width), int(height),
                                   float(focal_x), float(focal_y), float(center_x), float(center_y), float(near_plane), float(far_plane),
                                   float(clipping_tolerance), float(distance2filter), torch.cuda.current_stream(positions.device).cuda_stream))
