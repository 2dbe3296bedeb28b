"""Fused Adam, drop-in for FasterGSVDACudaBackend/FasterGSVDACudaBackend/torch_bindings/adam.py:6-36.

A torch.optim.Adam subclass whose step() updates every single-tensor parameter group in one kernel launch (up to
12 groups per launch). group['lr'] may be a float or a list of at most 7 floats cycled over the elements
(per-column learning rates); per-group 'betas' and 'eps' are honoured; bias corrections use the group's step count.
"""
import ctypes

import torch

from . import _lib
from ._lib import lib, check


def _segment(param: torch.Tensor, grad: torch.Tensor, exp_avg: torch.Tensor, exp_avg_sq: torch.Tensor, step: int, lr, betas, eps: float,
             column_offset: int = 0) -> _lib.AdamSegment:
    lrs = list(lr) if isinstance(lr, (list, tuple)) else [lr]
    if not 1 <= len(lrs) <= 7:
        raise RuntimeError('between 1 and 7 learning rates are supported')
    for t, name in ((param, 'param'), (grad, 'grad'), (exp_avg, 'exp_avg'), (exp_avg_sq, 'exp_avg_sq')):
        if t.dtype != torch.float32 or not t.is_contiguous() or t.device != param.device or t.numel() != param.numel():
            raise RuntimeError(f'{name} must be a contiguous float32 tensor on the device and of the size of param')
    seg = _lib.AdamSegment()
    seg.param, seg.grad, seg.exp_avg, seg.exp_avg_sq = param.data_ptr(), grad.data_ptr(), exp_avg.data_ptr(), exp_avg_sq.data_ptr()
    seg.n_elements = param.numel()
    seg.column_offset = column_offset
    seg.step = int(step)
    for i, v in enumerate(lrs):
        seg.learning_rates[i] = float(v)
    seg.n_learning_rates = len(lrs)
    seg.beta1, seg.beta2 = float(betas[0]), float(betas[1])
    seg.eps = float(eps)
    return seg


def adam_step_segments(segments: list, stream: int | None = None) -> None:
    """Runs the fused Adam kernel over the given segments (12 per launch)."""
    if stream is None:
        stream = torch.cuda.current_stream().cuda_stream
    for i in range(0, len(segments), 12):
        chunk = segments[i:i + 12]
        arr = (_lib.AdamSegment * len(chunk))(*chunk)
        check(lib.fgs_adam_step(arr, len(chunk), stream))


class FusedAdam(torch.optim.Adam):
    def __init__(self, params, lr, eps) -> None:
        super().__init__(params=params, lr=lr, eps=eps)

    @torch.no_grad()
    def step(self) -> None:
        segments = []
        for group in self.param_groups:
            assert len(group['params']) == 1, 'more than one tensor in group'
            param = group['params'][0]
            if param.grad is None or param.numel() == 0:
                continue
            state = self.state[param]
            if len(state) == 0:
                state['step'] = 0
                state['exp_avg'] = torch.zeros_like(param)
                state['exp_avg_sq'] = torch.zeros_like(param)
            state['step'] += 1
            if not param.is_cuda:
                raise RuntimeError('FusedAdam needs CUDA tensors')
            segments.append(_segment(param, param.grad, state['exp_avg'], state['exp_avg_sq'], state['step'], group['lr'],
                                     group['betas'], group['eps']))
        adam_step_segments(segments)
