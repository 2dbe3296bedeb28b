"""Data-parallel training step over views for the fused-appearance rasterizer.

The reference trains on one GPU (Renderer.py:62-65 warns and uses GPU 0). Here a global batch of views is split
over the ranks of a torch.distributed group (one process per GPU); every rank holds a full replica of the Gaussians.
Per step and rank:
  1. render its views and backpropagate the loss, accumulating the gradients of all local views into one flat
     fp32 gradient buffer (the backward kernels write the first view and add the following ones);
  2. reduce the gradients by Gaussian range: rank r receives the summed gradients of Gaussians [r*R, (r+1)*R) of
     every per-Gaussian parameter group (R = ceil(N / ranks), rounded up to a multiple of 4 rows);
  3. fused Adam on that range only (the optimizer moments of the per-Gaussian groups exist only for the range);
  4. gather the updated ranges back into every replica's parameters.
The MLP weights (a few thousand values shared by all Gaussians) are one more segment: owned by the last rank in the
peer exchange, all-reduced with a replicated Adam in the NCCL exchange.
The flat buffers hold the parameter groups one after another (means, scales, rotations, opacities, base colors,
residual parameters, MLP weights), each per-Gaussian group padded to ranks * R rows, so every group stays one
contiguous [N, ...] tensor for the kernels and every rank's rows of a group are one contiguous range. Padding rows
have zero gradients and stay zero. With one rank the collectives are skipped and the result equals the sequential
accumulation over the same views.

Exchange modes: 'nccl' runs steps 2-4 as one NCCL reduce-scatter and one all-gather per per-Gaussian group, an
all-reduce of the MLP gradient, and the fused Adam kernel; 'peer' keeps the flat buffers in symmetric memory (mapped
into every rank) and runs steps 2-4 as one kernel (fgs_dp_shard_adam) that, for every element of the rank's
segments, sums the gradients of all ranks over NVLink (or through the switch with multicast), applies Adam and writes
the new parameter into every rank's buffer, between two device-side barriers. 'auto' picks 'peer' when symmetric
memory can be set up on the group and falls back to 'nccl' otherwise. In the 'peer' exchange the sum is read with
one multimem.ld_reduce through the NVSwitch and the new parameters are written with one multimem.st where the switch
provides multicast mappings: the switch does the sum and the fan-out, so each GPU moves about the vector's size per
link direction and step instead of 2 (N - 1) / N of it (at 8 GPUs 1.1 against 1.9 GB). The multicast loads run at a
lower rate than peer loads, so the fewer bytes pay only at larger N: measured on the c4 step, 2 GPUs 62.5 steps/s with
peer loads / stores against 58.2 with multicast (exchange 1.64 against 2.83 ms), 8 GPUs 133.3 against 144.3 (2.92
against 2.37 ms). multicast='auto' (the default) uses multicast from MULTICAST_MIN_RANKS ranks on, True wherever the
switch provides the mappings, False never.
"""
from __future__ import annotations

import ctypes
import math
import warnings
from dataclasses import dataclass

import torch
import torch.nn.functional as tf

from FasterGSVDACudaBackend import rasterization as R, _lib
from FasterGSVDACudaBackend.adam import _segment, adam_step_segments

# ranks from which the 'auto' exchange reads and writes through NVSwitch multicast: the peer exchange moves
# 2 (N - 1) / N of the vector per link direction at about 0.67 TB/s (measured at 2 and 8 GPUs), the multicast one
# the vector's size at 0.39-0.46 TB/s, so multicast pays from about 5 ranks on
MULTICAST_MIN_RANKS = 5


def multicast_wanted(multicast: bool | str, world: int) -> bool:
    """Whether the peer exchange of `world` ranks reads and writes through NVSwitch multicast (where the switch provides
    the mappings): multicast='auto' from MULTICAST_MIN_RANKS ranks on, True always, False never."""
    if multicast == 'auto':
        return world >= MULTICAST_MIN_RANKS
    if isinstance(multicast, bool):
        return multicast
    raise ValueError(f"multicast must be True, False or 'auto', not {multicast!r}")

GROUP_ORDER = ('means', 'scales', 'rotations', 'opacities', 'base_colors', 'residual_params', 'mlp_weights')


@dataclass
class Group:
    name: str
    offset: int      # in floats, within the flat buffer
    numel: int
    shape: tuple
    lr: float | list
    betas: tuple = (0.9, 0.999)
    cols: int = 0    # floats per Gaussian (0 for the MLP weights)
    shard_offset: int = 0  # in floats, within a rank's moment buffer (per-Gaussian groups)


def gaussian_window(size: int, sigma: float, device, dtype=torch.float32) -> torch.Tensor:
    x = torch.arange(size, dtype=dtype, device=device) - (size - 1) / 2.0
    g = torch.exp(-x * x / (2.0 * sigma * sigma))
    return g / g.sum()


def blur(img: torch.Tensor, size: int, sigma: float) -> torch.Tensor:
    """Separable Gaussian blur of a [C,H,W] image with zero padding."""
    g = gaussian_window(size, sigma, img.device, img.dtype)
    c = img.shape[0]
    x = img[None]
    x = tf.conv2d(x, g.view(1, 1, 1, size).expand(c, 1, 1, size), padding=(0, size // 2), groups=c)
    x = tf.conv2d(x, g.view(1, 1, size, 1).expand(c, 1, size, 1), padding=(size // 2, 0), groups=c)
    return x[0]


def ssim(img: torch.Tensor, target: torch.Tensor, size: int = 11, sigma: float = 1.5) -> torch.Tensor:
    """Mean SSIM with an 11x11 Gaussian window (sigma 1.5), C1 = 0.01^2, C2 = 0.03^2, zero padding."""
    mu_x, mu_y = blur(img, size, sigma), blur(target, size, sigma)
    sxx = blur(img * img, size, sigma) - mu_x * mu_x
    syy = blur(target * target, size, sigma) - mu_y * mu_y
    sxy = blur(img * target, size, sigma) - mu_x * mu_y
    c1, c2 = 0.01 ** 2, 0.03 ** 2
    m = ((2 * mu_x * mu_y + c1) * (2 * sxy + c2)) / ((mu_x * mu_x + mu_y * mu_y + c1) * (sxx + syy + c2))
    return m.mean()


def loss_and_grad_reference(img: torch.Tensor, target: torch.Tensor, l1_weight: float = 0.8, dssim_weight: float = 0.2):
    """The loss definition in PyTorch fp32 (the check for the fused kernel): 0.8 * L1 + 0.2 * (1 - SSIM)
    (Loss.py:14-15 weights); returns (loss, dL/dimage)."""
    x = img.detach().requires_grad_(True)
    loss = l1_weight * (x - target).abs().mean() + dssim_weight * (1.0 - ssim(x, target))
    loss.backward()
    return loss.detach(), x.grad


def morton_order(means: torch.Tensor) -> torch.Tensor:
    """Permutation that sorts Gaussians by the Morton code of their means (21 bits per axis over the means' bounding
    box, fgs_morton_codes), ties kept in index order: the reordering the reference's trainer applies every 5000
    iterations (Trainer.py:165-169, Model.py:449-453) so that Gaussians close in space are close in memory."""
    m = means.detach().reshape(-1, 3).contiguous().float()
    n = m.shape[0]
    codes = torch.empty(n, dtype=torch.int64, device=m.device)
    if n == 0:
        return codes
    lo, hi = m.min(0).values.tolist(), m.max(0).values.tolist()
    _lib.check(_lib.lib.fgs_morton_codes(m.data_ptr(), n, (ctypes.c_float * 3)(*lo), (ctypes.c_float * 3)(*hi), codes.data_ptr(),
                                         torch.cuda.current_stream(m.device).cuda_stream))
    return torch.argsort(codes, stable=True)  # codes < 2^63: the signed order is the code order


class FusedLoss:
    """The same loss through the library's fused CUDA kernels (fgs_l1_dssim): loss value and image gradient stay on
    the device; the workspace is kept between calls of the same image size."""

    def __init__(self, l1_weight: float = 0.8, dssim_weight: float = 0.2) -> None:
        self.l1_weight, self.dssim_weight = l1_weight, dssim_weight
        self.ws = None

    def __call__(self, img: torch.Tensor, target: torch.Tensor, grad_out: torch.Tensor | None = None,
                 loss_out: torch.Tensor | None = None) -> tuple[torch.Tensor, torch.Tensor]:
        if not img.is_cuda:
            raise RuntimeError('FusedLoss needs CUDA tensors (the fused loss has no CPU path)')
        c, h, w = img.shape
        for t in (img, target):
            if t.dtype != torch.float32 or not t.is_contiguous() or t.shape != img.shape or t.device != img.device:
                raise ValueError('image and target must be contiguous float32 [C,H,W] tensors of the same shape on one device')
        need = _lib.size_out(_lib.lib.fgs_loss_workspace_bytes, c, h, w)
        if self.ws is None or self.ws.numel() < need or self.ws.device != img.device:
            self.ws = torch.empty(need, dtype=torch.uint8, device=img.device)
        grad = grad_out if grad_out is not None else torch.empty_like(img)
        loss = loss_out if loss_out is not None else torch.empty((), dtype=torch.float32, device=img.device)
        _lib.check(_lib.lib.fgs_l1_dssim(img.data_ptr(), target.data_ptr(), c, h, w, self.l1_weight, self.dssim_weight, grad.data_ptr(),
                                         loss.data_ptr(), self.ws.data_ptr(), self.ws.numel(), torch.cuda.current_stream(img.device).cuda_stream))
        return loss, grad


class Trainer:
    """Holds the flat parameter / gradient buffers of one replica and runs data-parallel steps."""

    def __init__(self, prims: dict[str, torch.Tensor], lrs: dict[str, float | list], device: torch.device, group=None,
                 mlp_betas: tuple = (0.9, 0.99), exchange: str = 'nccl', multicast: bool | str = 'auto', overlap_views: bool = True,
                 view_streams: int = 2) -> None:
        self.device = device
        self.overlap_views = overlap_views
        self.view_streams = max(1, view_streams)
        self.pg = group
        self.world = torch.distributed.get_world_size(group) if group is not None else 1
        self.rank = torch.distributed.get_rank(group) if group is not None else 0
        self.groups: list[Group] = []
        self.n = prims['means'].shape[0]
        # rows per rank, a multiple of 4 so that every rank's range of every group starts 16-byte aligned
        self.rows = (max(self.n, 1) + 4 * self.world - 1) // (4 * self.world) * 4
        padded = self.rows * self.world
        off, soff = 0, 0
        for name in GROUP_ORDER:
            t = prims.get(name)
            if t is None or t.numel() == 0:
                continue
            if name == 'mlp_weights':
                self.groups.append(Group(name, off, t.numel(), tuple(t.shape), lrs[name], mlp_betas))
                off += (t.numel() + 63) // 64 * 64
                continue
            cols = t.numel() // self.n
            self.groups.append(Group(name, off, t.numel(), tuple(t.shape), lrs[name], (0.9, 0.999), cols, soff))
            off += padded * cols
            soff += self.rows * cols
        self.total = off
        self.shard = soff  # floats of the per-Gaussian moments a rank holds
        self.mlp = next((g for g in self.groups if g.name == 'mlp_weights'), None)
        self.mlp_owner = self.world - 1
        self.exchange = 'nccl'
        self.peers = None
        multicast_wanted(multicast, 1)  # argument check
        self.use_multicast = multicast
        if self.world > 1 and exchange in ('peer', 'auto'):
            try:
                self._setup_peer_buffers()
                self.exchange = 'peer'
            except Exception as err:  # symmetric memory unavailable on this group / driver
                if exchange == 'peer':
                    raise
                self.exchange_error = str(err)
        if self.exchange != 'peer':
            self.params = torch.zeros(self.total, dtype=torch.float32, device=device)
            self.grads = torch.zeros(self.total, dtype=torch.float32, device=device)
        for g in self.groups:
            self.params[g.offset:g.offset + g.numel].copy_(prims[g.name].reshape(-1))
        self.exp_avg = torch.zeros(self.shard, dtype=torch.float32, device=device)
        self.exp_avg_sq = torch.zeros(self.shard, dtype=torch.float32, device=device)
        # MLP moments: on the owning rank (peer exchange) or on every rank (replicated Adam after the all-reduce)
        self.mlp_moments = None
        if self.mlp is not None and (self.exchange != 'peer' or self.rank == self.mlp_owner):
            self.mlp_moments = (torch.zeros(self.mlp.numel, dtype=torch.float32, device=device),
                                torch.zeros(self.mlp.numel, dtype=torch.float32, device=device))
        self.grad_shard = torch.empty(self.shard, dtype=torch.float32, device=device) if self.world > 1 else None
        self.step_count = 0
        self.loss_fns = [FusedLoss() for _ in range(self.view_streams)]
        self._images = [None] * self.view_streams
        self._grad_images = [None] * self.view_streams
        self._side_streams = []

    def _setup_peer_buffers(self) -> None:
        """Flat buffers in symmetric memory: every rank's buffers mapped on every device (peer pointers), plus the
        NVLink multicast mappings when the switch provides them."""
        import torch.distributed._symmetric_memory as symm
        name = self.pg.group_name
        if hasattr(symm, 'enable_symm_mem_for_group') and not symm.is_symm_mem_enabled_for_group(name):
            with warnings.catch_warnings():  # newer torch enables symmetric memory for every group and deprecates the call
                warnings.simplefilter('ignore', FutureWarning)
                symm.enable_symm_mem_for_group(name)
        self.params = symm.empty(self.total, dtype=torch.float32, device=self.device)
        self.grads = symm.empty(self.total, dtype=torch.float32, device=self.device)
        self.params.zero_()
        self.grads.zero_()
        self.h_params = symm.rendezvous(self.params, name)
        self.h_grads = symm.rendezvous(self.grads, name)
        pb = _lib.PeerBuffers()
        pb.n_ranks = self.world
        for r in range(self.world):
            pb.grads[r] = self.h_grads.buffer_ptrs[r]
            pb.params[r] = self.h_params.buffer_ptrs[r]
        pb.local_params = self.params.data_ptr()
        mg, mp = int(getattr(self.h_grads, 'multicast_ptr', 0) or 0), int(getattr(self.h_params, 'multicast_ptr', 0) or 0)
        self.multicast = bool(mg and mp) and multicast_wanted(self.use_multicast, self.world)
        pb.multicast_grads = mg if self.multicast else None
        pb.multicast_params = mp if self.multicast else None
        self.peers = pb

    def view(self, buf: torch.Tensor, name: str) -> torch.Tensor | None:
        """Parameter group `name` of a flat parameter or gradient buffer, as its [N, ...] tensor."""
        for g in self.groups:
            if g.name == name:
                return buf[g.offset:g.offset + g.numel].view(g.shape)
        return None

    def range_view(self, buf: torch.Tensor, name: str, rank: int | None = None) -> torch.Tensor:
        """Rows [rank * R, (rank + 1) * R) of per-Gaussian group `name` in a flat buffer, as an [R, cols] tensor."""
        g = next(x for x in self.groups if x.name == name)
        r = self.rank if rank is None else rank
        lo = g.offset + r * self.rows * g.cols
        return buf[lo:lo + self.rows * g.cols].view(self.rows, g.cols)

    def shard_view(self, buf: torch.Tensor, name: str) -> torch.Tensor:
        """This rank's part of per-Gaussian group `name` in a moment-layout buffer (exp_avg, exp_avg_sq, grad_shard)."""
        g = next(x for x in self.groups if x.name == name)
        return buf[g.shard_offset:g.shard_offset + self.rows * g.cols].view(self.rows, g.cols)

    def _prims(self) -> tuple:
        v = lambda k: self.view(self.params, k)
        empty = torch.empty(0, device=self.device)
        cp = R._c_primitives(v('means'), v('scales'), v('rotations'), v('opacities'), None, v('base_colors'), v('residual_params'),
                             v('mlp_weights') if v('mlp_weights') is not None else None)
        return cp

    def _grads(self) -> _lib.Gradients:
        v = lambda k: self.view(self.grads, k)
        p = lambda t: t.data_ptr() if t is not None else None
        return _lib.Gradients(p(v('means')), p(v('scales')), p(v('rotations')), p(v('opacities')), None, p(v('base_colors')),
                              p(v('residual_params')), p(v('mlp_weights')))

    def backward_views(self, settings_list: list, targets: list, ready: list | None = None) -> torch.Tensor:
        """Renders the local views and accumulates their gradients into the flat gradient buffer; returns the summed loss.

        With overlap_views (and more than one view) consecutive views go round `view_streams` streams (the current
        one and side streams), each with its own workspaces, image and loss buffers: the forward, loss and binning of
        the next views run while view k's backward runs. The backward passes stay chained in view order (each waits
        for the previous one's event), so gradients accumulate view by view as in the sequential order. `ready`
        (optional, one CUDA event per view) lets the targets arrive asynchronously: view k's loss waits for ready[k],
        its render does not."""
        cp = self._prims()
        cg = self._grads()
        main = torch.cuda.current_stream(self.device)
        S = self.view_streams if self.overlap_views and len(settings_list) > 1 else 1
        overlap = S > 1
        while len(self._side_streams) < S - 1:
            self._side_streams.append(torch.cuda.Stream(self.device))
        streams = [main] + self._side_streams[:S - 1]
        totals = [torch.zeros((), device=self.device) for _ in range(S)]
        for side in streams[1:]:
            side.wait_stream(main)  # parameters, targets and totals are ready
        prev_backward = None
        states = [None] * S  # a view's workspaces live until the next view on the same stream replaces them
        for k, (settings, target) in enumerate(zip(settings_list, targets)):
            j = k % S
            with torch.cuda.stream(streams[j]):
                st = R.ForwardState(R._rasterizer, cp, settings, self.device)
                st.preprocess(cp)
                shape = (3, settings.height, settings.width)
                if self._images[j] is None or tuple(self._images[j].shape) != shape:
                    self._images[j] = torch.empty(shape, device=self.device)
                    self._grad_images[j] = torch.empty(shape, device=self.device)
                st.render_train(self._images[j])
                if ready is not None:
                    streams[j].wait_event(ready[k])
                loss, _ = self.loss_fns[j](self._images[j], target, grad_out=self._grad_images[j])
                totals[j] += loss
                if prev_backward is not None:
                    streams[j].wait_event(prev_backward)
                st.backward(cp, self._images[j], self._grad_images[j], cg, None, accumulate=k > 0)
                if overlap:
                    prev_backward = torch.cuda.Event()
                    prev_backward.record(streams[j])
                states[j] = st
        for side in streams[1:]:
            main.wait_stream(side)
        return sum(totals[1:], totals[0])

    @torch.no_grad()
    def apply_morton_ordering(self) -> None:
        """Reorders every per-Gaussian parameter group and its Adam moments by the Morton order of the means (the same
        permutation on every rank: all replicas hold the same means). A rank's moments cover only its Gaussian range,
        so with several ranks the moments are gathered, permuted and split into ranges again."""
        order = morton_order(self.view(self.params, 'means'))
        n, rows, world = self.n, self.rows, self.world
        if world > 1:
            full_m = torch.empty(self.shard * world, dtype=torch.float32, device=self.device)
            full_v = torch.empty(self.shard * world, dtype=torch.float32, device=self.device)
            torch.distributed.all_gather_into_tensor(full_m, self.exp_avg, group=self.pg)
            torch.distributed.all_gather_into_tensor(full_v, self.exp_avg_sq, group=self.pg)
        for g in self.groups:
            if g.name == 'mlp_weights':
                continue
            p_rows = self.params[g.offset:g.offset + g.numel].view(n, g.cols)
            p_rows.copy_(p_rows[order])
            for local, full in ((self.exp_avg, full_m if world > 1 else None), (self.exp_avg_sq, full_v if world > 1 else None)):
                if full is None:
                    rows_m = local[g.shard_offset:g.shard_offset + rows * g.cols].view(rows, g.cols)[:n]
                    rows_m.copy_(rows_m[order])
                    continue
                # the group's moments of all ranks in row order: rank r's part sits at r * shard + shard_offset
                parts = full.view(world, self.shard)[:, g.shard_offset:g.shard_offset + rows * g.cols]
                allrows = parts.reshape(world * rows, g.cols)
                allrows[:n] = allrows[:n][order]
                local[g.shard_offset:g.shard_offset + rows * g.cols].copy_(allrows[self.rank * rows:(self.rank + 1) * rows].reshape(-1))

    def adam_segments(self, grads: torch.Tensor | None = None, with_mlp: bool = True) -> list:
        """Adam segments of this rank: its Gaussian range of every per-Gaussian group (gradients from `grads`, a
        moment-layout buffer, by default the local flat gradient buffer's rows of the range) and, with_mlp, the MLP
        weights."""
        segs = []
        for g in self.groups:
            if g.name == 'mlp_weights':
                continue
            lo = g.offset + self.rank * self.rows * g.cols
            size = self.rows * g.cols
            grad = self.grads[lo:lo + size] if grads is None else grads[g.shard_offset:g.shard_offset + size]
            segs.append(_segment(self.params[lo:lo + size], grad, self.exp_avg[g.shard_offset:g.shard_offset + size],
                                 self.exp_avg_sq[g.shard_offset:g.shard_offset + size], self.step_count, g.lr, g.betas, 1e-15,
                                 column_offset=self.rank * self.rows * g.cols))
        if with_mlp and self.mlp is not None and self.mlp_moments is not None:
            g = self.mlp
            segs.append(_segment(self.params[g.offset:g.offset + g.numel], self.grads[g.offset:g.offset + g.numel], self.mlp_moments[0],
                                 self.mlp_moments[1], self.step_count, g.lr, g.betas, 1e-15))
        return segs

    def apply_gradients(self, adam_fn=None) -> None:
        """Exchange step: gradients reduced by Gaussian range, Adam on this rank's range (and the MLP weights), the
        ranges gathered back into every replica. `adam_fn(segments)` replaces the fused GPU Adam (used by the CPU tests
        with the checker's Adam)."""
        self.step_count += 1
        if self.exchange == 'peer':
            self.h_grads.barrier(channel=0)  # every rank's gradients are final
            segs = self.adam_segments(with_mlp=self.rank == self.mlp_owner)
            arr = (_lib.AdamSegment * len(segs))(*segs)
            _lib.check(_lib.lib.fgs_dp_shard_adam(arr, len(segs), ctypes.byref(self.peers), torch.cuda.current_stream(self.device).cuda_stream))
            self.h_params.barrier(channel=1)  # every rank's parameters are written
            return
        if self.world == 1:
            (adam_fn or adam_step_segments)(self.adam_segments())
            return
        for g in self.groups:
            if g.name == 'mlp_weights':
                torch.distributed.all_reduce(self.grads[g.offset:g.offset + g.numel], group=self.pg)
                continue
            size = self.rows * g.cols
            torch.distributed.reduce_scatter_tensor(self.grad_shard[g.shard_offset:g.shard_offset + size],
                                                    self.grads[g.offset:g.offset + size * self.world], group=self.pg)
        (adam_fn or adam_step_segments)(self.adam_segments(self.grad_shard))
        for g in self.groups:
            if g.name == 'mlp_weights':
                continue
            size = self.rows * g.cols
            full = self.params[g.offset:g.offset + size * self.world]
            torch.distributed.all_gather_into_tensor(full, full[self.rank * size:(self.rank + 1) * size], group=self.pg)

    def step(self, settings_list: list, targets: list, ready: list | None = None) -> torch.Tensor:
        loss = self.backward_views(settings_list, targets, ready)
        self.apply_gradients()
        return loss
