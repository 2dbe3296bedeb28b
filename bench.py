"""Benchmark of the B200-native fused-appearance rasterizer (driver contract: one JSON line on rank 0).

Default workload c4 (the headline "train steps/s @1080p"): one data-parallel training step of the Neural appearance
model -- 6,000,000 Gaussians, 32 latent features per Gaussian, MLP 80 -> 64 -> 64 -> 3 (fp16 tensor cores) -- over a
global batch of 8 views at 1920x1080. Every rank renders its share of the views (forward, loss 0.8 L1 + 0.2 (1 - SSIM)
against a blurred random target, backward with gradients accumulated over its views); the gradients are summed by
Gaussian range, every rank runs the fused Adam on its range, and the updated ranges go back to every rank (one fused
kernel over NVLink, or NCCL with --exchange nccl). The total work is fixed as N grows ("scaling": "strong"). The
line also carries "render": inference of configuration c3 (3M Gaussians, NASG 8 lobes, 64 ring views at 1920x1080,
views split over the GPUs) in frames/s, timed the same way after the training step (--no-render skips it).

Workload c1 (--workload c1): one SH-3 training step (forward, backward, fused Adam through the public autograd API)
of 1,000,000 Gaussians on one 1280x720 view with a fixed upstream image gradient; with N GPUs every rank trains its
own replica (no exchange step, "scaling": "weak").

value: steps/s with every input resident in HBM. e2e: the same step with the step's inputs (c4: the target images of
the rank's views; c1: the upstream gradient) copied host->device from pinned memory and the step's result (c4: the
loss; c1: the rendered image) copied back, every step. --impl reference times the CPU restatement of the reference
path (oracle/, "port", on every host core) on a bounded sample of the same workload.
"""
from __future__ import annotations

import argparse
import json
import os
import sys
import threading
import time
from pathlib import Path

ROOT = Path(__file__).resolve().parent
sys.path.insert(0, str(ROOT))
sys.path.insert(0, str(ROOT / 'efficient-gaussian-appearance_b200'))

import numpy as np
import torch

WORKLOADS = {
    'c1': dict(n=1_000_000, width=1280, height=720, model='sh', degree=3, views=1),
    'c2': dict(n=1_000_000, width=1264, height=832, model='neural', degree=3, views=1, feature_dim=32, n_freq=1, neurons=64, hidden=2),
    # the paper's default network (550 of the reference's 559 paper configurations): 8 features, 1 octave, 2 x 16 hidden
    'c2paper': dict(n=1_000_000, width=1264, height=832, model='neural', degree=3, views=1, feature_dim=8, n_freq=1, neurons=16, hidden=2),
    'c4': dict(n=6_000_000, width=1920, height=1080, model='neural', degree=3, views=8, feature_dim=32, n_freq=1, neurons=64, hidden=2),
    'c3': dict(n=3_000_000, width=1920, height=1080, model='nasg', degree=8, views=64),
    'c3sv': dict(n=3_000_000, width=1920, height=1080, model='sv', degree=8, views=64),
}
C1_LRS = {'means': 1.6e-4, 'scales': 0.005, 'rotations': 0.001, 'opacities': 0.05, 'base_colors': 0.000705237, 'residual_params': 0.000125}
C2_LRS = {'means': 1.6e-4, 'scales': 0.005, 'rotations': 0.001, 'opacities': 0.05, 'base_colors': 0.00025, 'residual_params': 0.008,
          'mlp_weights': 0.003}
SINGLE_VIEW = ('c1', 'c2', 'c2paper')
C4_LRS = {'means': 1.6e-4, 'scales': 0.005, 'rotations': 0.001, 'opacities': 0.05, 'base_colors': 0.00025, 'residual_params': 0.008,
          'mlp_weights': 0.003}
RENDER = ('c3', 'c3sv')
METRIC = {'c3': 'render FPS (inference, NASG 8 lobes, 3M Gaussians, 64 ring views @1920x1080, views sharded over the GPUs)',
          'c3sv': 'render FPS (inference, Spherical Voronoi 8 sites, 3M Gaussians, 64 ring views @1920x1080, views sharded over the GPUs)',
          'c1': 'train steps/s (forward + backward + fused Adam), fused SH-3 appearance, 1M Gaussians @1280x720',
          'c2': 'train steps/s (forward + backward + fused Adam), Neural appearance (32 features, 2x64 MLP), 1M Gaussians @1264x832',
          'c2paper': 'train steps/s (forward + backward + fused Adam), Neural appearance (8 features, 2x16 MLP), 1M Gaussians @1264x832',
          'c4': 'train steps/s (8 views @1920x1080, forward + loss + backward + gradient reduce-scatter + sharded fused Adam + '
                'parameter all-gather), Neural appearance, 6M Gaussians'}
# this library's kernel launches per view: preprocess 1, compaction 4 (group sums, group scan, chunk offsets, compact),
# depth sort 4 passes x 3 (upsweep, row scan, downsweep), depth reorder 1, offset scan 3, emission 1, tile sort
# 2 passes x 3 (end_bit 13 or 14 at these sizes), ranges + bucket scan 2, blend 1; training adds the fused loss 3
# (c4), the backward blend 1 and the backward preprocess (SH: 1; Neural: tcgen05 backward + geometry 2), plus the
# Neural colour pass 1 in the forward. Per step: one fused Adam (or the fused exchange kernel). The first view's
# gradient arrays are cleared with memsets; those, NCCL and torch's own kernels are not counted.
RENDER_LAUNCHES_PER_VIEW = 1 + 4 + 12 + 1 + 3 + 1 + 6 + 2 + 1


def own_launches(wl_name: str, views: int) -> int:
    if wl_name in RENDER:
        return RENDER_LAUNCHES_PER_VIEW * views
    if wl_name == 'c4':  # per view: loss 3, colour pass, blend backward, MLP backward + geometry; per step: Adam
        return (RENDER_LAUNCHES_PER_VIEW + 3 + 1 + 1 + 2) * views + 1
    if WORKLOADS[wl_name]['model'] == 'neural':  # colour pass, blend backward, MLP backward + geometry, Adam
        return RENDER_LAUNCHES_PER_VIEW + 1 + 1 + 2 + 1
    return RENDER_LAUNCHES_PER_VIEW + 1 + 1 + 1


def _peaks() -> tuple[float, str]:
    p = ROOT / 'MEASURED_PEAKS.json'
    if p.exists():
        d = json.loads(p.read_text())
        return float(d['hbm_gbs']), 'measured'
    return 6650.0, 'fallback'


class ClockSampler:
    """Samples SM clock and clock-event reasons through NVML every 20 ms while the timed region runs."""

    REASONS = {0x4: 'sw_power_cap', 0x8: 'hw_slowdown', 0x20: 'sw_thermal_slowdown', 0x40: 'hw_thermal_slowdown', 0x80: 'hw_power_brake'}

    def __init__(self, device: torch.device) -> None:
        self.device = device
        self.samples = []
        self.reasons = set()
        self.stop = threading.Event()
        self.thread = None
        self.handle = None
        self.max_mhz = None

    def __enter__(self):
        try:
            import pynvml
            pynvml.nvmlInit()
            try:
                uuid = str(torch.cuda.get_device_properties(self.device).uuid)
                self.handle = pynvml.nvmlDeviceGetHandleByUUID(uuid if uuid.startswith('GPU-') else 'GPU-' + uuid)
            except Exception:
                self.handle = pynvml.nvmlDeviceGetHandleByIndex(self.device.index or 0)
            self.max_mhz = pynvml.nvmlDeviceGetMaxClockInfo(self.handle, pynvml.NVML_CLOCK_SM)
            self.pynvml = pynvml

            def run():
                while not self.stop.is_set():
                    try:
                        self.samples.append(pynvml.nvmlDeviceGetClockInfo(self.handle, pynvml.NVML_CLOCK_SM))
                        bits = pynvml.nvmlDeviceGetCurrentClocksEventReasons(self.handle) if hasattr(
                            pynvml, 'nvmlDeviceGetCurrentClocksEventReasons') else pynvml.nvmlDeviceGetCurrentClocksThrottleReasons(self.handle)
                        for b, name in self.REASONS.items():
                            if bits & b:
                                self.reasons.add(name)
                    except Exception:
                        pass
                    self.stop.wait(0.02)

            self.thread = threading.Thread(target=run, daemon=True)
            self.thread.start()
        except Exception:
            self.handle = None
        return self

    def __exit__(self, *exc):
        self.stop.set()
        if self.thread is not None:
            self.thread.join(timeout=5)

    def summary(self) -> dict:
        if not self.samples:
            return {'sm_mhz': None, 'sm_max_mhz': self.max_mhz, 'reasons': ['unsampled']}
        return {'sm_mhz': float(np.median(self.samples)), 'sm_max_mhz': float(self.max_mhz), 'reasons': sorted(self.reasons),
                'samples': len(self.samples)}


# ------------------------------------------------------------------------------------------------------------
# scenes

def scene(wl: dict) -> dict:
    import synthetic as S
    n = wl['n']
    geo = S.geometry(n)
    if wl['model'] == 'sh':
        return {**geo, **S.sh_appearance(n, wl['degree'])}
    if wl['model'] == 'nasg':
        return {**geo, **S.nasg_appearance(n, wl['degree'])}
    if wl['model'] == 'sv':
        return {**geo, **S.sv_appearance(n, wl['degree'])}
    n_in = wl['feature_dim'] * 2 * wl['n_freq'] + 16
    pad = (n_in + 15) // 16 * 16
    return {**geo, **S.neural_appearance(n, wl['feature_dim'], layer_shapes=S.mlp_layer_shapes(pad, wl['neurons'], wl['hidden']))}


def configure(wl: dict) -> None:
    import FasterGSVDACudaBackend as F
    if wl['model'] in ('sh', 'nasg', 'sv'):
        F.initialize_appearance(wl['model'], wl['degree'], 'none', 'none', 'relu', True)
        return
    F.initialize_appearance('neural', 0, 'none', 'tanh', 'relu', True)
    F.initialize_residual_mlp(wl['feature_dim'] * 2 * wl['n_freq'] + 16, 3, {'otype': 'Identity'},
                              {'otype': 'FullyFusedMLP', 'activation': 'ReLU', 'output_activation': 'None', 'n_neurons': wl['neurons'],
                               'n_hidden_layers': wl['hidden']}, False, wl['n_freq'], [0, 1, 2, 3])


def targets(wl: dict) -> list[torch.Tensor]:
    """Per-view training targets: U(0,1) images smoothed by a 9x9 Gaussian blur (sigma 2), seed 2."""
    from trainer import blur
    g = torch.Generator().manual_seed(2)
    return [blur(torch.rand(3, wl['height'], wl['width'], generator=g), 9, 2.0).contiguous() for _ in range(wl['views'])]


def settings_of(cam, degree: int, dev):
    import FasterGSVDACudaBackend as F
    return F.RasterizerSettings(cam.w2c.to(dev), cam.position.to(dev), cam.bg.to(dev), degree, cam.width, cam.height, cam.focal_x,
                                cam.focal_y, cam.center_x, cam.center_y, cam.near_plane, cam.far_plane, False, True, True)


# DRAM bytes (read + write) measured by ncu on the small c4 case (2M Gaussians in Morton order, one view: 945,338
# visible rows, 3,455,838 instances), per visible row and per instance: backward preprocess = warp-specialised MLP
# backward (566.6 MB) + its geometry pass (274.3 MB), per visible row; blend backward (170.6 MB) over the instances.
# Scaled by the view's visible rows and instances.
TRAFFIC_PER_UNIT = {('c4', 'preprocess_backward'): ((566.6e6 + 274.3e6) / 945338, 0.0), ('c4', 'blend_backward'): (0.0, (157.0e6 + 13.2e6) / 3455837)}
# how each stage is bound at these sizes (ncu): the blends issue-bound (warps walking subtiles or bands of the tile),
# the tensor-core MLP stages latency-bound on their per-tile MMA -> epilogue chains; the rest streams HBM
BOUND = {'blend_forward': 'issue', 'blend_inference': 'issue', 'blend_backward': 'issue', 'appearance_mlp': 'latency',
         'preprocess_backward': 'latency'}


def stage_bytes(stage: str, s: dict) -> float:
    """Algorithmic DRAM bytes of one occurrence of each stage per view (per-unit figures x the frame's units): N
    Gaussians, V visible, I instances, P pixels, A appearance bytes read per visible Gaussian by the fused preprocess
    (0 for Neural, whose colour pass reads the latent), F latent floats, K key bytes (2 or 4), T tiles."""
    N, V, I, P, A, F, K, T = s['N'], s['V'], s['I'], s['pixels'], s['appearance_bytes'], s['features'], s['key_bytes'], s['tiles']
    neural = s['model'] == 'neural'
    if stage == 'preprocess':  # geometry of every Gaussian, appearance of the visible ones; counts and keys, records
        return N * 44 + (0 if neural else V * A) + N * 8 + V * 52
    if stage == 'compaction':
        return N * 8 + V * 8
    if stage == 'appearance_mlp':  # index, mean, latent, base in; colour out; activation store (training) out
        return V * (4 + 12 + 4 * F + 12 + 12) + V * s['store_bytes']
    if stage == 'depth_sort':  # 4 passes of 8 bits over (key, value) pairs, read and written
        return 4 * V * 16
    if stage == 'reorder_scan':
        return V * (48 + 48 + 12) + V * 12
    if stage == 'emit':
        return V * 52 + I * (K + 4)
    if stage == 'tile_sort':
        return 2 * I * (K + 4) * 2
    if stage == 'ranges':
        return I * K + T * 12
    if stage == 'blend_forward':
        return I * 52 + P * 20
    if stage == 'blend_inference':
        return I * 52 + P * 12
    if stage == 'loss':
        return 3 * P * 44
    if stage == 'blend_backward':
        return I * 52 + P * 32 + V * 48
    if stage == 'preprocess_backward':
        # Neural: the gradient arrays of all N rows (geometry 44, base 12, latent 4F bytes) are cleared by memsets
        # when a view does not accumulate (every view of c2; the first of the step's views in c4: clear_share)
        clear = s['clear_share'] * N * (56 + 4 * F)
        if neural and s['store_bytes']:
            # tensor-core path, per visible row. Geometry pass: index, rank, blend sums (48) and record (48), geometry
            # parameters (44) and base (12), stored raw outputs (8), the 80-byte row block written, gradients of the
            # geometry parameters and base added (read + write). MLP backward: index, latent, the activation store and
            # row block, latent gradient and mean gradient added (read + write).
            geometry = 4 + 4 + 48 + 48 + 44 + 12 + 8 + 80 + 2 * (44 + 12)
            mlp = 4 + 4 * F + s['store_bytes'] + 80 + 8 * F + 24
            return V * (geometry + mlp) + clear
        if neural:  # touched rows: MLP backward + geometry backward
            return V * (128 + 8 * F) + V * 192 + clear
        return N * 4 + V * (44 + A + 96) + N * (44 + A)
    if stage == 'adam':
        return 28 * s['params']
    return 0.0


def stage_flops(stage: str, s: dict) -> float:
    """Tensor-core FLOPs of the Neural MLP stages per view: 2 x (multiply-adds of every layer, the output padded to 16
    rows) per visible row forward; twice that backward (data and weight gradients; the activations come from the store)."""
    if s['model'] != 'neural':
        return 0.0
    if stage == 'appearance_mlp':
        return s['V'] * s['mlp_flops']
    if stage == 'preprocess_backward':
        return 2.0 * s['V'] * s['mlp_flops']
    return 0.0


def frame_stats(wl: dict, n_visible: int, n_instances: int, n_params: int, clear_share: float = 1.0) -> dict:
    """The per-view units the byte and FLOP counts scale with (clear_share: the fraction of views that clear the
    gradient arrays instead of accumulating into them)."""
    model = wl['model']
    stride = {'sh': 45, 'neural': wl.get('feature_dim', 0), 'nasg': 8 * wl['degree'], 'sv': 7 * wl['degree']}[model]
    tiles = ((wl['width'] + 15) // 16) * ((wl['height'] + 11) // 12)
    out = dict(N=wl['n'], V=n_visible, I=n_instances, pixels=wl['width'] * wl['height'], params=n_params, model=model,
               appearance_bytes=0 if model == 'neural' else 12 + 4 * stride, features=wl.get('feature_dim', 0),
               key_bytes=2 if tiles <= 65536 else 4, tiles=tiles, store_bytes=0, mlp_flops=0, clear_share=clear_share)
    if model == 'neural':
        nn, hidden = wl['neurons'], wl['hidden']
        kin = (wl['feature_dim'] * 2 * wl['n_freq'] + 16 + 15) // 16 * 16
        out['mlp_flops'] = 2 * (kin * nn + (hidden - 1) * nn * nn + nn * 16)
        out['store_bytes'] = 128 * hidden + 8 if nn == 64 else 0  # the tensor-core kernels' activation store (training)
    return out


def static_config(wl_name: str, world: int, args, exchange_desc: str = 'none') -> dict:
    """The workload description both arms print (no measured quantities)."""
    wl = WORKLOADS[wl_name]
    render, strong = wl_name in RENDER, wl_name == 'c4' or wl_name in RENDER
    if render:
        desc = f"{wl['model']}-{wl['degree']} {wl['n'] / 1e6:g}M Gaussians, {wl['views']} views {wl['width']}x{wl['height']}, inference, views sharded"
    elif strong:
        desc = f"Neural {wl['n'] / 1e6:g}M Gaussians, {wl['views']} views {wl['width']}x{wl['height']} global batch, data-parallel"
    elif wl['model'] == 'neural':
        desc = (f"Neural ({wl['feature_dim']} features, {wl['hidden']}x{wl['neurons']} MLP) {wl['n'] / 1e6:g}M Gaussians, 1 view "
                f"{wl['width']}x{wl['height']} per GPU")
    else:
        desc = f"SH-3 {wl['n'] / 1e6:g}M Gaussians, 1 view {wl['width']}x{wl['height']} per GPU"
    views_per_gpu = ((wl['views'] + world - 1) // world) if render else (wl['views'] // world if strong else 1)
    return {'workload': f'{wl_name}: {desc}', 'n_gaussians': wl['n'], 'width': wl['width'], 'height': wl['height'], 'views_per_gpu': views_per_gpu,
            'parallelism': (f'{world} GPU(s), views split, no collective' if render else
                            f'dp{world} (reduce-scatter / sharded Adam / all-gather: {exchange_desc})' if strong else f'replicas x{world}'),
            'l2': 'inputs larger than L2 (parameters alone exceed 126 MB)', 'gaussian_order': getattr(args, 'order', 'morton')}


def _tensor_peak() -> float:
    """Sustained dense bf16/fp16 tensor TFLOP/s of this pool's B200s (the MLP stages run inside a long step)."""
    p = ROOT / 'MEASURED_PEAKS.json'
    if p.exists():
        d = json.loads(p.read_text())
        return float(d.get('bf16_tflops_sustained', d.get('bf16_tflops', 1400.0)))
    return 1400.0


# ------------------------------------------------------------------------------------------------------------
# B200 arm

def run_b200(args, wl_name: str, companion: bool = False) -> dict | None:
    """One workload on this rank's GPU. With companion=True (the render measurement that follows the c4 training
    step in the same process) only the timed and end-to-end loops run, and the process group is left open."""
    from FasterGSVDACudaBackend import _lib, rasterization as R
    import synthetic as S
    wl = WORKLOADS[wl_name]
    world = int(os.environ.get('WORLD_SIZE', '1'))
    rank = int(os.environ.get('RANK', '0'))
    local = int(os.environ.get('LOCAL_RANK', '0'))
    torch.cuda.set_device(local)
    dev = torch.device('cuda', local)
    pg = None
    if world > 1:
        if not torch.distributed.is_initialized():
            import datetime
            torch.distributed.init_process_group('nccl', timeout=datetime.timedelta(seconds=300), device_id=dev)
        pg = torch.distributed.group.WORLD
    configure(wl)
    prims = scene(wl)
    if getattr(args, 'order', 'morton') == 'morton':
        # a scene in training is kept in Morton order by the reference's trainer (Trainer.py:165-169, every 5000
        # iterations): the same Gaussians, reordered so that neighbours in space are neighbours in memory
        from trainer import morton_order
        order = morton_order(prims['means'].to(dev)).cpu()
        prims = {k: (v if k == 'mlp_weights' else v[order].contiguous()) for k, v in prims.items()}
    cams = S.ring_cameras(wl['views'] if wl_name in RENDER else 8, wl['width'], wl['height'])

    def barrier():
        if world > 1:
            torch.distributed.barrier()
        torch.cuda.synchronize()

    if wl_name in RENDER:
        import FasterGSVDACudaBackend as F
        per = (wl['views'] + world - 1) // world
        mine = [v for v in range(rank * per, min((rank + 1) * per, wl['views']))]
        dp = {k: v.to(dev).contiguous() for k, v in prims.items()}
        del prims
        settings = [settings_of(cams[v], wl['degree'], dev) for v in mine]
        imgs_host = [torch.empty((wl['height'], wl['width'], 3), pin_memory=True) for _ in range(2)]

        def render(s0):
            return F.rasterize(dp['means'], dp['scales'], dp['rotations'], dp['opacities'], s0, False, True,
                               base_colors=dp['base_colors'], residual_params=dp['residual_params'])

        def step():
            for s0 in settings:
                render(s0)

        copy_stream = torch.cuda.Stream(dev)

        def step_e2e():
            # each image goes down on a copy stream while the next view renders; the step ends with the last image on
            # the host
            main = torch.cuda.current_stream()
            for k, s0 in enumerate(settings):
                img = render(s0)
                copy_stream.wait_stream(main)
                with torch.cuda.stream(copy_stream):
                    imgs_host[k % 2].copy_(img, non_blocking=True)
                img.record_stream(copy_stream)
            main.wait_stream(copy_stream)

        h2d = 0
        d2h = len(mine) * wl['height'] * wl['width'] * 3 * 4
        views_per_step = len(mine)
        n_params = sum(v.numel() for v in dp.values())
        stat_settings = settings[0]
        stat_prims = R._c_primitives(dp['means'], dp['scales'], dp['rotations'], dp['opacities'], None, dp['base_colors'], dp['residual_params'], None)
    elif wl_name == 'c4':
        from trainer import Trainer
        assert wl['views'] % world == 0, 'the global batch of 8 views must split evenly over the GPUs'
        per = wl['views'] // world
        mine = list(range(rank * per, (rank + 1) * per))
        trainer = Trainer({k: v.to(dev) for k, v in prims.items()}, C4_LRS, dev, group=pg, exchange=args.exchange, multicast=args.multicast)
        del prims
        settings = [settings_of(cams[v], wl['degree'], dev) for v in mine]
        tg_host = [t.pin_memory() for t in [targets(wl)[v] for v in mine]]
        tg_dev = [t.to(dev) for t in tg_host]
        n_params = trainer.shard + (trainer.mlp.numel if trainer.mlp_moments is not None else 0)  # parameters this rank's Adam updates

        def step():
            return trainer.step(settings, tg_dev)

        copy_stream = torch.cuda.Stream(dev)
        arrived = [torch.cuda.Event() for _ in tg_dev]

        def step_e2e():
            # the step's targets go up on a copy stream, one event per view, so the first views render while the later
            # targets are still in flight; the previous step's losses were the last readers of the device buffers
            copy_stream.wait_stream(torch.cuda.current_stream())
            with torch.cuda.stream(copy_stream):
                for h, d, ev in zip(tg_host, tg_dev, arrived):
                    d.copy_(h, non_blocking=True)
                    ev.record(copy_stream)
            loss = trainer.step(settings, tg_dev, ready=arrived)
            return loss.to('cpu', non_blocking=True)

        h2d = sum(t.numel() * 4 for t in tg_host)
        d2h = 4
        views_per_step = per
        stat_settings = settings[0]
        stat_prims = trainer._prims()
    else:
        import FasterGSVDACudaBackend as F
        cam = cams[rank % len(cams)]
        s0 = settings_of(cam, wl['degree'], dev)
        params = {k: torch.nn.Parameter(v.to(dev).contiguous()) for k, v in prims.items()}
        lrs = C1_LRS if wl['model'] == 'sh' else C2_LRS
        opt = F.FusedAdam([{'params': [params[k]], 'lr': lr} for k, lr in lrs.items()], lr=0.0, eps=1e-15)
        mlp = params.get('mlp_weights')
        grad_host = (torch.randn(3, wl['height'], wl['width'], generator=torch.Generator().manual_seed(2)) * 0.01).pin_memory()
        grad_dev = grad_host.to(dev)
        img_host = torch.empty((3, wl['height'], wl['width']), pin_memory=True)
        empty = torch.empty(0, device=dev)
        n_params = sum(p.numel() for p in params.values())

        def run(g):
            img = F.diff_rasterize(params['means'], params['scales'], params['rotations'], params['opacities'], empty, s0,
                                   base_colors=params['base_colors'], residual_params=params['residual_params'], mlp_weights=mlp)
            img.backward(g)
            opt.step()
            for p in params.values():
                p.grad = None
            return img

        def step():
            return run(grad_dev)

        copy_stream = torch.cuda.Stream(dev)
        grad_in = torch.empty_like(grad_dev)
        grad_ready = torch.cuda.Event()

        def step_e2e():
            # the upstream gradient goes up on a copy stream during the forward; the image goes down during the backward
            main = torch.cuda.current_stream()
            copy_stream.wait_stream(main)
            with torch.cuda.stream(copy_stream):
                grad_in.copy_(grad_host, non_blocking=True)
                grad_ready.record(copy_stream)
            img = F.diff_rasterize(params['means'], params['scales'], params['rotations'], params['opacities'], empty, s0,
                                   base_colors=params['base_colors'], residual_params=params['residual_params'], mlp_weights=mlp)
            copy_stream.wait_stream(main)
            with torch.cuda.stream(copy_stream):
                img_host.copy_(img.detach(), non_blocking=True)
            main.wait_event(grad_ready)
            img.backward(grad_in)
            opt.step()
            for p in params.values():
                p.grad = None
            main.wait_stream(copy_stream)
            return img_host

        h2d = grad_host.numel() * 4
        d2h = img_host.numel() * 4
        views_per_step = 1
        stat_settings = s0
        stat_prims = R._c_primitives(params['means'].detach(), params['scales'].detach(), params['rotations'].detach(),
                                     params['opacities'].detach(), None, params['base_colors'].detach(), params['residual_params'].detach(),
                                     mlp.detach() if mlp is not None else None)

    exchange_desc = 'none'
    if wl_name == 'c4' and world > 1:
        exchange_desc = ('one fused kernel over NVLink ' + ('multicast (multimem)' if trainer.multicast else 'peer loads/stores')
                         if trainer.exchange == 'peer' else 'NCCL + fused Adam')
    for _ in range(args.warmup):
        step()
    barrier()

    stream = torch.cuda.current_stream()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    with ClockSampler(dev) as clk:
        barrier()
        e0.record(stream)
        for _ in range(args.steps):
            step()
        e1.record(stream)
        barrier()
    ms = e0.elapsed_time(e1) / args.steps
    clocks = clk.summary()

    barrier()
    e2, e3 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e2.record(stream)
    for _ in range(args.steps):
        step_e2e()
    e3.record(stream)
    barrier()
    ms_e2e = e2.elapsed_time(e3) / args.steps

    if companion:
        if world > 1:
            t = torch.tensor([ms, ms_e2e], device=dev)
            torch.distributed.all_reduce(t, op=torch.distributed.ReduceOp.MAX)
            ms, ms_e2e = float(t[0]), float(t[1])
        fps, fps_e2e = wl['views'] * 1000.0 / ms, wl['views'] * 1000.0 / ms_e2e
        return {'metric': METRIC[wl_name], 'value': fps, 'unit': 'frames/s', 'ms_per_step': ms, 'steps': args.steps, 'warmup': args.warmup,
                'scaling': 'strong', 'config': static_config(wl_name, world, args),
                'mpix_per_s': fps * wl['width'] * wl['height'] / 1e6,
                'e2e': {'value': fps_e2e, 'unit': 'frames/s', 'h2d_bytes_per_step': int(h2d), 'd2h_bytes_per_step': int(d2h)},
                'gpu_launches': own_launches(wl_name, views_per_step) * args.steps, 'clocks': clocks} if rank == 0 else None

    # per-stage timing pass (CUDA events on the launching stream), averaged per step; the training step runs its views
    # one after another here (no second stream), so every stage's events bracket only that stage's kernels
    overlapped = wl_name == 'c4' and trainer.overlap_views
    if overlapped:
        trainer.overlap_views = False
    _lib.profile_enable(True)
    n_prof = 2
    for _ in range(n_prof):
        step()
    torch.cuda.synchronize()
    _lib.profile_enable(False)
    if overlapped:
        trainer.overlap_views = True
    stage_ms = {k: v / n_prof for k, v in _lib.profile_collect().items()}

    # frame statistics of one view
    st = R.ForwardState(R._rasterizer, stat_prims, stat_settings, dev)
    st.preprocess(stat_prims)
    fr = st.frame
    del st
    stats = frame_stats(wl, fr.n_visible, fr.n_instances, n_params, 1.0 / views_per_step if wl_name == 'c4' else 1.0)
    per_view = {k: (v if k == 'adam' else v / views_per_step) for k, v in stage_ms.items()}
    dominant = max(stage_ms, key=stage_ms.get)
    peak, peak_kind = _peaks()
    bytes_dom = stage_bytes(dominant, stats)
    achieved = bytes_dom / (per_view[dominant] * 1e-3) / 1e9 if bytes_dom else 0.0
    per_unit = TRAFFIC_PER_UNIT.get((wl_name, dominant))
    traffic = per_unit[0] * stats['V'] + per_unit[1] * stats['I'] if per_unit else None
    traffic_src = ('ncu dram__bytes_read.sum + dram__bytes_write.sum per visible row and per instance on the 2M-Gaussian one-view case (Morton '
                   'order), x visible rows and instances of view 0 (per view launch)') if per_unit else None
    fracs = {k: round(stage_bytes(k, stats) / (per_view[k] * 1e-3) / 1e9 / peak, 4) for k in per_view if stage_bytes(k, stats) and per_view[k] > 0}
    tflops_peak = _tensor_peak()
    tensor_fracs = {k: round(stage_flops(k, stats) / (per_view[k] * 1e-3) / 1e12 / tflops_peak, 4) for k in per_view
                    if stage_flops(k, stats) and per_view[k] > 0}

    if world > 1:
        t = torch.tensor([ms, ms_e2e], device=dev)
        torch.distributed.all_reduce(t, op=torch.distributed.ReduceOp.MAX)
        ms, ms_e2e = float(t[0]), float(t[1])
    strong = wl_name == 'c4' or wl_name in RENDER
    render = wl_name in RENDER
    units_per_step = wl['views'] if render else 1  # frames (render) or training steps per timed step, all ranks together
    steps_per_s = units_per_step * 1000.0 / ms if strong else world * 1000.0 / ms
    e2e_per_s = units_per_step * 1000.0 / ms_e2e if strong else world * 1000.0 / ms_e2e
    out = {
        'metric': METRIC[wl_name],
        'value': steps_per_s,
        'unit': 'frames/s' if render else 'steps/s',
        'n_gpus': world,
        'steps': args.steps,
        'warmup': args.warmup,
        'ms_per_step': ms,
        'higher_is_better': True,
        'scaling': 'strong' if strong else 'weak',
        'vs_baseline': None,
        'dtype': 'f32 (MLP fp16 operands, fp32 accumulation)' if wl['model'] == 'neural' else 'f32',
        'data': 'synthetic (seeded scene with the configuration shapes and distributions; no dataset available)',
        'config': static_config(wl_name, world, args, exchange_desc),
        'frame': {'n_visible_view0': fr.n_visible, 'n_instances_view0': fr.n_instances,
                  'mpix_per_s': steps_per_s * wl['width'] * wl['height'] / 1e6 if render else None},
        'e2e': {'value': e2e_per_s, 'unit': 'frames/s' if render else 'steps/s', 'h2d_bytes_per_step': int(h2d), 'd2h_bytes_per_step': int(d2h)},
        'gpu_launches': own_launches(wl_name, views_per_step) * args.steps,
        'clocks': clocks,
        'stage_ms_per_step': {k: round(v, 4) for k, v in stage_ms.items()},
        'roofline': {'kernel': dominant, 'bound': 'hbm', 'achieved': achieved, 'peak': peak, 'peak_kind': peak_kind, 'unit': 'GB/s',
                     'frac': achieved / peak, 'traffic': traffic, 'traffic_source': traffic_src, 'algorithmic_bytes': bytes_dom,
                     'frac_by_stage': fracs, 'tensor_frac_by_stage': tensor_fracs, 'tensor_peak_tflops': tflops_peak,
                     'bound_by_stage': {k: BOUND.get(k, 'hbm') for k in per_view},
                     # training with the tensor-core MLP: the fp16 activations the colour pass writes and the MLP
                     # backward reads back (inside both stages' algorithmic bytes), per view
                     'activation_store_bytes_per_view': stats['V'] * stats['store_bytes']},
    }
    if wl_name == 'c4' and args.render:
        # the other half of the headline metric (train steps/s and render FPS): inference of configuration c3 on the
        # same GPUs, measured after the training step (the training state stays allocated: it is a few GB)
        torch.cuda.synchronize()
        r = run_b200(args, 'c3', companion=True)
        if rank == 0:
            out['render'] = r
    if world > 1:
        torch.distributed.destroy_process_group()
    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        prep = cpu_prepare(wl_name, args.cpu_sample)
        runs = [cpu_step(prep) for _ in range(3)]
        base = {k: runs[0][k] for k in ('unit', 'cores', 'kind', 'sample')}
        base['value'] = float(np.median([r['value'] for r in runs]))
        out['cpu_baseline'] = base
        out['cpu_baseline_appearance'] = cpu_appearance_baseline()
    return out if rank == 0 else None


# ------------------------------------------------------------------------------------------------------------
# CPU restatement (reference arm and cpu_baseline)

def cpu_prepare(wl_name: str, tile_sample: float = 0.05, threads: int = 0) -> dict:
    """The bounded sample of the CPU restatement (oracle/, its per-primitive and per-pixel loops on `threads` OpenMP
    threads, by default every host core), prepared once:
    c1: preprocess / depth order / binning / backward preprocess / Adam of all Gaussians, blends on a random
        `tile_sample` fraction of the tiles (scaled to all tiles).
    c2 / c4: one view of a scene with 1/64 of the Gaussians (same distributions) with blends on `tile_sample` of the
        tiles; preprocess, binning and backward-preprocess times scaled x64, blend times x64 / tile_sample, times the
        views, plus Adam over all the workload's parameters (timed on 1/64 and scaled).
    c3: one frame of a 1/32 scene with the blend on `tile_sample` of the tiles, scaled x32 (x32 / tile_sample)."""
    import synthetic as S
    from oracle import oracle as O
    wl = dict(WORKLOADS[wl_name])
    scale = 1
    if wl['model'] == 'neural' or wl_name in RENDER:
        scale = 32 if wl_name in RENDER else 64
        wl['n'] = wl['n'] // scale
    prims = scene(wl)
    cam = S.ring_cameras(8, wl['width'], wl['height'])[0]
    threads = threads or os.cpu_count() or 1
    return dict(wl_name=wl_name, wl=wl, prims=prims, cam=cam, lib=O.load(False), O=O, scale=scale, tile_sample=tile_sample, threads=threads)


def cpu_step(prep: dict) -> dict:
    """One timed sample: the scaled estimate in the metric's unit, and the sample's own wall time."""
    O = prep['O']
    O.set_threads(prep['threads'])
    try:
        t0 = time.perf_counter()
        out = _cpu_step_timed(prep['wl_name'], prep['wl'], prep['prims'], prep['cam'], prep['lib'], O, prep['scale'], prep['tile_sample'],
                              prep['threads'])
        out['sample_ms'] = (time.perf_counter() - t0) * 1e3
        return out
    finally:
        O.set_threads(1)


def cpu_appearance_baseline(n: int = 100_000, reps: int = 5) -> dict:
    """Configuration c0: the reference's CPU-runnable path, its unfused PyTorch appearance (SH degree 3, activations
    none / none / relu) forward plus autograd backward for N Gaussians on the host cores, timed through the PyTorch
    restatement oracle/appearance_torch.py (pinned to the reference modules' own outputs). Inputs as configs[0]: base
    ~N(0,1), rest ~N(0,0.3), means uniform in a radius-5 ball, camera at distance 8, upstream gradient ~N(0,1)."""
    from oracle import appearance_torch as AT
    threads = os.cpu_count() or 1
    torch.set_num_threads(threads)
    g = torch.Generator().manual_seed(1)
    base = torch.randn(n, 3, generator=g).requires_grad_(True)
    rest = (torch.randn(n, 15, 3, generator=g) * 0.3).requires_grad_(True)
    d = torch.nn.functional.normalize(torch.randn(n, 3, generator=g))
    means = (d * 5.0 * torch.rand(n, 1, generator=g) ** (1.0 / 3.0)).requires_grad_(True)
    cam = torch.tensor([0.0, 0.0, 8.0])
    up = torch.randn(n, 3, generator=torch.Generator().manual_seed(2))
    times = []
    for r in range(reps + 1):
        t0 = time.perf_counter()
        AT.sh_colors(means, cam, base, rest, 3).backward(up)
        times.append(time.perf_counter() - t0)
        for t in (base, rest, means):
            t.grad = None
    t = float(np.median(times[1:]))
    return {'value': 1.0 / t, 'unit': 'c0 steps/s (SH-3 colours of 100,000 Gaussians, forward + autograd backward)', 'cores': threads,
            'kind': 'port', 'sample': f'full c0 workload, median of {reps} after 1 warm-up; PyTorch restatement of the reference\'s unfused '
                                      f'Appearance/SH.py path'}


def _cpu_step_timed(wl_name, wl, prims, cam, lib, O, scale, tile_sample, threads) -> dict:
    import ctypes
    if wl['model'] in ('sh', 'nasg', 'sv'):
        a = O.make_appearance(wl['model'], wl['degree'], 0, 0, 1, True)
    else:
        n_in = wl['feature_dim'] * 2 * wl['n_freq'] + 16
        neural = dict(feature_dim=wl['feature_dim'], base_input=0, n_freq=wl['n_freq'], sh_mask=15, n_input=n_in,
                      n_input_pad=(n_in + 15) // 16 * 16, n_neurons=wl['neurons'], n_hidden=wl['hidden'], hidden_act=1)
        a = O.make_appearance('neural', 0, 0, 1, 1, True, neural=neural)
    v = O.make_view(cam, wl['degree'])
    p = {k: O._f32(x) for k, x in prims.items()}
    n, W, H = wl['n'], wl['width'], wl['height']
    mlp = p.get('mlp_weights')
    t0 = time.perf_counter()
    n_touched = np.zeros(n, np.uint32)
    depth_key = np.zeros(n, np.uint32)
    rec = np.zeros((n, 14))
    lib.orc_preprocess(ctypes.byref(a), ctypes.byref(v), n, O._p(p['means']), O._p(p['scales']), O._p(p['rotations']), O._p(p['opacities']),
                       None, O._p(p['base_colors']), O._p(p['residual_params']), O._p(mlp), O._p(n_touched), O._p(depth_key), O._p(rec))
    sidx = np.zeros(n, np.uint32)
    V = lib.orc_depth_order(n, O._p(n_touched), O._p(depth_key), O._p(sidx))
    I = lib.orc_count_instances(V, O._p(sidx), O._p(n_touched))
    T = ((W + 15) // 16) * ((H + 11) // 12)
    keys = np.zeros(max(I, 1), np.uint32)
    ranks = np.zeros(max(I, 1), np.uint32)
    ranges = np.zeros((T, 2), np.uint32)
    lib.orc_bin(V, O._p(sidx), O._p(rec), W, H, O._p(keys), O._p(ranks), O._p(ranges))
    t1 = time.perf_counter()
    keep = np.random.default_rng(0).random(T) < tile_sample
    frac = max(float(keep.mean()), 1.0 / T)
    ranges_s = ranges.copy()
    ranges_s[~keep] = 0
    image = np.zeros((3, H, W), np.float32)
    fT = np.zeros((H, W), np.float32)
    nc = np.zeros((H, W), np.uint32)
    lib.orc_blend(V, O._p(sidx), O._p(rec), O._p(ranks), O._p(ranges_s), ctypes.byref(v), O._p(image), O._p(fT), O._p(nc), 1, 0)
    if wl_name in RENDER:  # inference: one frame = preprocess + binning + blend
        t2 = time.perf_counter()
        frame_s = (t1 - t0) * scale + (t2 - t1) * scale / frac
        sample = (f'{wl_name} frame estimated from one view of a {n}-Gaussian scene (1/32 of 3M) at 1920x1080 with the blend on '
                  f'{int(keep.sum())} of {T} tiles, scaled x32 (x{32 / frac:.0f} for the blend); C restatement on {threads} threads')
        return {'value': 1.0 / frame_s, 'unit': 'frames/s', 'cores': threads, 'kind': 'port', 'sample': sample}
    gimg = np.ascontiguousarray((np.random.default_rng(2).standard_normal((3, H, W)) * 0.01).astype(np.float32))
    rg = np.zeros((max(V, 1), 12))
    lib.orc_blend_backward(V, O._p(sidx), O._p(rec), O._p(ranks), O._p(ranges_s), ctypes.byref(v), O._p(nc), O._p(gimg), O._p(rg))
    t2 = time.perf_counter()
    rank_of = np.full(n, 0xffffffff, np.uint32)
    rank_of[sidx[:V]] = np.arange(V, dtype=np.uint32)
    outs = [np.zeros((n, 3)), np.zeros((n, 3)), np.zeros((n, 4)), np.zeros(n), np.zeros((n, 3)), np.zeros(p['residual_params'].reshape(n, -1).shape)]
    gm = np.zeros(mlp.shape[0]) if mlp is not None else None
    lib.orc_preprocess_backward(ctypes.byref(a), ctypes.byref(v), n, O._p(p['means']), O._p(p['scales']), O._p(p['rotations']),
                                O._p(p['opacities']), None, O._p(p['base_colors']), O._p(p['residual_params']), O._p(mlp), O._p(rank_of),
                                O._p(rec), O._p(rg), *[O._p(x) for x in outs[:4]], None, O._p(outs[4]), O._p(outs[5]), O._p(gm), None, 0)
    t3 = time.perf_counter()
    for x in p.values():
        xx = np.ascontiguousarray(x, np.float32).reshape(-1).copy()
        O.adam(xx, np.ones_like(xx), np.zeros_like(xx), np.zeros_like(xx), 1, 1e-3, (0.9, 0.999), 1e-15)
    t4 = time.perf_counter()
    view_s = (t1 - t0) * scale + (t2 - t1) * scale / frac + (t3 - t2) * scale
    step_s = view_s * wl['views'] + (t4 - t3) * scale
    if wl['model'] == 'neural':
        sample = (f'{wl_name} step estimated from one view of a {n}-Gaussian scene (1/64 of {n * 64 / 1e6:g}M) at {W}x{H} with blends on '
                  f'{int(keep.sum())} of {T} tiles, scaled x64 (x{64 / frac:.0f} for blends), x{wl["views"]} views, plus Adam; C restatement on '
                  f'{threads} threads')
    else:
        sample = (f'c1 step: preprocess/binning/backward-preprocess/Adam on all {n} Gaussians, blends on {int(keep.sum())} of {T} tiles scaled '
                  f'x{1 / frac:.1f}; C restatement on {threads} threads')
    return {'value': 1.0 / step_s, 'unit': 'steps/s', 'cores': threads, 'kind': 'port', 'sample': sample}


def main() -> None:
    ap = argparse.ArgumentParser()
    ap.add_argument('--gpus', type=int, default=1)
    ap.add_argument('--steps', type=int, default=20)
    ap.add_argument('--warmup', type=int, default=3)
    ap.add_argument('--impl', default='b200', choices=['b200', 'reference'])
    ap.add_argument('--workload', default='c4', choices=sorted(WORKLOADS))
    ap.add_argument('--cpu-sample', type=float, default=0.05)
    ap.add_argument('--no-cpu-baseline', action='store_true')
    ap.add_argument('--no-render', dest='render', action='store_false',
                    help='c4: skip the render measurement of configuration c3 that the line carries under "render"')
    ap.add_argument('--exchange', default='auto', choices=['auto', 'peer', 'nccl'], help='c4 data-parallel exchange (N > 1)')
    ap.add_argument('--no-multicast', dest='multicast', action='store_const', const=False, default='auto',
                    help='c4 peer exchange by loads / stores only (by default NVSwitch multicast from trainer.MULTICAST_MIN_RANKS GPUs on)')
    ap.add_argument('--multicast', dest='multicast', action='store_const', const=True,
                    help='c4 peer exchange through NVSwitch multicast (multimem) at any GPU count where the switch provides it')
    ap.add_argument('--gaussians', type=int, default=0, help='override the workload\'s Gaussian count (small profiling cases)')
    ap.add_argument('--views', type=int, default=0, help='override the workload\'s global batch of views (c4)')
    ap.add_argument('--order', default='morton', choices=['morton', 'generated'],
                    help='order of the Gaussians in memory: Morton order of the means (as the reference trainer keeps them) or as generated')
    args = ap.parse_args()
    if args.gaussians:
        WORKLOADS[args.workload]['n'] = args.gaussians
    if args.views:
        WORKLOADS[args.workload]['views'] = args.views
    if args.impl == 'reference':
        if int(os.environ.get('RANK', '0')) != 0:
            return
        prep = cpu_prepare(args.workload, args.cpu_sample)
        for _ in range(args.warmup):
            cpu_step(prep)
        runs = [cpu_step(prep) for _ in range(args.steps)]
        v = float(np.median([r['value'] for r in runs]))
        ms = float(np.median([r['sample_ms'] for r in runs]))
        unit = 'frames/s' if args.workload in RENDER else 'steps/s'
        base = {k: runs[0][k] for k in ('unit', 'cores', 'kind', 'sample')}
        base['value'] = v
        print(json.dumps({'impl': 'reference', 'metric': METRIC[args.workload], 'value': v, 'unit': unit, 'n_gpus': args.gpus,
                          'steps': args.steps, 'warmup': args.warmup, 'ms_per_step': ms, 'higher_is_better': True,
                          'scaling': 'strong' if args.workload in ('c4',) + RENDER else 'weak', 'vs_baseline': None, 'dtype': 'f32',
                          'data': 'synthetic (seeded scene with the configuration shapes and distributions; no dataset available)',
                          'config': static_config(args.workload, args.gpus, args),
                          'estimate': {'value_is_estimate': True, 'timed': 'each of the steps is one bounded sample of the workload (ms_per_step is '
                                       'its measured wall time); value is the sample scaled to one full step of the workload', 'sample': base['sample']},
                          'cpu_baseline': base, 'cpu_baseline_appearance': cpu_appearance_baseline(),
                          'e2e': {'value': v, 'unit': unit, 'h2d_bytes_per_step': 0, 'd2h_bytes_per_step': 0}}))
        return
    out = run_b200(args, args.workload)
    if out is not None:
        print(json.dumps(out))


if __name__ == '__main__':
    main()
