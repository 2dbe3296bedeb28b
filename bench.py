"""Benchmark of the B200-native fused-appearance rasterizer (driver contract: one JSON line on rank 0).

Default workload (c1 of the benchmark configurations): one full training step of the differentiable rasterizer with
fused SH degree 3 -- forward (preprocess, binning, blend), backward (blend backward, preprocess backward) and the fused
Adam update of every parameter group -- for N = 1,000,000 synthetic Gaussians and one 1280x720 view. With --gpus N
(torchrun, one process per GPU) every rank trains its own replica on its own view (replicas only: the workload has no
exchange step), so the aggregate value is the sum over ranks ("scaling": "weak").

value: steps/s with all inputs resident in HBM; e2e: the same through the public API with the view's upstream
gradient copied host->device from pinned memory and the rendered image copied back every step.
--impl reference times the CPU restatement of the reference path (oracle/, single thread) on a bounded sample.
"""
from __future__ import annotations

import argparse
import json
import math
import os
import subprocess
import sys
import time
from pathlib import Path

ROOT = Path(__file__).resolve().parent
sys.path.insert(0, str(ROOT))
sys.path.insert(0, str(ROOT / 'efficient-gaussian-appearance_b200'))

import numpy as np
import torch

WORKLOADS = {
    'c1': dict(n=1_000_000, width=1280, height=720, model='sh', degree=3),
}

# kernels of this library launched per training step (preprocess, chunk scan, compaction, reorder, emit, ranges,
# bucket scan, forward blend, backward blend, backward preprocess, adam); CUB sort / scan kernels are not counted
OWN_KERNELS_PER_STEP = 11


def _peaks() -> tuple[float, str]:
    p = ROOT / 'MEASURED_PEAKS.json'
    if p.exists():
        d = json.loads(p.read_text())
        return float(d['hbm_gbs']), 'measured'
    return 6650.0, 'fallback'


class ClockSampler:
    """Samples nvidia-smi clocks and throttle reasons while the timed region runs."""

    def __init__(self, index: int) -> None:
        self.index = index
        self.proc = None
        self.path = Path(f'/tmp/fgs_clocks_{os.getpid()}.csv')

    def __enter__(self):
        q = ('index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,clocks_event_reasons.hw_slowdown,'
             'clocks_event_reasons.hw_thermal_slowdown,clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap')
        try:
            self.proc = subprocess.Popen(['nvidia-smi', f'--id={self.index}', f'--query-gpu={q}', '--format=csv,noheader,nounits', '-lms', '200'],
                                         stdout=open(self.path, 'w'), stderr=subprocess.DEVNULL)
        except (FileNotFoundError, OSError):
            self.proc = None
        return self

    def __exit__(self, *exc):
        if self.proc is not None:
            self.proc.terminate()
            self.proc.wait(timeout=10)

    def summary(self) -> dict:
        if not self.path.exists():
            return {'sm_mhz': None, 'sm_max_mhz': None, 'reasons': ['unsampled']}
        sm, smax, reasons = [], [], set()
        for line in self.path.read_text().splitlines():
            f = [x.strip() for x in line.split(',')]
            if len(f) < 9:
                continue
            try:
                sm.append(float(f[1]))
                smax.append(float(f[2]))
            except ValueError:
                continue
            for name, val in zip(('hw_slowdown', 'hw_thermal_slowdown', 'sw_thermal_slowdown', 'sw_power_cap'), f[5:9]):
                if val.lower() == 'active':
                    reasons.add(name)
        self.path.unlink(missing_ok=True)
        if not sm:
            return {'sm_mhz': None, 'sm_max_mhz': None, 'reasons': ['unsampled']}
        return {'sm_mhz': float(np.median(sm)), 'sm_max_mhz': float(max(smax)), 'reasons': sorted(reasons), 'samples': len(sm)}


def make_scene(wl: dict, seed_view: int):
    import synthetic as S
    n = wl['n']
    prims = {**S.geometry(n), **S.sh_appearance(n, wl['degree'])}
    cams = S.ring_cameras(8, wl['width'], wl['height'])
    cam = cams[seed_view % len(cams)]
    grad = torch.randn(3, wl['height'], wl['width'], generator=torch.Generator().manual_seed(2)) * 0.01
    return prims, cam, grad


def stage_bytes(stage: str, s: dict) -> float:
    """Algorithmic DRAM bytes of one launch of each stage (per-unit figures x units of the frame)."""
    N, V, I, P = s['N'], s['V'], s['I'], s['pixels']
    A = s['appearance_bytes']
    B = s['buckets_used']
    if stage == 'preprocess':
        return N * (44 + A) + N * 8 + V * (48 + 4)
    if stage == 'blend_forward':
        return I * (4 + 48) + P * (12 + 4 + 4) + B * 192 * 16
    if stage == 'blend_backward':
        return I * (4 + 48) + B * 192 * (16 + 12 + 12 + 4 + 4) + V * 48
    if stage == 'preprocess_backward':
        return N * (44 + A) * 2 + N * 4 + V * 96
    if stage == 'adam':
        return 28 * s['params']
    return 0.0


def run_b200(args, wl) -> dict:
    import FasterGSVDACudaBackend as F
    from FasterGSVDACudaBackend import _lib

    world = int(os.environ.get('WORLD_SIZE', '1'))
    rank = int(os.environ.get('RANK', '0'))
    local = int(os.environ.get('LOCAL_RANK', '0'))
    torch.cuda.set_device(local)
    dev = torch.device('cuda', local)
    if world > 1:
        import datetime
        torch.distributed.init_process_group('nccl', timeout=datetime.timedelta(seconds=120), device_id=dev)

    F.initialize_appearance('sh', wl['degree'], 'none', 'none', 'relu', True)
    prims, cam, grad_cpu = make_scene(wl, rank)
    params = {k: torch.nn.Parameter(v.to(dev).contiguous()) for k, v in prims.items()}
    settings = F.RasterizerSettings(cam.w2c.to(dev), cam.position.to(dev), cam.bg.to(dev), wl['degree'], wl['width'], wl['height'],
                                    cam.focal_x, cam.focal_y, cam.center_x, cam.center_y, cam.near_plane, cam.far_plane, False, True, True)
    lrs = {'means': 1.6e-4, 'scales': 0.005, 'rotations': 0.001, 'opacities': 0.05, 'base_colors': 0.000705237, 'residual_params': 0.000125}
    opt = F.FusedAdam([{'params': [params[k]], 'lr': lr} for k, lr in lrs.items()], lr=0.0, eps=1e-15)
    grad_dev = grad_cpu.to(dev)
    empty = torch.empty(0, device=dev)

    def step(grad_image):
        img = F.diff_rasterize(params['means'], params['scales'], params['rotations'], params['opacities'], empty, settings,
                               base_colors=params['base_colors'], residual_params=params['residual_params'])
        img.backward(grad_image)
        opt.step()
        for p in params.values():
            p.grad = None
        return img

    def barrier():
        if world > 1:
            torch.distributed.barrier()
        torch.cuda.synchronize()

    for _ in range(args.warmup):
        step(grad_dev)
    barrier()

    # device-resident timing
    stream = torch.cuda.current_stream()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    with ClockSampler(local) as clk:
        barrier()
        e0.record(stream)
        for _ in range(args.steps):
            step(grad_dev)
        e1.record(stream)
        barrier()
    ms = e0.elapsed_time(e1) / args.steps
    clocks = clk.summary()

    # end to end: upstream gradient H2D from pinned memory, rendered image D2H, every step
    grad_pinned = grad_cpu.pin_memory()
    img_host = torch.empty((3, wl['height'], wl['width']), pin_memory=True)
    barrier()
    e2, e3 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e2.record(stream)
    for _ in range(args.steps):
        g = grad_pinned.to(dev, non_blocking=True)
        img = step(g)
        img_host.copy_(img.detach(), non_blocking=True)
    e3.record(stream)
    barrier()
    ms_e2e = e2.elapsed_time(e3) / args.steps

    # per-stage timing pass (CUDA events on the launching stream) for the roofline of the dominant kernel
    _lib.profile_enable(True)
    n_prof = 3
    stats = None
    for _ in range(n_prof):
        img = F.diff_rasterize(params['means'], params['scales'], params['rotations'], params['opacities'], empty, settings,
                               base_colors=params['base_colors'], residual_params=params['residual_params'])
        img.backward(grad_dev)
        opt.step()
        for p in params.values():
            p.grad = None
    torch.cuda.synchronize()
    _lib.profile_enable(False)
    stage_ms = {k: v / n_prof for k, v in _lib.profile_collect().items()}
    # frame statistics of this view (visible primitives, instances, buckets actually used)
    from FasterGSVDACudaBackend import rasterization as R
    cp = R._c_primitives(params['means'].detach(), params['scales'].detach(), params['rotations'].detach(), params['opacities'].detach(),
                         None, params['base_colors'].detach(), params['residual_params'].detach(), None)
    st = R.ForwardState(R._rasterizer, cp, settings, dev)
    st.preprocess(cp)
    im = torch.empty((3, wl['height'], wl['width']), device=dev)
    st.render_train(im)
    torch.cuda.synchronize()
    fr = st.frame
    views = st.views()
    T = fr.grid_w * fr.grid_h
    off = views.bucket_offsets - st.tile_ws.data_ptr()
    buckets_used = int(st.tile_ws[off + 4 * (T - 1): off + 4 * T].view(torch.int32).item())
    n_params = sum(p.numel() for p in params.values())
    s = dict(N=wl['n'], V=fr.n_visible, I=fr.n_instances, pixels=wl['width'] * wl['height'], appearance_bytes=12 + 4 * params['residual_params'][0].numel(),
             buckets_used=buckets_used, params=n_params)
    dominant = max(stage_ms, key=stage_ms.get)
    peak, peak_kind = _peaks()
    achieved = stage_bytes(dominant, s) / (stage_ms[dominant] * 1e-3) / 1e9 if stage_bytes(dominant, s) else 0.0

    # max over ranks
    if world > 1:
        t = torch.tensor([ms, ms_e2e], device=dev)
        torch.distributed.all_reduce(t, op=torch.distributed.ReduceOp.MAX)
        ms, ms_e2e = float(t[0]), float(t[1])
    out = {
        'metric': 'train steps/s (forward + backward + fused Adam), fused SH-3 appearance',
        'value': world * 1000.0 / ms,
        'unit': 'steps/s',
        'n_gpus': world,
        'steps': args.steps,
        'warmup': args.warmup,
        'ms_per_step': ms,
        'higher_is_better': True,
        'scaling': 'weak',
        'vs_baseline': None,
        'dtype': 'f32',
        'data': 'synthetic (seeded scene with the c1 shapes and distributions; no dataset available)',
        'config': {'workload': 'c1: SH-3 differentiable rasterization fwd+bwd+Adam, 1,000,000 Gaussians, 1 view 1280x720 per GPU',
                   'n_gaussians': wl['n'], 'width': wl['width'], 'height': wl['height'], 'n_visible': fr.n_visible,
                   'n_instances': fr.n_instances, 'parallelism': f'replicas x{world}',
                   'l2': 'inputs larger than L2 (236 MB of Gaussian parameters per step)'},
        'e2e': {'value': world * 1000.0 / ms_e2e, 'unit': 'steps/s', 'h2d_bytes_per_step': int(grad_cpu.numel() * 4),
                'd2h_bytes_per_step': int(img_host.numel() * 4)},
        'gpu_launches': OWN_KERNELS_PER_STEP * args.steps,
        'clocks': clocks,
        'stage_ms': {k: round(v, 4) for k, v in stage_ms.items()},
        'roofline': {'kernel': dominant, 'bound': 'hbm', 'achieved': achieved, 'peak': peak, 'peak_kind': peak_kind, 'unit': 'GB/s',
                     'frac': achieved / peak, 'traffic': None, 'algorithmic_bytes': stage_bytes(dominant, s)},
    }
    if world > 1:
        torch.distributed.destroy_process_group()
    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        out['cpu_baseline'] = cpu_step(wl, sample_tiles=args.cpu_sample)
    return out if rank == 0 else None


def cpu_step(wl: dict, sample_tiles: float = 0.05) -> dict:
    """One training step of the CPU restatement (oracle/, one thread): preprocess, depth order and binning of all
    Gaussians, forward and backward blend of a random `sample_tiles` fraction of the tiles (scaled to the full image),
    backward preprocess of all Gaussians. Returns steps/s."""
    import ctypes
    from oracle import oracle as O
    prims, cam, grad = make_scene(wl, 0)
    lib = O.load(False)
    a = O.make_appearance('sh', wl['degree'], 0, 0, 1, True)
    v = O.make_view(cam, wl['degree'])
    p = {k: O._f32(x) for k, x in prims.items()}
    n = wl['n']
    W, H = wl['width'], wl['height']
    t0 = time.perf_counter()
    n_touched = np.zeros(n, np.uint32)
    depth_key = np.zeros(n, np.uint32)
    rec = np.zeros((n, 14))
    lib.orc_preprocess(ctypes.byref(a), ctypes.byref(v), n, O._p(p['means']), O._p(p['scales']), O._p(p['rotations']), O._p(p['opacities']),
                       None, O._p(p['base_colors']), O._p(p['residual_params']), None, O._p(n_touched), O._p(depth_key), O._p(rec))
    sidx = np.zeros(n, np.uint32)
    V = lib.orc_depth_order(n, O._p(n_touched), O._p(depth_key), O._p(sidx))
    I = lib.orc_count_instances(V, O._p(sidx), O._p(n_touched))
    T = ((W + 15) // 16) * ((H + 11) // 12)
    keys = np.zeros(max(I, 1), np.uint32)
    ranks = np.zeros(max(I, 1), np.uint32)
    ranges = np.zeros((T, 2), np.uint32)
    lib.orc_bin(V, O._p(sidx), O._p(rec), W, H, O._p(keys), O._p(ranks), O._p(ranges))
    t1 = time.perf_counter()
    rng = np.random.default_rng(0)
    keep = rng.random(T) < sample_tiles
    frac = max(keep.mean(), 1.0 / T)
    ranges_s = ranges.copy()
    ranges_s[~keep] = 0
    image = np.zeros((3, H, W), np.float32)
    fT = np.zeros((H, W), np.float32)
    nc = np.zeros((H, W), np.uint32)
    lib.orc_blend(V, O._p(sidx), O._p(rec), O._p(ranks), O._p(ranges_s), ctypes.byref(v), O._p(image), O._p(fT), O._p(nc), 1, 0)
    gimg = np.ascontiguousarray(grad.numpy())
    rg = np.zeros((max(V, 1), 12))
    lib.orc_blend_backward(V, O._p(sidx), O._p(rec), O._p(ranks), O._p(ranges_s), ctypes.byref(v), O._p(nc), O._p(gimg), O._p(rg))
    t2 = time.perf_counter()
    rank_of = np.full(n, 0xffffffff, np.uint32)
    rank_of[sidx[:V]] = np.arange(V, dtype=np.uint32)
    outs = [np.zeros((n, 3)), np.zeros((n, 3)), np.zeros((n, 4)), np.zeros(n), np.zeros((n, 3)), np.zeros(p['residual_params'].reshape(n, -1).shape)]
    lib.orc_preprocess_backward(ctypes.byref(a), ctypes.byref(v), n, O._p(p['means']), O._p(p['scales']), O._p(p['rotations']),
                                O._p(p['opacities']), None, O._p(p['base_colors']), O._p(p['residual_params']), None, O._p(rank_of), O._p(rec),
                                O._p(rg), *[O._p(x) for x in outs[:4]], None, O._p(outs[4]), O._p(outs[5]), None, None, 0)
    mom = [np.zeros_like(np.asarray(x, np.float32)) for x in p.values()]
    for (k, x), m in zip(p.items(), mom):
        xx = x.copy().reshape(-1)
        O.adam(xx, np.ones_like(xx), m.reshape(-1), m.copy().reshape(-1), 1, 1e-3, (0.9, 0.999), 1e-15)
    t3 = time.perf_counter()
    step_s = (t1 - t0) + (t2 - t1) / frac + (t3 - t2)
    return {'value': 1.0 / step_s, 'unit': 'steps/s', 'cores': 1, 'kind': 'port',
            'sample': f'c1 step: preprocess/binning/backward-preprocess/adam on all {n} Gaussians, blend fwd+bwd on {keep.sum()} of {T} tiles '
                      f'scaled x{1 / frac:.1f}; single-threaded C restatement'}


def main() -> None:
    ap = argparse.ArgumentParser()
    ap.add_argument('--gpus', type=int, default=1)
    ap.add_argument('--steps', type=int, default=20)
    ap.add_argument('--warmup', type=int, default=3)
    ap.add_argument('--impl', default='b200', choices=['b200', 'reference'])
    ap.add_argument('--workload', default='c1', choices=sorted(WORKLOADS))
    ap.add_argument('--cpu-sample', type=float, default=0.05)
    ap.add_argument('--no-cpu-baseline', action='store_true')
    args = ap.parse_args()
    wl = WORKLOADS[args.workload]
    if args.impl == 'reference':
        rank = int(os.environ.get('RANK', '0'))
        if rank != 0:
            return
        vals = [cpu_step(wl, args.cpu_sample) for _ in range(max(1, min(args.steps, 3)))]
        v = float(np.median([x['value'] for x in vals]))
        base = vals[0]
        base['value'] = v
        print(json.dumps({'impl': 'reference', 'metric': 'train steps/s (forward + backward + fused Adam), fused SH-3 appearance', 'value': v,
                          'unit': 'steps/s', 'n_gpus': args.gpus, 'steps': len(vals), 'warmup': 0, 'ms_per_step': 1000.0 / v,
                          'higher_is_better': True, 'scaling': 'weak', 'vs_baseline': None, 'dtype': 'f32', 'data': 'synthetic',
                          'config': {'workload': 'c1: SH-3 differentiable rasterization fwd+bwd+Adam, 1,000,000 Gaussians, 1 view 1280x720'},
                          'cpu_baseline': base, 'e2e': {'value': v, 'unit': 'steps/s', 'h2d_bytes_per_step': 0, 'd2h_bytes_per_step': 0}}))
        return
    out = run_b200(args, wl)
    if out is not None:
        print(json.dumps(out))


if __name__ == '__main__':
    main()
