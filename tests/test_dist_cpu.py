"""Data-parallel exchange step on CPU ranks (gloo, world size 2): reduce-scatter of the flat gradient buffer, Adam on
each rank's slice (the checker's float Adam, same operations as the kernel) and all-gather of the parameters give
bit-identical parameters to a single process applying Adam to the summed gradients. Also a rank that fails before
the collective makes the others fail with an error instead of hanging (short process-group timeout)."""
import os
import socket
import sys
from pathlib import Path

import numpy as np
import pytest
import torch
import torch.multiprocessing as mp

ROOT = Path(__file__).resolve().parent.parent


def _free_port() -> int:
    s = socket.socket()
    s.bind(('127.0.0.1', 0))
    port = s.getsockname()[1]
    s.close()
    return port


def _oracle_adam(segments):
    from oracle import oracle as O
    import ctypes
    lib = O.load(False)
    for seg in segments:
        lrs = (ctypes.c_double * 7)(*[seg.learning_rates[i] for i in range(7)])
        lib.orc_adam(seg.n_elements, seg.param, seg.grad, seg.exp_avg, seg.exp_avg_sq, seg.step, lrs, seg.n_learning_rates, seg.column_offset,
                     seg.beta1, seg.beta2, seg.eps)


def _prims(n=1000, feat=7):
    g = torch.Generator().manual_seed(0)
    return {'means': torch.randn(n, 3, generator=g), 'scales': torch.randn(n, 3, generator=g), 'rotations': torch.randn(n, 4, generator=g),
            'opacities': torch.randn(n, 1, generator=g), 'base_colors': torch.randn(n, 3, generator=g),
            'residual_params': torch.randn(n, 8, feat, generator=g), 'mlp_weights': torch.randn(1234, generator=g)}


LRS = {'means': 1.6e-4, 'scales': 0.005, 'rotations': 0.001, 'opacities': 0.05, 'base_colors': 0.00025,
       'residual_params': [0.002] * 3 + [0.006] + [0.0008] * 3, 'mlp_weights': 0.003}


def _grads(trainer, rank, step):
    g = torch.Generator().manual_seed(1000 * step + rank)
    trainer.grads.copy_(torch.randn(trainer.total, generator=g))


def _worker(rank, world, port, out_dir):
    for p in (str(ROOT), str(ROOT / 'efficient-gaussian-appearance_b200'), str(ROOT / 'tests')):
        sys.path.insert(0, p)
    import datetime
    os.environ['MASTER_ADDR'] = '127.0.0.1'
    os.environ['MASTER_PORT'] = str(port)
    torch.distributed.init_process_group('gloo', rank=rank, world_size=world, timeout=datetime.timedelta(seconds=30))
    from trainer import Trainer
    t = Trainer(_prims(), LRS, torch.device('cpu'), group=torch.distributed.group.WORLD)
    for step in range(3):
        _grads(t, rank, step)
        t.apply_gradients(adam_fn=_oracle_adam)
    torch.save(t.params.clone(), os.path.join(out_dir, f'params_{rank}.pt'))
    torch.distributed.destroy_process_group()


def test_sharded_adam_matches_single_process(tmp_path):
    for p in (str(ROOT), str(ROOT / 'efficient-gaussian-appearance_b200')):
        if p not in sys.path:
            sys.path.insert(0, p)
    from trainer import Trainer
    world = 2
    port = _free_port()
    mp.start_processes(_worker, args=(world, port, str(tmp_path)), nprocs=world, start_method='spawn', join=True)
    # single process: same flat layout (padded for 2 ranks), gradients summed over the ranks
    ref = Trainer(_prims(), LRS, torch.device('cpu'))
    dist_total = (ref.total + 64 * world - 1) // (64 * world) * (64 * world)
    for step in range(3):
        total = None
        for rank in range(world):
            g = torch.Generator().manual_seed(1000 * step + rank)
            x = torch.randn(dist_total, generator=g)
            total = x if total is None else total + x
        # the distributed run pads the flat buffer to a multiple of 64 * world; use the same prefix
        ref.grads.copy_(total[:ref.total])
        ref.apply_gradients(adam_fn=_oracle_adam)
    p0 = torch.load(tmp_path / 'params_0.pt')
    p1 = torch.load(tmp_path / 'params_1.pt')
    assert torch.equal(p0, p1)
    n = ref.total
    assert torch.equal(p0[:n], ref.params[:n])


def _failing_worker(rank, world, port):
    import datetime
    os.environ['MASTER_ADDR'] = '127.0.0.1'
    os.environ['MASTER_PORT'] = str(port)
    torch.distributed.init_process_group('gloo', rank=rank, world_size=world, timeout=datetime.timedelta(seconds=5))
    if rank == 1:
        raise RuntimeError('rank 1 fails before the exchange step')
    x = torch.ones(16)
    out = torch.empty(8)
    try:
        torch.distributed.reduce_scatter_tensor(out, x)
    except Exception:
        os._exit(3)  # the surviving rank sees an error instead of waiting forever
    os._exit(0)


def test_failed_rank_surfaces_as_error():
    port = _free_port()
    ctx = mp.get_context('spawn')
    procs = [ctx.Process(target=_failing_worker, args=(r, 2, port)) for r in range(2)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(timeout=120)
    assert all(not p.is_alive() for p in procs)
    assert procs[1].exitcode != 0
    assert procs[0].exitcode == 3


def _position_order(means: torch.Tensor) -> torch.Tensor:
    """Stand-in for the Morton order on CPU ranks (the codes come from a GPU kernel): any fixed permutation of the
    Gaussians exercises the same gather / permute / re-slice logic."""
    m = means.reshape(-1, 3)
    return torch.argsort(m[:, 0] + 0.37 * m[:, 1] - 0.11 * m[:, 2], stable=True)


def _morton_worker(rank, world, port, out_dir):
    for p in (str(ROOT), str(ROOT / 'efficient-gaussian-appearance_b200'), str(ROOT / 'tests')):
        sys.path.insert(0, p)
    import datetime
    os.environ['MASTER_ADDR'] = '127.0.0.1'
    os.environ['MASTER_PORT'] = str(port)
    torch.distributed.init_process_group('gloo', rank=rank, world_size=world, timeout=datetime.timedelta(seconds=30))
    import trainer as T
    T.morton_order = _position_order
    t = T.Trainer(_prims(), LRS, torch.device('cpu'), group=torch.distributed.group.WORLD)
    lo = rank * t.shard
    t.exp_avg.copy_(torch.arange(lo, lo + t.shard, dtype=torch.float32))
    t.exp_avg_sq.copy_(-torch.arange(lo, lo + t.shard, dtype=torch.float32))
    t.apply_morton_ordering()
    torch.save({'params': t.params.clone(), 'm': t.exp_avg.clone(), 'v': t.exp_avg_sq.clone(), 'shard': t.shard},
               os.path.join(out_dir, f'morton_{rank}.pt'))
    torch.distributed.destroy_process_group()


def test_morton_ordering_two_ranks_matches_single_process(tmp_path):
    """Every rank holds only its slice of the Adam moments: the ordering gathers them, permutes every per-Gaussian
    group (the MLP weights stay) and hands each rank its slice again, as one process permuting everything would."""
    for p in (str(ROOT), str(ROOT / 'efficient-gaussian-appearance_b200')):
        if p not in sys.path:
            sys.path.insert(0, p)
    import trainer as T
    world = 2
    mp.start_processes(_morton_worker, args=(world, _free_port(), str(tmp_path)), nprocs=world, start_method='spawn', join=True)
    parts = [torch.load(tmp_path / f'morton_{r}.pt') for r in range(world)]
    saved, T.morton_order = T.morton_order, _position_order
    try:
        ref = T.Trainer(_prims(), LRS, torch.device('cpu'))
        ref.exp_avg.copy_(torch.arange(ref.shard, dtype=torch.float32))
        ref.exp_avg_sq.copy_(-torch.arange(ref.shard, dtype=torch.float32))
        ref.apply_morton_ordering()
    finally:
        T.morton_order = saved
    n = sum((g.numel + 63) // 64 * 64 for g in ref.groups)
    assert torch.equal(parts[0]['params'], parts[1]['params'])
    assert torch.equal(parts[0]['params'][:n], ref.params[:n])
    m = torch.cat([p['m'] for p in parts])
    v = torch.cat([p['v'] for p in parts])
    assert torch.equal(m[:n], ref.exp_avg[:n]) and torch.equal(v[:n], ref.exp_avg_sq[:n])
    means = _prims()['means']
    g = next(x for x in ref.groups if x.name == 'means')
    assert torch.equal(ref.params[g.offset:g.offset + g.numel].view(-1, 3), means[_position_order(means)])
