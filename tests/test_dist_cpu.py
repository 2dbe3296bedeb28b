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
