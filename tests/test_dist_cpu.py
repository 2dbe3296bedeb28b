"""Data-parallel exchange step on CPU ranks (gloo, world size 2): gradients reduced by Gaussian range (a reduce-scatter
per parameter group, an all-reduce of the MLP weights), Adam on each rank's Gaussian range (the checker's float Adam,
same operations as the kernel) and the ranges gathered back give bit-identical parameters to a single process applying
Adam to the summed gradients. Also a rank that fails before the collective makes the others fail with an error
instead of hanging (short process-group timeout); and the rank-count rule of the multicast exchange."""
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


def _prims(n=1001, feat=7):
    g = torch.Generator().manual_seed(0)
    return {'means': torch.randn(n, 3, generator=g), 'scales': torch.randn(n, 3, generator=g), 'rotations': torch.randn(n, 4, generator=g),
            'opacities': torch.randn(n, 1, generator=g), 'base_colors': torch.randn(n, 3, generator=g),
            'residual_params': torch.randn(n, 8, feat, generator=g), 'mlp_weights': torch.randn(1234, generator=g)}


LRS = {'means': 1.6e-4, 'scales': 0.005, 'rotations': 0.001, 'opacities': 0.05, 'base_colors': 0.00025,
       'residual_params': [0.002] * 3 + [0.006] + [0.0008] * 3, 'mlp_weights': 0.003}


def _grads(trainer, rank, step, fill=True):
    """Per-group random gradients of one rank and step (padding rows of the flat buffer stay zero)."""
    g = torch.Generator().manual_seed(1000 * step + rank)
    out = {}
    for grp in trainer.groups:
        out[grp.name] = torch.randn(grp.shape, generator=g)
        if fill:
            trainer.view(trainer.grads, grp.name).copy_(out[grp.name])
    return out


def _worker(rank, world, port, out_dir):
    for p in (str(ROOT), str(ROOT / 'efficient-gaussian-appearance_b200'), str(ROOT / 'tests')):
        sys.path.insert(0, p)
    import datetime
    os.environ['MASTER_ADDR'] = '127.0.0.1'
    os.environ['MASTER_PORT'] = str(port)
    torch.distributed.init_process_group('gloo', rank=rank, world_size=world, timeout=datetime.timedelta(seconds=30))
    from trainer import Trainer
    t = Trainer(_prims(), LRS, torch.device('cpu'), group=torch.distributed.group.WORLD)
    assert t.rows * world >= t.n and t.rows % 4 == 0
    for step in range(3):
        _grads(t, rank, step)
        t.apply_gradients(adam_fn=_oracle_adam)
    torch.save({g.name: t.view(t.params, g.name).clone() for g in t.groups}, os.path.join(out_dir, f'params_{rank}.pt'))
    torch.distributed.destroy_process_group()


def test_sharded_adam_matches_single_process(tmp_path):
    for p in (str(ROOT), str(ROOT / 'efficient-gaussian-appearance_b200')):
        if p not in sys.path:
            sys.path.insert(0, p)
    from trainer import Trainer
    world = 2
    port = _free_port()
    mp.start_processes(_worker, args=(world, port, str(tmp_path)), nprocs=world, start_method='spawn', join=True)
    # single process: the gradients summed over the ranks
    ref = Trainer(_prims(), LRS, torch.device('cpu'))
    for step in range(3):
        parts = [_grads(ref, rank, step, fill=False) for rank in range(world)]
        for grp in ref.groups:
            ref.view(ref.grads, grp.name).copy_(parts[0][grp.name] + parts[1][grp.name])
        ref.apply_gradients(adam_fn=_oracle_adam)
    p0 = torch.load(tmp_path / 'params_0.pt')
    p1 = torch.load(tmp_path / 'params_1.pt')
    for grp in ref.groups:
        assert torch.equal(p0[grp.name], p1[grp.name]), grp.name
        assert torch.equal(p0[grp.name], ref.view(ref.params, grp.name)), grp.name


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


def _moments(name, rows_total, cols, sign):
    """A known full moment tensor of one group: row-major counting values (negated for the second moment)."""
    base = {'means': 0, 'scales': 1e5, 'rotations': 2e5, 'opacities': 3e5, 'base_colors': 4e5, 'residual_params': 5e5}[name]
    return sign * (base + torch.arange(rows_total * cols, dtype=torch.float32)).view(rows_total, cols)


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
    groups = [g for g in t.groups if g.name != 'mlp_weights']
    for g in groups:
        for buf, sign in ((t.exp_avg, 1.0), (t.exp_avg_sq, -1.0)):
            t.shard_view(buf, g.name).copy_(_moments(g.name, t.rows * world, g.cols, sign)[rank * t.rows:(rank + 1) * t.rows])
    t.apply_morton_ordering()
    torch.save({'params': {g.name: t.view(t.params, g.name).clone() for g in t.groups},
                'm': {g.name: t.shard_view(t.exp_avg, g.name).clone() for g in groups},
                'v': {g.name: t.shard_view(t.exp_avg_sq, g.name).clone() for g in groups}}, os.path.join(out_dir, f'morton_{rank}.pt'))
    torch.distributed.destroy_process_group()


def test_morton_ordering_two_ranks_matches_single_process(tmp_path):
    """Every rank holds only its Gaussian range of the Adam moments: the ordering gathers them, permutes every
    per-Gaussian group (the MLP weights stay) and hands each rank its range again, as one process permuting everything
    would (the first N rows; the ranges' padding rows differ between the layouts and are not used)."""
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
        groups = [g for g in ref.groups if g.name != 'mlp_weights']
        for g in groups:
            ref.shard_view(ref.exp_avg, g.name).copy_(_moments(g.name, ref.rows, g.cols, 1.0))
            ref.shard_view(ref.exp_avg_sq, g.name).copy_(_moments(g.name, ref.rows, g.cols, -1.0))
        ref.apply_morton_ordering()
    finally:
        T.morton_order = saved
    n = ref.n
    for g in ref.groups:
        assert torch.equal(parts[0]['params'][g.name], parts[1]['params'][g.name])
        assert torch.equal(parts[0]['params'][g.name], ref.view(ref.params, g.name))
    for g in groups:
        for key, buf in (('m', ref.exp_avg), ('v', ref.exp_avg_sq)):
            dist = torch.cat([p[key][g.name] for p in parts])[:n]
            assert torch.equal(dist, ref.shard_view(buf, g.name)[:n]), (key, g.name)
    means = _prims()['means']
    assert torch.equal(ref.view(ref.params, 'means'), means[_position_order(means)])


def test_multicast_choice_by_rank_count():
    """The peer exchange reads and writes through NVSwitch multicast from trainer.MULTICAST_MIN_RANKS ranks on by
    default (measured: peer loads and stores faster at 2 GPUs, multicast at 8); True and False force either."""
    sys.path.insert(0, str(ROOT / 'efficient-gaussian-appearance_b200'))
    import trainer as T
    assert T.MULTICAST_MIN_RANKS == 5
    assert [T.multicast_wanted('auto', w) for w in (1, 2, 4, 5, 8)] == [False, False, False, True, True]
    assert T.multicast_wanted(True, 2) and not T.multicast_wanted(False, 8)
    with pytest.raises(ValueError):
        T.multicast_wanted('yes', 8)
