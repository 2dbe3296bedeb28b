"""Data-parallel exchange on 2 GPUs: the fused peer-memory kernel (fgs_dp_shard_adam over symmetric memory) against
NCCL reduce-scatter + fused Adam + all-gather, from the same state and gradients. Needs two visible GPUs (skipped
otherwise); the ranks run as spawned processes over NCCL on 127.0.0.1."""
import os
import socket

import pytest
import torch

pytestmark = pytest.mark.gpu


def _worker(rank: int, world: int, port: int, mode: str, out_path: str) -> None:
    import datetime
    import sys
    sys.path.insert(0, os.path.join(os.path.dirname(__file__), '..', 'efficient-gaussian-appearance_b200'))
    os.environ.update(MASTER_ADDR='127.0.0.1', MASTER_PORT=str(port), RANK=str(rank), WORLD_SIZE=str(world), NCCL_NVLS_ENABLE='0')
    torch.cuda.set_device(rank)
    dev = torch.device('cuda', rank)
    torch.distributed.init_process_group('nccl', timeout=datetime.timedelta(seconds=60), device_id=dev)
    try:
        from trainer import Trainer
        g = torch.Generator().manual_seed(1)
        n = 5000
        prims = {'means': torch.randn(n, 3, generator=g), 'scales': torch.randn(n, 3, generator=g), 'rotations': torch.randn(n, 4, generator=g),
                 'opacities': torch.randn(n, 1, generator=g), 'base_colors': torch.randn(n, 3, generator=g),
                 'residual_params': torch.randn(n, 45, generator=g)}
        lrs = {'means': 1e-3, 'scales': 5e-3, 'rotations': 1e-3, 'opacities': 5e-2, 'base_colors': 2.5e-3, 'residual_params': [1e-3, 2e-3, 3e-3]}
        mc = mode == 'peer-mc'
        tr = Trainer({k: v.to(dev) for k, v in prims.items()}, lrs, dev, group=torch.distributed.group.WORLD,
                     exchange='peer' if mc else mode, multicast=mc)
        assert tr.exchange == ('peer' if mc else mode), (tr.exchange, getattr(tr, 'exchange_error', ''))
        if mc and not tr.multicast:  # no multicast mapping on this system: nothing to compare
            torch.save(None, out_path + f'.{mode}.{rank}')
            return
        gr = torch.Generator().manual_seed(100 + rank)
        for _ in range(2):  # two steps: moments carried over
            tr.grads.copy_(torch.randn(tr.total, generator=gr).to(dev))
            tr.apply_gradients()
        torch.cuda.synchronize()
        torch.save(tr.params.cpu(), out_path + f'.{mode}.{rank}')
    finally:
        torch.distributed.destroy_process_group()


def _free_port() -> int:
    s = socket.socket()
    s.bind(('127.0.0.1', 0))
    port = s.getsockname()[1]
    s.close()
    return port


@pytest.mark.skipif(not torch.cuda.is_available() or torch.cuda.device_count() < 2, reason='needs two GPUs')
@pytest.mark.parametrize('mode', ['peer', 'peer-mc'])
def test_peer_exchange_matches_nccl(tmp_path, mode):
    import torch.multiprocessing as mp
    out = str(tmp_path / 'params')
    for m in ('nccl', mode):
        mp.spawn(_worker, args=(2, _free_port(), m, out), nprocs=2, join=True)
    if torch.load(out + f'.{mode}.0') is None:
        pytest.skip('no NVLink multicast mapping on this system')
    for r in range(2):
        a, b = torch.load(out + f'.nccl.{r}'), torch.load(out + f'.{mode}.{r}')
        err = float((a - b).abs().max())
        assert err <= 1e-5 * float(a.abs().max()), err
    # both ranks hold identical parameters after the all-gather
    assert torch.equal(torch.load(out + f'.{mode}.0'), torch.load(out + f'.{mode}.1'))
