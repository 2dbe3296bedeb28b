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


def _scene_and_views(n=60000, views=8, W=320, H=192):
    import synthetic as S
    from trainer import blur
    shapes = S.mlp_layer_shapes(80, 64, 2)
    prims = {**S.geometry(n, seed=21), **S.neural_appearance(n, 32, layer_shapes=shapes, seed=22)}
    cams = S.ring_cameras(views, W, H)
    g = torch.Generator().manual_seed(2)
    targets = [blur(torch.rand(3, H, W, generator=g), 9, 2.0).contiguous() for _ in range(views)]
    return prims, cams, targets


LRS_C4 = {'means': 1.6e-4, 'scales': 0.005, 'rotations': 0.001, 'opacities': 0.05, 'base_colors': 0.00025, 'residual_params': 0.008,
          'mlp_weights': 0.003}


def _train(rank, world, dev, exchange, group):
    import FasterGSVDACudaBackend as F
    from trainer import Trainer
    F.initialize_appearance('neural', 0, 'none', 'tanh', 'relu', True)
    F.initialize_residual_mlp(80, 3, {'otype': 'Identity'}, {'otype': 'FullyFusedMLP', 'activation': 'ReLU', 'output_activation': 'None',
                                                              'n_neurons': 64, 'n_hidden_layers': 2}, False, 1, [0, 1, 2, 3])
    prims, cams, targets = _scene_and_views()
    # 'peer-mc': the peer exchange through NVSwitch multicast at any rank count (the default 'auto' uses it from
    # trainer.MULTICAST_MIN_RANKS ranks on, so two ranks would otherwise take peer loads and stores)
    tr = Trainer({k: v.to(dev) for k, v in prims.items()}, LRS_C4, dev, group=group, exchange=exchange.split('-')[0],
                 multicast=True if exchange == 'peer-mc' else 'auto')
    per = len(cams) // world
    mine = range(rank * per, (rank + 1) * per)
    settings = [F.RasterizerSettings(cams[v].w2c.to(dev), cams[v].position.to(dev), cams[v].bg.to(dev), 3, cams[v].width, cams[v].height,
                                     cams[v].focal_x, cams[v].focal_y, cams[v].center_x, cams[v].center_y, cams[v].near_plane,
                                     cams[v].far_plane, False, True, True) for v in mine]
    tg = [targets[v].to(dev) for v in mine]
    # step 1 with the accumulated gradients kept (summed over the ranks), then step 2
    tr.backward_views(settings, tg)
    grads = {g.name: tr.view(tr.grads, g.name).detach().clone() for g in tr.groups}
    if world > 1:
        for t in grads.values():
            torch.distributed.all_reduce(t, group=group)
    tr.apply_gradients()
    tr.step(settings, tg)
    torch.cuda.synchronize()
    out = {g.name: tr.view(tr.params, g.name).detach().cpu().clone() for g in tr.groups}
    out.update({'grad_' + k: v.cpu() for k, v in grads.items()})
    return out, tr.exchange


def _dp_worker(rank: int, world: int, port: int, exchange: str, out_path: str) -> None:
    import datetime
    import sys
    root = os.path.join(os.path.dirname(__file__), '..')
    for p in (root, os.path.join(root, 'efficient-gaussian-appearance_b200')):
        sys.path.insert(0, p)
    os.environ.update(MASTER_ADDR='127.0.0.1', MASTER_PORT=str(port), RANK=str(rank), WORLD_SIZE=str(world), NCCL_NVLS_ENABLE='0')
    torch.cuda.set_device(rank)
    dev = torch.device('cuda', rank)
    torch.distributed.init_process_group('nccl', timeout=datetime.timedelta(seconds=120), device_id=dev)
    try:
        params, used = _train(rank, world, dev, exchange, torch.distributed.group.WORLD)
        assert used == exchange.split('-')[0], used
        torch.save(params, out_path + f'.{exchange}.{rank}')
    finally:
        torch.distributed.destroy_process_group()


@pytest.mark.skipif(not torch.cuda.is_available() or torch.cuda.device_count() < 2, reason='needs two GPUs')
@pytest.mark.parametrize('exchange', ['nccl', 'peer', 'peer-mc'])
def test_data_parallel_training_matches_one_gpu(tmp_path, exchange):
    """Two ranks, each rendering 4 of a global batch of 8 Neural views (forward, fused loss, backward), exchanging
    gradients by Gaussian range and applying Adam to their ranges, against one process training on all 8 views: the
    first step's gradients summed over the ranks and the parameters after two steps agree within 1e-3 relative L2 per
    parameter group (the views' gradients are summed in another order), and both ranks hold identical parameters.
    (Adam is invariant to the scale of the gradient, hence the separate gradient comparison.)"""
    import sys
    import torch.multiprocessing as mp
    root = os.path.join(os.path.dirname(__file__), '..')
    for p in (root, os.path.join(root, 'efficient-gaussian-appearance_b200')):
        if p not in sys.path:
            sys.path.insert(0, p)
    out = str(tmp_path / 'params')
    mp.spawn(_dp_worker, args=(2, _free_port(), exchange, out), nprocs=2, join=True)
    ref, _ = _train(0, 1, torch.device('cuda', 0), 'nccl', None)
    p0, p1 = torch.load(out + f'.{exchange}.0'), torch.load(out + f'.{exchange}.1')
    for k, want in ref.items():
        assert torch.equal(p0[k], p1[k]), k
        err = float((p0[k] - want).norm() / want.norm())
        print(f'[dp {exchange}] {k} rel {err:.2e}')
        assert err <= 1e-3, (k, err)
