"""The benchmark's roofline model (bench.py) on the CPU: the algorithmic bytes it divides by a stage's time are the
per-unit figures of the kernel table (visible rows V, tile instances I, pixels P, Gaussians N of one view), so that a
change to a formula that would inflate a reported fraction fails here; and the launch count the line claims."""
import sys
from pathlib import Path

import pytest

sys.path.insert(0, str(Path(__file__).resolve().parents[1]))
import bench  # noqa: E402

# view 0 of the c4 benchmark scene (Morton order), as the bench line reports it
V, I = 2_836_253, 10_365_001
N, P, F = 6_000_000, 1920 * 1080, 32


@pytest.fixture
def c4():
    wl = bench.WORKLOADS['c4']
    return bench.frame_stats(wl, V, I, N * 46, clear_share=1.0 / 8)


def test_c4_units(c4):
    assert c4['tiles'] == 120 * 90 and c4['key_bytes'] == 2
    assert c4['appearance_bytes'] == 0 and c4['features'] == F
    assert c4['store_bytes'] == 2 * 128 + 8  # two hidden layers of 64 fp16 activations, the two raw outputs
    assert c4['mlp_flops'] == 2 * (80 * 64 + 64 * 64 + 64 * 16)


def test_c4_stage_bytes(c4):
    per_row_geometry = 4 + 4 + 48 + 48 + 44 + 12 + 8 + 80 + 2 * (44 + 12)   # 360
    per_row_mlp_bwd = 4 + 4 * F + 264 + 80 + 8 * F + 24                     # 756
    expect = {
        'preprocess': N * 44 + N * 8 + V * 52,                  # no latent: the colour pass reads it
        'compaction': N * 8 + V * 8,
        'appearance_mlp': V * (4 + 12 + 4 * F + 12 + 12) + V * 264,
        'depth_sort': 4 * V * 16,
        'emit': V * 52 + I * (2 + 4),
        'tile_sort': 2 * I * (2 + 4) * 2,
        'blend_forward': I * 52 + P * 20,
        'loss': 3 * P * 44,
        'blend_backward': I * 52 + P * 32 + V * 48,
        # visible rows only, plus an eighth of the clearing memsets of all N rows (the first of the 8 views clears)
        'preprocess_backward': V * (per_row_geometry + per_row_mlp_bwd) + N * (56 + 4 * F) / 8,
        'adam': 28 * N * 46,
    }
    for stage, b in expect.items():
        assert bench.stage_bytes(stage, c4) == pytest.approx(b, rel=1e-12), stage
    assert per_row_geometry + per_row_mlp_bwd == 1116


def test_single_view_clears_every_view():
    wl = bench.WORKLOADS['c2']
    s1 = bench.frame_stats(wl, 500_000, 1_500_000, 1)
    s8 = bench.frame_stats(wl, 500_000, 1_500_000, 1, clear_share=1.0 / 8)
    diff = bench.stage_bytes('preprocess_backward', s1) - bench.stage_bytes('preprocess_backward', s8)
    assert diff == pytest.approx(wl['n'] * (56 + 4 * 32) * (1 - 1 / 8))


def test_tensor_flops(c4):
    assert bench.stage_flops('appearance_mlp', c4) == V * c4['mlp_flops']
    assert bench.stage_flops('preprocess_backward', c4) == 2 * V * c4['mlp_flops']
    assert bench.stage_flops('blend_backward', c4) == 0


def test_launch_counts():
    per_view = bench.RENDER_LAUNCHES_PER_VIEW
    assert per_view == 31
    assert bench.own_launches('c4', 8) == (per_view + 7) * 8 + 1
    assert bench.own_launches('c3', 64) == per_view * 64
    assert bench.own_launches('c1', 1) == per_view + 3
