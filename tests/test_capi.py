"""The C-ABI library loads without a GPU, exports every symbol include/fgs_b200.h declares, and validates its
arguments with error codes and messages (no compute calls)."""
import ctypes
import re
from pathlib import Path

import pytest

ROOT = Path(__file__).resolve().parent.parent


def _declared_symbols():
    text = (ROOT / 'include' / 'fgs_b200.h').read_text()
    return sorted(set(re.findall(r'^\s*(?:int|const char\*|void)\s+(fgs_\w+)\s*\(', text, re.M)))


def test_library_exports_header_symbols():
    from FasterGSVDACudaBackend import _lib
    names = _declared_symbols()
    assert len(names) >= 18
    for n in names:
        assert hasattr(_lib.lib, n), n


def test_argument_validation_without_gpu():
    import FasterGSVDACudaBackend as F
    from FasterGSVDACudaBackend import rasterization as R
    with pytest.raises(RuntimeError, match='invalid appearance model id'):
        R._rasterizer.set_appearance(9, 3, 0, 0, 1, True)
    with pytest.raises(RuntimeError, match='invalid color activation id'):
        R._rasterizer.set_appearance(1, 3, 0, 0, 9, True)
    with pytest.raises(RuntimeError, match='must select the neural appearance'):
        F.initialize_appearance('sh', 3, 'none', 'none', 'relu', True)
        F.initialize_residual_mlp(32, 3, {'otype': 'Identity'}, {'otype': 'FullyFusedMLP', 'activation': 'ReLU', 'output_activation': 'None',
                                                                  'n_neurons': 16, 'n_hidden_layers': 2}, False, 1, [0, 1, 2, 3])
    F.initialize_appearance('neural', 0, 'none', 'tanh', 'relu', True)
    F.initialize_residual_mlp(32, 3, {'otype': 'Identity'}, {'otype': 'FullyFusedMLP', 'activation': 'ReLU', 'output_activation': 'None',
                                                              'n_neurons': 16, 'n_hidden_layers': 2}, False, 1, [0, 1, 2, 3])
    assert R._rasterizer.n_mlp_params == 16 * 32 + 16 * 16 + 16 * 16
    assert R._rasterizer.residual_stride == 8
    F.initialize_appearance('sv', 7, 'none', 'none', 'relu', True)
    assert R._rasterizer.residual_stride == 49


def test_workspace_queries():
    from FasterGSVDACudaBackend._lib import lib, size_out
    from FasterGSVDACudaBackend import rasterization as R
    a = size_out(lib.fgs_primitive_workspace_bytes, R._rasterizer.handle, 1000)
    b = size_out(lib.fgs_primitive_workspace_bytes, R._rasterizer.handle, 2000)
    assert 0 < a < b
    assert size_out(lib.fgs_tile_workspace_bytes, 1920, 1080) > 120 * 90 * 192 * 8
    assert size_out(lib.fgs_instance_workspace_bytes, 10, 64, 48) > 0
    with pytest.raises(RuntimeError):
        size_out(lib.fgs_tile_workspace_bytes, 0, 10)


def test_workspace_activation_store_size():
    """A rasterizer whose Neural MLP runs on the tensor cores (64 neurons) sizes the primitive workspace with the
    activation store: per 128-row tile one 16 KB block per hidden layer, 1 KB of raw outputs and the 80-byte row block
    of each row (filled by the geometry pass of the warp-specialised backward), after the other buffers (one 256-byte
    alignment step at most); NULL, SH and 16-wide networks size it without."""
    import FasterGSVDACudaBackend as F
    from FasterGSVDACudaBackend._lib import lib, size_out
    from FasterGSVDACudaBackend import rasterization as R
    n = 100_000
    tiles = (n + 127) // 128
    for hidden in (1, 2, 3):
        F.initialize_appearance('neural', 0, 'none', 'tanh', 'relu', True)
        F.initialize_residual_mlp(80, 3, {'otype': 'Identity'}, {'otype': 'FullyFusedMLP', 'activation': 'ReLU', 'output_activation': 'None',
                                                                  'n_neurons': 64, 'n_hidden_layers': hidden}, False, 1, [0, 1, 2, 3])
        with_store = size_out(lib.fgs_primitive_workspace_bytes, R._rasterizer.handle, n)
        without = size_out(lib.fgs_primitive_workspace_bytes, None, n)
        extra = with_store - without
        store = tiles * (hidden * 128 * 64 * 2 + 128 * 8 + 128 * 80)
        assert store <= extra < store + 256, (hidden, extra, store)
    F.initialize_residual_mlp(80, 3, {'otype': 'Identity'}, {'otype': 'FullyFusedMLP', 'activation': 'ReLU', 'output_activation': 'None',
                                                              'n_neurons': 16, 'n_hidden_layers': 2}, False, 1, [0, 1, 2, 3])
    assert size_out(lib.fgs_primitive_workspace_bytes, R._rasterizer.handle, n) == size_out(lib.fgs_primitive_workspace_bytes, None, n)
    F.initialize_appearance('sh', 3, 'none', 'none', 'relu', True)
    assert size_out(lib.fgs_primitive_workspace_bytes, R._rasterizer.handle, n) == size_out(lib.fgs_primitive_workspace_bytes, None, n)
    assert [f[0] for f in F._lib.Frame._fields_][-1] == 'mlp_activations'


def test_settings_field_order_matches_reference():
    import FasterGSVDACudaBackend as F
    assert F.RasterizerSettings._fields == ('w2c', 'cam_position', 'bg_color', 'appearance_degree', 'width', 'height', 'focal_x', 'focal_y',
                                            'center_x', 'center_y', 'near_plane', 'far_plane', 'proper_antialiasing', 'render_base',
                                            'render_residual')


def test_size_validation_rejects_mismatched_tensors():
    import torch
    import FasterGSVDACudaBackend as F
    from FasterGSVDACudaBackend import rasterization as R
    F.initialize_appearance('sh', 3, 'none', 'none', 'relu', True)
    n = 10
    with pytest.raises(ValueError, match='residual_params'):
        R._check_sizes(n, torch.zeros(n, 3), torch.zeros(n, 4), torch.zeros(n, 1), None, torch.zeros(n, 3), torch.zeros(n, 14, 3), None,
                       R._rasterizer)
    with pytest.raises(ValueError, match='rotations'):
        R._check_sizes(n, torch.zeros(n, 3), torch.zeros(n, 3), torch.zeros(n, 1), None, torch.zeros(n, 3), torch.zeros(n, 15, 3), None,
                       R._rasterizer)
    R._check_sizes(n, torch.zeros(n, 3), torch.zeros(n, 4), torch.zeros(n, 1), None, torch.zeros(n, 3), torch.zeros(n, 15, 3), None,
                   R._rasterizer)


def test_noalloc_size_example_fits():
    """The allocation-free entry point's documented example (100,000 primitives at 1280x720 with 1,000,000 tile
    instances) fits its static array, and 1.1M instances do not: the same workspace queries size both."""
    from FasterGSVDACudaBackend._lib import lib, size_out
    limit = 32 * 1024 * 1024
    header = (ROOT / 'include' / 'fgs_b200.h').read_text()
    assert '#define FGS_NOALLOC_SCRATCH_BYTES (32u * 1024u * 1024u)' in header
    rnd = lambda b: (b + 255) // 256 * 256
    base = rnd(size_out(lib.fgs_primitive_workspace_bytes, None, 100_000)) + rnd(size_out(lib.fgs_tile_workspace_bytes, 1280, 720))
    assert base + size_out(lib.fgs_instance_workspace_bytes, 1_000_000, 1280, 720) <= limit
    assert base + size_out(lib.fgs_instance_workspace_bytes, 1_100_000, 1280, 720) > limit
    # the per-item costs the header states
    per_prim = (size_out(lib.fgs_primitive_workspace_bytes, None, 2_000_000) - size_out(lib.fgs_primitive_workspace_bytes, None, 1_000_000)) / 1e6
    per_inst = (size_out(lib.fgs_instance_workspace_bytes, 2_000_000, 1280, 720) - size_out(lib.fgs_instance_workspace_bytes, 1_000_000, 1280, 720)) / 1e6
    assert abs(per_prim - 132.3) < 0.1 and abs(per_inst - 12.25) < 0.01
    assert size_out(lib.fgs_tile_workspace_bytes, 16 * 80, 12 * 60) // (80 * 60) == 1552
