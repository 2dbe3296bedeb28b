"""ctypes binding of libfgs_b200.so (declarations in include/fgs_b200.h).

The library is the only compute path: if it is missing, importing this module raises ImportError; there is
no CPU fallback.
"""
import ctypes
import os
from pathlib import Path

_LIB_PATH = Path(os.environ.get('FGS_B200_LIB', Path(__file__).resolve().parent / 'lib' / 'libfgs_b200.so'))

if not _LIB_PATH.exists():
    raise ImportError(f'libfgs_b200.so not found at {_LIB_PATH}; build it with `python efficient-gaussian-appearance_b200/build.py` '
                      f'(or __graft_entry__.build())')

lib = ctypes.CDLL(str(_LIB_PATH))

c_int, c_int32, c_int64, c_size_t, c_void_p, c_float, c_double = (ctypes.c_int, ctypes.c_int32, ctypes.c_int64, ctypes.c_size_t,
                                                                   ctypes.c_void_p, ctypes.c_float, ctypes.c_double)
c_float_p = ctypes.POINTER(ctypes.c_float)


class Primitives(ctypes.Structure):
    _fields_ = [('means', c_void_p), ('scales', c_void_p), ('rotations', c_void_p), ('opacities', c_void_p),
                ('precomputed_colors', c_void_p), ('base_colors', c_void_p), ('residual_params', c_void_p),
                ('mlp_weights', c_void_p), ('n_primitives', c_int64)]


class Settings(ctypes.Structure):
    _fields_ = [('w2c', c_void_p), ('cam_position', c_void_p), ('bg_color', c_void_p), ('appearance_degree', c_int),
                ('width', c_int), ('height', c_int), ('focal_x', c_float), ('focal_y', c_float), ('center_x', c_float),
                ('center_y', c_float), ('near_plane', c_float), ('far_plane', c_float), ('proper_antialiasing', c_int),
                ('render_base', c_int), ('render_residual', c_int)]


class Frame(ctypes.Structure):
    _fields_ = [('n_primitives', c_int64), ('n_visible', c_int64), ('n_instances', c_int64), ('n_buckets', c_int64),
                ('width', c_int32), ('height', c_int32), ('grid_w', c_int32), ('grid_h', c_int32), ('end_bit', c_int32),
                ('wide_keys', c_int32), ('depth_selector', c_int32), ('tile_selector', c_int32), ('precomputed', c_int32),
                ('mlp_activations', c_int32)]


class Gradients(ctypes.Structure):
    _fields_ = [('means', c_void_p), ('scales', c_void_p), ('rotations', c_void_p), ('opacities', c_void_p),
                ('precomputed_colors', c_void_p), ('base_colors', c_void_p), ('residual_params', c_void_p),
                ('mlp_weights', c_void_p)]


class FrameViews(ctypes.Structure):
    _fields_ = [(name, c_void_p) for name in (
        'n_touched', 'depth_keys', 'sorted_indices', 'rank_of', 'sorted_records', 'instance_offsets', 'instance_keys',
        'instance_ranks', 'tile_ranges', 'bucket_offsets', 'tile_max_contributors', 'final_transmittance', 'n_contributors')]


class AdamSegment(ctypes.Structure):
    _fields_ = [('param', c_void_p), ('grad', c_void_p), ('exp_avg', c_void_p), ('exp_avg_sq', c_void_p),
                ('n_elements', c_int64), ('column_offset', c_int64), ('step', c_int64), ('learning_rates', c_double * 7),
                ('n_learning_rates', c_int32), ('beta1', c_double), ('beta2', c_double), ('eps', c_double)]


class PeerBuffers(ctypes.Structure):
    _fields_ = [('n_ranks', c_int), ('grads', c_void_p * 8), ('params', c_void_p * 8), ('local_params', c_void_p),
                ('multicast_grads', c_void_p), ('multicast_params', c_void_p)]


_P = ctypes.POINTER
PROTOTYPES = {
    'fgs_last_error': (ctypes.c_char_p, []),
    'fgs_version': (c_int, []),
    'fgs_rasterizer_create': (c_int, [_P(c_void_p)]),
    'fgs_rasterizer_destroy': (c_int, [c_void_p]),
    'fgs_set_appearance': (c_int, [c_void_p, c_int, c_int, c_int, c_int, c_int, c_int]),
    'fgs_set_residual_mlp': (c_int, [c_void_p, c_int, c_int, c_int, c_int, c_int, c_int, c_int, c_int]),
    'fgs_mlp_param_count': (c_int, [c_void_p, _P(c_int64)]),
    'fgs_residual_stride': (c_int, [c_void_p, _P(c_int64)]),
    'fgs_primitive_workspace_bytes': (c_int, [c_void_p, c_int64, _P(c_size_t)]),
    'fgs_tile_workspace_bytes': (c_int, [c_int, c_int, _P(c_size_t)]),
    'fgs_instance_workspace_bytes': (c_int, [c_int64, c_int, c_int, _P(c_size_t)]),
    'fgs_bucket_workspace_bytes': (c_int, [c_int64, _P(c_size_t)]),
    'fgs_gradient_workspace_bytes': (c_int, [c_void_p, c_int64, _P(c_size_t)]),
    'fgs_forward_preprocess': (c_int, [c_void_p, _P(Primitives), _P(Settings), c_void_p, c_size_t, c_void_p, _P(Frame)]),
    'fgs_forward_render': (c_int, [c_void_p, _P(Settings), _P(Frame), c_void_p, c_void_p, c_size_t, c_void_p, c_size_t, c_void_p,
                                   c_size_t, c_void_p, c_void_p]),
    'fgs_inference_render': (c_int, [c_void_p, _P(Settings), _P(Frame), c_void_p, c_void_p, c_size_t, c_void_p, c_size_t, c_void_p,
                                     c_int, c_int, c_void_p]),
    'fgs_backward': (c_int, [c_void_p, _P(Primitives), _P(Settings), _P(Frame), c_void_p, c_void_p, c_void_p, c_void_p, c_void_p,
                             c_size_t, c_void_p, c_void_p, _P(Gradients), c_void_p, c_int, c_int, c_void_p]),
    'fgs_frame_buffers': (c_int, [_P(Frame), c_void_p, c_void_p, c_void_p, _P(FrameViews)]),
    'fgs_pruning_scores': (c_int, [_P(Settings), _P(Frame), c_void_p, c_void_p, c_void_p, c_void_p, c_void_p, c_void_p]),
    'fgs_relocation_adjustment': (c_int, [c_void_p, c_void_p, c_void_p, c_void_p, c_void_p, c_int64, c_void_p]),
    'fgs_add_noise': (c_int, [c_void_p, c_void_p, c_void_p, c_void_p, c_int64, c_float, ctypes.c_uint64, ctypes.c_uint64, c_void_p]),
    'fgs_tc_timeout': (c_int, [_P(c_int), c_int]),
    'fgs_morton_codes': (c_int, [c_void_p, c_int64, _P(c_float), _P(c_float), c_void_p, c_void_p]),
    'fgs_update_3d_filter': (c_int, [c_void_p, c_void_p, c_void_p, c_void_p, c_int64, c_int, c_int, c_float, c_float, c_float, c_float, c_float,
                                     c_float, c_float, c_float, c_void_p]),
    'fgs_adam_step': (c_int, [_P(AdamSegment), c_int, c_void_p]),
    'fgs_profile_enable': (c_int, [c_int]),
    'fgs_inference_noalloc': (c_int, [c_void_p, _P(Primitives), _P(Settings), c_void_p, c_int, c_int, c_void_p, _P(c_int64), _P(c_int64)]),
    'fgs_profile_collect': (c_int, [ctypes.c_char_p, c_size_t, _P(c_double), c_int, _P(c_int)]),
    'fgs_loss_workspace_bytes': (c_int, [c_int, c_int, c_int, _P(c_size_t)]),
    'fgs_tc_selftest': (c_int, [c_void_p, _P(c_int), c_void_p]),
    'fgs_dp_shard_adam': (c_int, [_P(AdamSegment), c_int, _P(PeerBuffers), c_void_p]),
    'fgs_l1_dssim': (c_int, [c_void_p, c_void_p, c_int, c_int, c_int, ctypes.c_float, ctypes.c_float, c_void_p, c_void_p, c_void_p, c_size_t,
                             c_void_p]),
}

for _name, (_res, _args) in PROTOTYPES.items():
    _fn = getattr(lib, _name)
    _fn.restype = _res
    _fn.argtypes = _args


def check(rc: int) -> None:
    """Raises RuntimeError with the library's message for a non-zero status."""
    if rc != 0:
        raise RuntimeError(lib.fgs_last_error().decode(errors='replace'))


def size_out(fn, *args) -> int:
    out = c_size_t(0)
    check(fn(*args, ctypes.byref(out)))
    return int(out.value)


def ptr(t) -> int | None:
    """Device pointer of a tensor, or None for an empty / absent tensor."""
    if t is None or t.numel() == 0:
        return None
    return t.data_ptr()


def profile_enable(enabled: bool) -> None:
    check(lib.fgs_profile_enable(int(bool(enabled))))


def profile_collect() -> dict[str, float]:
    """Milliseconds per stage recorded since the last collect (waits for the recorded events)."""
    names = ctypes.create_string_buffer(4096)
    ms = (c_double * 64)()
    n = c_int(0)
    check(lib.fgs_profile_collect(names, 4096, ms, 64, ctypes.byref(n)))
    keys = names.value.decode().split(',') if n.value else []
    return {k: float(ms[i]) for i, k in enumerate(keys)}
