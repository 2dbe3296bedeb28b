"""ctypes front end of the CPU oracle (TEST INFRASTRUCTURE ONLY: imported by tests/, __graft_entry__.smoke() and the
cpu_baseline leg of bench.py, never by the product path).

`run(...)` executes the whole restated pipeline on numpy arrays: preprocess, depth order, binning, forward blend
and (optionally) the backward, returning every intermediate the GPU exposes so tests can compare stage by stage.
"""
from __future__ import annotations

import ctypes
import os
import subprocess
from pathlib import Path

import numpy as np

HERE = Path(__file__).resolve().parent
BUILD = HERE / '_build'

MODEL_IDS = {'precomputed': 0, 'sh': 1, 'sv': 2, 'nasg': 3, 'nasgabor': 4, 'neural': 5}


class View(ctypes.Structure):
    _fields_ = [('w2c', ctypes.c_float * 16), ('cam', ctypes.c_float * 3), ('bg', ctypes.c_float * 3), ('width', ctypes.c_int),
                ('height', ctypes.c_int), ('fx', ctypes.c_float), ('fy', ctypes.c_float), ('cx', ctypes.c_float), ('cy', ctypes.c_float),
                ('near_plane', ctypes.c_float), ('far_plane', ctypes.c_float), ('proper_aa', ctypes.c_int), ('render_base', ctypes.c_int),
                ('degree', ctypes.c_int)]


class Appearance(ctypes.Structure):
    _fields_ = [(n, ctypes.c_int) for n in ('model', 'max_degree', 'base_act', 'res_act', 'color_act', 'dir_grad', 'feature_dim',
                                            'base_input', 'n_freq', 'sh_mask', 'n_input', 'n_input_pad', 'n_neurons', 'n_hidden',
                                            'hidden_act')]


def build() -> None:
    """Compiles the oracle with the committed Makefile (gcc, no GPU needed)."""
    subprocess.run(['make', '-s', '-C', str(HERE)], check=True)


_LIBS: dict[bool, ctypes.CDLL] = {}


def load(double: bool = False) -> ctypes.CDLL:
    if double in _LIBS:
        return _LIBS[double]
    path = BUILD / ('liboracle_f64.so' if double else 'liboracle_f32.so')
    src_mtime = max(p.stat().st_mtime for p in HERE.glob('*.[ch]'))
    if not path.exists() or path.stat().st_mtime < src_mtime:
        build()
    lib = ctypes.CDLL(str(path))
    P = ctypes.c_void_p
    i64 = ctypes.c_int64
    lib.orc_preprocess.argtypes = [P, P, i64, P, P, P, P, P, P, P, P, P, P, P]
    lib.orc_depth_order.argtypes = [i64, P, P, P]
    lib.orc_depth_order.restype = i64
    lib.orc_bin.argtypes = [i64, P, P, ctypes.c_int, ctypes.c_int, P, P, P]
    lib.orc_bin.restype = i64
    lib.orc_count_instances.argtypes = [i64, P, P]
    lib.orc_count_instances.restype = i64
    lib.orc_blend.argtypes = [i64, P, P, P, P, P, P, P, P, ctypes.c_int, ctypes.c_int]
    lib.orc_blend_backward.argtypes = [i64, P, P, P, P, P, P, P, P]
    lib.orc_pruning_scores.argtypes = [i64, P, P, P, P, P, P, P]
    lib.orc_set_threads.argtypes = [ctypes.c_int]
    lib.orc_threads.restype = ctypes.c_int
    lib.orc_preprocess_backward.argtypes = [P, P, i64, P, P, P, P, P, P, P, P, P, P, P, P, P, P, P, P, P, P, P, P, ctypes.c_int]
    lib.orc_adam.argtypes = [i64, P, P, P, P, i64, P, ctypes.c_int, i64, ctypes.c_double, ctypes.c_double, ctypes.c_double]
    lib.orc_adam.restype = None
    for f in ('orc_det_exp', 'orc_det_exp_blend', 'orc_det_log'):
        getattr(lib, f).argtypes = [ctypes.c_float]
        getattr(lib, f).restype = ctypes.c_float
    lib.orc_residual_stride.argtypes = [P]
    lib.orc_det_sincos.argtypes = [ctypes.c_float, P, P]
    lib.orc_det_sincos.restype = None
    _LIBS[double] = lib
    return lib


def _p(a: np.ndarray | None):
    return None if a is None else a.ctypes.data_as(ctypes.c_void_p)


def _f32(a) -> np.ndarray | None:
    if a is None:
        return None
    if hasattr(a, 'detach'):
        a = a.detach().cpu().numpy()
    return np.ascontiguousarray(a, dtype=np.float32)


def _in(a, double: bool) -> np.ndarray | None:
    if a is None:
        return None
    if hasattr(a, 'detach'):
        a = a.detach().cpu().numpy()
    return np.ascontiguousarray(a, dtype=np.float64 if double else np.float32)


def make_view(cam, degree: int, proper_aa: bool = False, render_base: bool = True, render_residual: bool = True) -> View:
    v = View()
    w2c = _f32(cam.w2c).reshape(-1)
    for k in range(16):
        v.w2c[k] = float(w2c[k])
    pos, bg = _f32(cam.position).reshape(-1), _f32(cam.bg).reshape(-1)
    for k in range(3):
        v.cam[k] = float(pos[k])
        v.bg[k] = float(bg[k])
    v.width, v.height = int(cam.width), int(cam.height)
    v.fx, v.fy, v.cx, v.cy = float(cam.focal_x), float(cam.focal_y), float(cam.center_x), float(cam.center_y)
    v.near_plane, v.far_plane = float(cam.near_plane), float(cam.far_plane)
    v.proper_aa, v.render_base = int(proper_aa), int(render_base)
    v.degree = int(degree) if render_residual else 0
    return v


def make_appearance(model: str, max_degree: int = 0, base_act: int = 0, res_act: int = 0, color_act: int = 1, dir_grad: bool = True,
                    neural: dict | None = None) -> Appearance:
    a = Appearance()
    a.model = MODEL_IDS[model]
    a.max_degree = max_degree
    a.base_act, a.res_act, a.color_act, a.dir_grad = base_act, res_act, color_act, int(dir_grad)
    if neural:
        for k, v in neural.items():
            setattr(a, k, int(v))
        a.max_degree = sum(1 for l in range(1, 7) if neural['sh_mask'] & (1 << l))
    return a


def run(app: Appearance, view: View, prims: dict, grad_image=None, double: bool = False, densification_rows: int = 0,
        pruning: bool = False, rank_grads=None) -> dict:
    """Runs the restated pipeline; prims holds numpy/torch arrays (means, scales, rotations, opacities and the
    appearance inputs). Returns intermediates, the image [3,H,W], with pruning the per-primitive pruning scores and,
    with grad_image, all gradients. With rank_grads ([V, 12] per depth rank of this run, in the blend backward's
    layout {mean2d x, y, conic a, b, c, colour r, g, b, opacity, |mean2d x|, |mean2d y|, 0}) the backward preprocess
    runs on those per-primitive blend sums instead of the restated blend backward."""
    lib = load(double)
    means, scales, rots, opac = (_in(prims[k], double) for k in ('means', 'scales', 'rotations', 'opacities'))
    pre = _in(prims.get('precomputed_colors'), double)
    base = _in(prims.get('base_colors'), double)
    res = _in(prims.get('residual_params'), double)
    mlp = _in(prims.get('mlp_weights'), double)
    n = means.shape[0]
    n_touched = np.zeros(n, np.uint32)
    depth_key = np.zeros(n, np.uint32)
    rec = np.zeros((n, 14), np.float64)
    app_c = app
    if pre is not None:
        app_c = Appearance()
        ctypes.memmove(ctypes.byref(app_c), ctypes.byref(app), ctypes.sizeof(Appearance))
        app_c.model = 0
    lib.orc_preprocess(ctypes.byref(app_c), ctypes.byref(view), n, _p(means), _p(scales), _p(rots), _p(opac), _p(pre), _p(base), _p(res),
                       _p(mlp), _p(n_touched), _p(depth_key), _p(rec))
    sorted_idx = np.zeros(max(n, 1), np.uint32)
    V = lib.orc_depth_order(n, _p(n_touched), _p(depth_key), _p(sorted_idx))
    sorted_idx = sorted_idx[:V]
    I = lib.orc_count_instances(V, _p(sorted_idx), _p(n_touched))
    W, H = view.width, view.height
    T = ((W + 15) // 16) * ((H + 11) // 12)
    tile_keys = np.zeros(max(I, 1), np.uint32)
    ranks = np.zeros(max(I, 1), np.uint32)
    ranges = np.zeros((T, 2), np.uint32)
    I2 = lib.orc_bin(V, _p(sorted_idx), _p(rec), W, H, _p(tile_keys), _p(ranks), _p(ranges))
    assert I2 == I
    tile_keys, ranks = tile_keys[:I], ranks[:I]
    rdt = np.float64 if double else np.float32
    image = np.zeros((3, H, W), rdt)
    final_T = np.zeros((H, W), rdt)
    n_contrib = np.zeros((H, W), np.uint32)
    lib.orc_blend(V, _p(sorted_idx), _p(rec), _p(ranks), _p(ranges), ctypes.byref(view), _p(image), _p(final_T), _p(n_contrib), 1, 0)
    offsets = np.zeros(V, np.uint32)
    if V:
        counts = n_touched[sorted_idx].astype(np.int64)
        offsets = (np.cumsum(counts) - counts).astype(np.uint32)
    out = dict(n_visible=int(V), n_instances=int(I), n_touched=n_touched, depth_key=depth_key, records=rec, sorted_idx=sorted_idx,
               instance_offsets=offsets, tile_keys=tile_keys, ranks=ranks, ranges=ranges, image=image, final_T=final_T, n_contrib=n_contrib)
    if pruning:
        scores = np.zeros(max(n, 1), np.float64)
        lib.orc_pruning_scores(V, _p(sorted_idx), _p(rec), _p(ranks), _p(ranges), ctypes.byref(view), _p(n_contrib), _p(scores))
        out['pruning_scores'] = scores[:n]
    if grad_image is None and rank_grads is None:
        return out
    grads = np.zeros((max(V, 1), 12), np.float64)
    if rank_grads is not None:
        grads[:V] = np.asarray(rank_grads, np.float64).reshape(V, 12)
    else:
        gimg = _f32(grad_image)
        lib.orc_blend_backward(V, _p(sorted_idx), _p(rec), _p(ranks), _p(ranges), ctypes.byref(view), _p(n_contrib), _p(gimg), _p(grads))
    rank_of = np.full(n, 0xffffffff, np.uint32)
    rank_of[sorted_idx] = np.arange(V, dtype=np.uint32)
    stride = res.shape[1] if res is not None and res.ndim == 2 else (int(np.prod(res.shape[1:])) if res is not None else 0)
    g = {
        'means': np.zeros((n, 3)), 'scales': np.zeros((n, 3)), 'rotations': np.zeros((n, 4)), 'opacities': np.zeros((n, 1)),
        'precomputed_colors': np.zeros((n, 3)) if pre is not None else None,
        'base_colors': np.zeros((n, 3)) if base is not None and pre is None else None,
        'residual_params': np.zeros((n, stride)) if res is not None and pre is None else None,
        'mlp_weights': np.zeros(mlp.shape[0]) if mlp is not None and pre is None else None,
    }
    dens = np.zeros((densification_rows, n)) if densification_rows else None
    lib.orc_preprocess_backward(ctypes.byref(app_c), ctypes.byref(view), n, _p(means), _p(scales), _p(rots), _p(opac), _p(pre), _p(base),
                                _p(res), _p(mlp), _p(rank_of), _p(rec), _p(grads), _p(g['means']), _p(g['scales']), _p(g['rotations']),
                                _p(g['opacities']), _p(g['precomputed_colors']), _p(g['base_colors']), _p(g['residual_params']),
                                _p(g['mlp_weights']), _p(dens), densification_rows)
    out['rank_grads'] = grads[:V]
    out['rank_of'] = rank_of
    out['grads'] = g
    out['densification'] = dens
    return out


def adam(param, grad, m, v, step, lrs, betas, eps, col_offset: int = 0):
    """In-place fused-Adam update restated in float (adam.cu:18-42); arrays are float32 numpy."""
    lib = load(False)
    lrs = list(lrs) if isinstance(lrs, (list, tuple)) else [lrs]
    arr = (ctypes.c_double * 7)(*([float(x) for x in lrs] + [0.0] * (7 - len(lrs))))
    lib.orc_adam(param.size, _p(param), _p(grad), _p(m), _p(v), int(step), arr, len(lrs), int(col_offset), float(betas[0]),
                 float(betas[1]), float(eps))


def appearance(app: Appearance, means, cam_pos, base, residual, degree: int, upstream=None, double: bool = True) -> dict:
    """Fused-appearance colors (and, with `upstream`, the gradients of sum(colors * upstream)) evaluated in double."""
    lib = load(double)
    P = ctypes.c_void_p
    lib.orc_appearance_eval.argtypes = [P, ctypes.c_int64, P, P, P, P, ctypes.c_int, P]
    lib.orc_appearance_grad.argtypes = [P, ctypes.c_int64, P, P, P, P, ctypes.c_int, P, P, P, P]
    means, base, residual = _in(means, double), _in(base, double), _in(residual, double)
    cam = np.ascontiguousarray(np.asarray(cam_pos, dtype=np.float32).reshape(3))
    n = means.shape[0]
    colors = np.zeros((n, 3))
    lib.orc_appearance_eval(ctypes.byref(app), n, _p(means), _p(cam), _p(base), _p(residual), int(degree), _p(colors))
    out = {'colors': colors}
    if upstream is not None:
        up = np.ascontiguousarray(np.asarray(upstream, dtype=np.float64))
        gb, gr, gm = np.zeros((n, 3)), np.zeros(residual.reshape(n, -1).shape), np.zeros((n, 3))
        lib.orc_appearance_grad(ctypes.byref(app), n, _p(means), _p(cam), _p(base), _p(residual), int(degree), _p(up), _p(gb), _p(gr), _p(gm))
        out.update(grad_base=gb, grad_residual=gr, grad_means=gm)
    return out


def set_threads(n: int) -> None:
    """Threads of the oracle's per-primitive and per-pixel loops (both builds); 1, the default, keeps every loop in
    order. Used by the CPU-baseline timing; the parity tests run with one thread."""
    for double in (False, True):
        load(double).orc_set_threads(int(n))

