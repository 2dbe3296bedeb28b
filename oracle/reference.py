"""Test infrastructure only: ctypes access to the reference harness (oracle/_ref/libfgsref.so and its preprocess
cubins, built by oracle/ref_build.py from the reference's own sources), so the GPU parity tests can run the reference
rasterizer on the same device tensors as this library. Imported by tests only; the product never loads it.

The calls mirror the reference's torch glue (rasterization/src/rasterization_api.cu:16-335): forward() allocates the
image and runs faster_gs::rasterization::forward, backward() allocates the gradient and helper tensors with the
reference's initialisation (helpers and the opacity gradient zeroed) and runs faster_gs::rasterization::backward,
inference() runs faster_gs::rasterization::inference; buffers() copies the stage buffers of the last forward out.
"""
from __future__ import annotations

import ctypes
import json
from pathlib import Path

import numpy as np
import torch

REF_DIR = Path(__file__).resolve().parent / '_ref'
P = ctypes.c_void_p
F = ctypes.c_float
I = ctypes.c_int

# appearance configurations with cubins (tag -> model, base act, residual act, color act, max degree); see ref_build.CONFIGS
ACT_NAMES = {'base': ['none', 'exp'], 'res': ['none', 'tanh', 'softplus'], 'color': ['none', 'relu', 'softplus', 'sigmoid', 'hardsigmoid', 'satexp']}
MODELS = {0: 'precomputed', 1: 'sh', 2: 'sv', 3: 'nasg', 4: 'nasgabor'}


def available() -> bool:
    return (REF_DIR / 'libfgsref.so').is_file() and (REF_DIR / 'index.json').is_file()


def tag_of(model: str, degree: int, base: str, res: str, color: str) -> str:
    if model == 'precomputed':
        return 'precomputed'
    return f'{model}{degree}_{base}_{res}_{color}'


def tags() -> list[str]:
    idx = json.loads((REF_DIR / 'index.json').read_text())
    return sorted({k.split('_', 2)[2] for k in idx})


_lib = None


def lib():
    global _lib
    if _lib is None:
        l = ctypes.CDLL(str(REF_DIR / 'libfgsref.so'))
        l.ref_last_error.restype = ctypes.c_char_p
        l.ref_create.argtypes = [P, ctypes.c_char_p, P, ctypes.c_char_p, ctypes.POINTER(P)]
        l.ref_destroy.argtypes = [P]
        l.ref_forward.argtypes = [P] + [P] * 11 + [I] * 4 + [F] * 6 + [I, I, P, ctypes.POINTER(I)]
        l.ref_backward.argtypes = [P] + [P] * 24 + [I] + [F] * 4 + [I, I, P]
        l.ref_inference.argtypes = [P] + [P] * 11 + [I] * 4 + [F] * 6 + [I, I, I, I, P]
        l.ref_copy.argtypes = [P, I, P, ctypes.c_size_t]
        l.ref_copy.restype = ctypes.c_longlong
        _lib = l
    return _lib


def _check(rc: int) -> None:
    if rc:
        raise RuntimeError('reference harness: ' + lib().ref_last_error().decode())


def _ptr(t):
    return None if t is None or t.numel() == 0 else t.data_ptr()


class Reference:
    """One reference rasterizer configuration (the appearance model's preprocess cubins)."""

    def __init__(self, tag: str):
        idx = json.loads((REF_DIR / 'index.json').read_text())
        fwd = idx[f'preprocess_forward_{tag}']
        bwd = idx[f'preprocess_backward_{tag}']
        self._fwd_bytes = ctypes.create_string_buffer((REF_DIR / fwd['cubin']).read_bytes())
        self._bwd_bytes = ctypes.create_string_buffer((REF_DIR / bwd['cubin']).read_bytes())
        h = P()
        _check(lib().ref_create(ctypes.addressof(self._fwd_bytes), fwd['kernel'].encode(), ctypes.addressof(self._bwd_bytes),
                                bwd['kernel'].encode(), ctypes.byref(h)))
        self.h = h
        self.n = 0

    def close(self):
        if self.h:
            lib().ref_destroy(self.h)
            self.h = None

    def __del__(self):
        try:
            self.close()
        except Exception:  # interpreter shutdown: the library may already be gone
            pass

    @staticmethod
    def _cam(settings, device):
        w2c = torch.as_tensor(settings.w2c, dtype=torch.float32, device=device).contiguous()
        cam = torch.as_tensor(settings.cam_position, dtype=torch.float32, device=device).contiguous()
        bg = torch.as_tensor(settings.bg_color, dtype=torch.float32, device=device).contiguous()
        return w2c, cam, bg

    def forward(self, p: dict, settings) -> torch.Tensor:
        """Training forward; returns the [3,H,W] image (render_residual as rasterization_api.cu:105)."""
        dev = p['means'].device
        w2c, cam, bg = self._cam(settings, dev)
        self._keep = (w2c, cam, bg)
        image = torch.empty(3, settings.height, settings.width, device=dev)
        counts = (I * 3)()
        deg = settings.appearance_degree if settings.render_residual else 0
        _check(lib().ref_forward(self.h, _ptr(p['means']), _ptr(p['scales']), _ptr(p['rotations']), _ptr(p['opacities']),
                                 _ptr(p.get('precomputed_colors')), _ptr(p.get('base_colors')), _ptr(p.get('residual_params')), w2c.data_ptr(),
                                 cam.data_ptr(), bg.data_ptr(), image.data_ptr(), p['means'].shape[0], deg, settings.width, settings.height,
                                 settings.focal_x, settings.focal_y, settings.center_x, settings.center_y, settings.near_plane, settings.far_plane,
                                 int(bool(settings.proper_antialiasing)), int(bool(settings.render_base)),
                                 torch.cuda.current_stream().cuda_stream, counts))
        torch.cuda.synchronize()
        self.n = p['means'].shape[0]
        self.n_instances, self.n_buckets, self.selector = counts[0], counts[1], counts[2]
        self.settings = settings
        return image

    def backward(self, p: dict, image: torch.Tensor, grad_image: torch.Tensor, densification_rows: int = 0) -> dict:
        """Gradients of the last forward for the upstream image gradient (rasterization_api.cu:125-247)."""
        s = self.settings
        dev = p['means'].device
        n = self.n
        w2c, cam, bg = self._keep
        z = lambda *shape: torch.zeros(*shape, device=dev)
        out = {'means': z(n, 3), 'scales': z(n, 3), 'rotations': z(n, 4), 'opacities': z(n, 1)}
        pre = p.get('precomputed_colors')
        out['precomputed_colors'] = z(n, 3) if pre is not None else None
        out['base_colors'] = z(n, 3) if pre is None else None
        out['residual_params'] = torch.zeros_like(p['residual_params']) if pre is None and p.get('residual_params') is not None else None
        h_mean2d, h_conic, h_color = z(n, 2), z(3, n), z(3, n)
        h_abs = z(n, 2) if densification_rows == 3 else None
        dens = z(densification_rows, n) if densification_rows else None
        deg = s.appearance_degree if s.render_residual else 0
        gi = grad_image.contiguous()
        _check(lib().ref_backward(self.h, gi.data_ptr(), _ptr(p['means']), _ptr(p['scales']), _ptr(p['rotations']), _ptr(p['opacities']),
                                  _ptr(pre), _ptr(p.get('base_colors')), _ptr(p.get('residual_params')), w2c.data_ptr(), cam.data_ptr(),
                                  bg.data_ptr(), image.data_ptr(), h_mean2d.data_ptr(), h_conic.data_ptr(), _ptr(h_abs), h_color.data_ptr(),
                                  out['means'].data_ptr(), out['scales'].data_ptr(), out['rotations'].data_ptr(), out['opacities'].data_ptr(),
                                  _ptr(out['precomputed_colors']), _ptr(out['base_colors']), _ptr(out['residual_params']), _ptr(dens), deg,
                                  s.focal_x, s.focal_y, s.center_x, s.center_y, int(bool(s.proper_antialiasing)), int(bool(s.render_base)),
                                  torch.cuda.current_stream().cuda_stream))
        torch.cuda.synchronize()
        out['densification_info'] = dens
        return out

    def inference(self, p: dict, settings, to_chw: bool, clamp: bool) -> torch.Tensor:
        dev = p['means'].device
        w2c, cam, bg = self._cam(settings, dev)
        shape = (3, settings.height, settings.width) if to_chw else (settings.height, settings.width, 3)
        image = torch.empty(*shape, device=dev)
        deg = settings.appearance_degree if settings.render_residual else 0
        _check(lib().ref_inference(self.h, _ptr(p['means']), _ptr(p['scales']), _ptr(p['rotations']), _ptr(p['opacities']),
                                   _ptr(p.get('precomputed_colors')), _ptr(p.get('base_colors')), _ptr(p.get('residual_params')), w2c.data_ptr(),
                                   cam.data_ptr(), bg.data_ptr(), image.data_ptr(), p['means'].shape[0], deg, settings.width, settings.height,
                                   settings.focal_x, settings.focal_y, settings.center_x, settings.center_y, settings.near_plane,
                                   settings.far_plane, int(bool(settings.proper_antialiasing)), int(bool(settings.render_base)), int(to_chw),
                                   int(clamp), torch.cuda.current_stream().cuda_stream))
        torch.cuda.synchronize()
        return image

    def buffers(self) -> dict:
        """Stage buffers of the last training forward, as numpy arrays."""
        s = self.settings
        n, ni = self.n, self.n_instances
        gw, gh = (s.width + 15) // 16, (s.height + 11) // 12
        T = gw * gh
        wide = (T - 1).bit_length() > 16

        def get(which, dtype, count, shape=None):
            a = np.zeros(max(count, 1) * np.dtype(dtype).itemsize, np.uint8)
            got = lib().ref_copy(self.h, which, a.ctypes.data, a.nbytes)
            if got < 0:
                _check(1)
            a = a[:got].view(dtype)
            return a.reshape(shape) if shape else a

        out = {'n_touched': get(0, np.uint32, n), 'screen_bounds': get(1, np.uint16, 4 * n, (n, 4)), 'mean2d': get(2, np.float32, 2 * n, (n, 2)),
               'conic_opacity': get(3, np.float32, 4 * n, (n, 4)), 'color': get(4, np.float32, 3 * n, (n, 3)),
               'tile_keys': get(5, np.uint32 if wide else np.uint16, ni).astype(np.uint32), 'instance_prims': get(6, np.uint32, ni),
               'ranges': get(7, np.uint32, 2 * T, (T, 2)), 'final_T': get(8, np.float32, s.width * s.height, (s.height, s.width)),
               'n_contrib': get(9, np.uint32, s.width * s.height, (s.height, s.width)), 'tile_max': get(10, np.uint32, T),
               'counters': get(11, np.uint32, 2)}
        out['n_visible'] = int(out['counters'][0])
        out['n_instances'] = ni
        return out
