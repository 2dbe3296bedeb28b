"""Rasterizer operator API, drop-in for FasterGSVDACudaBackend/FasterGSVDACudaBackend/torch_bindings/rasterization.py.

Same names, argument order and meaning as the reference (initialize_appearance :11-32, initialize_residual_mlp
:35-46, RasterizerSettings :49-83, _Rasterize :86-169, diff_rasterize :172-195, rasterize :198-224). Every call
goes through libfgs_b200.so; device memory (images, gradients, workspaces) is allocated with torch on the current
device and the kernels run on torch's current stream.
"""
from __future__ import annotations

import ctypes
from typing import Any, NamedTuple

import torch
from torch.autograd.function import once_differentiable

from . import _lib
from ._lib import lib, check, size_out, ptr

APPEARANCE_MODEL_IDS = {'sh': 1, 'sv': 2, 'nasg': 3, 'nasgabor': 4, 'neural': 5}  # 0 is the internal precomputed-colors variant
BASE_ACTIVATION_IDS = {'none': 0, 'exp': 1}
RESIDUAL_ACTIVATION_IDS = {'none': 0, 'tanh': 1, 'softplus': 2}
COLOR_ACTIVATION_IDS = {'none': 0, 'relu': 1, 'softplus': 2, 'sigmoid': 3, 'hardsigmoid': 4, 'satexp': 5}
HIDDEN_ACTIVATION_IDS = {'none': 0, 'relu': 1}


class Rasterizer:
    """Owns the library-side configuration (the reference's module-level `_C.Rasterizer`)."""

    def __init__(self) -> None:
        handle = ctypes.c_void_p()
        check(lib.fgs_rasterizer_create(ctypes.byref(handle)))
        self.handle = handle
        self.model = None
        self.mlp = None

    def __del__(self) -> None:
        try:
            if self.handle:
                lib.fgs_rasterizer_destroy(self.handle)
        except Exception:  # interpreter shutdown
            pass

    def set_appearance(self, model: int, max_degree: int, base: int, residual: int, color: int, direction_gradient: bool) -> None:
        check(lib.fgs_set_appearance(self.handle, model, max_degree, base, residual, color, int(bool(direction_gradient))))
        self.model = model
        self.mlp = None

    def set_residual_mlp(self, n_input_dims: int, n_output_dims: int, n_neurons: int, n_hidden_layers: int, hidden_activation: int,
                         base_input: bool, n_frequencies: int, sh_degree_mask: int) -> None:
        check(lib.fgs_set_residual_mlp(self.handle, n_input_dims, n_output_dims, n_neurons, n_hidden_layers, hidden_activation,
                                       int(bool(base_input)), n_frequencies, sh_degree_mask))
        self.mlp = (n_input_dims, n_output_dims, n_neurons, n_hidden_layers, hidden_activation, base_input, n_frequencies, sh_degree_mask)

    @property
    def n_mlp_params(self) -> int:
        out = ctypes.c_int64(0)
        check(lib.fgs_mlp_param_count(self.handle, ctypes.byref(out)))
        return int(out.value)

    @property
    def residual_stride(self) -> int:
        out = ctypes.c_int64(0)
        check(lib.fgs_residual_stride(self.handle, ctypes.byref(out)))
        return int(out.value)


# module-level rasterizer instance (rasterization.py:8)
_rasterizer = Rasterizer()


def initialize_appearance(
    appearance_model: str,
    max_degree: int,
    base_activation: str,
    residual_activation: str,
    color_activation: str,
    direction_gradient: bool,
) -> None:
    """Configures the rasterizer's kernels for the given appearance model."""
    _rasterizer.set_appearance(
        APPEARANCE_MODEL_IDS[appearance_model],
        max_degree,
        BASE_ACTIVATION_IDS[base_activation],
        RESIDUAL_ACTIVATION_IDS[residual_activation],
        COLOR_ACTIVATION_IDS[color_activation],
        direction_gradient,
    )


def initialize_residual_mlp(
    n_input_dims: int,
    n_output_dims: int,
    encoding_config: dict[str, Any],
    network_config: dict[str, Any],
    base_input: bool,
    n_frequencies: int,
    sh_degrees: list[int],
) -> None:
    """Configures the fused residual MLP from a tinycudann-style configuration (requires initialize_appearance('neural', ...) first).

    Supported: Identity encoding; FullyFusedMLP / CutlassMLP networks with 16, 32 or 64 neurons, ReLU or None hidden
    activation, no output activation; SH bands 0-3 of the view direction (every reference configuration). Weights are a flat fp32 vector: the input layer [n_neurons, pad16(n_input_dims)],
    n_hidden_layers - 1 hidden layers [n_neurons, n_neurons], the output layer [16, n_neurons] (rows beyond n_output_dims
    unused), each row-major; padded input dims carry the value 1.
    """
    if encoding_config.get('otype', 'Identity') != 'Identity':
        raise RuntimeError(f"FasterGSVDA: unsupported encoding {encoding_config.get('otype')} (only Identity)")
    otype = network_config.get('otype', 'FullyFusedMLP')
    if otype not in ('FullyFusedMLP', 'CutlassMLP'):
        raise RuntimeError(f'FasterGSVDA: unsupported network {otype}')
    if str(network_config.get('output_activation', 'None')).lower() != 'none':
        raise RuntimeError('FasterGSVDA: the residual mlp output activation must be None')
    hidden = str(network_config.get('activation', 'ReLU')).lower()
    if hidden not in HIDDEN_ACTIVATION_IDS:
        raise RuntimeError(f"FasterGSVDA: unsupported hidden activation {network_config.get('activation')}")
    sh_degree_mask = sum(1 << degree for degree in sh_degrees)
    _rasterizer.set_residual_mlp(n_input_dims, n_output_dims, int(network_config['n_neurons']), int(network_config['n_hidden_layers']),
                                 HIDDEN_ACTIVATION_IDS[hidden], base_input, n_frequencies, sh_degree_mask)


class RasterizerSettings(NamedTuple):
    w2c: torch.Tensor  # affine transformation from model/world space to view space
    cam_position: torch.Tensor  # camera position in world space
    bg_color: torch.Tensor  # background color in RGB format
    appearance_degree: int  # appearance degree used for rendering
    width: int  # width of the image plane in pixels
    height: int  # height of the image plane in pixels
    focal_x: float  # focal length in x direction in pixels
    focal_y: float  # focal length in y direction in pixels
    center_x: float  # x coordinate of the image center in pixels (positive -> right)
    center_y: float  # y coordinate of the image center in pixels (positive -> down)
    near_plane: float  # near clipping plane distance
    far_plane: float  # far clipping plane distance
    proper_antialiasing: bool  # whether to use proper antialiasing
    render_base: bool  # whether the view-independent base color contributes to the rendered color
    render_residual: bool  # whether the view-dependent appearance term contributes (if False, the appearance degree is treated as 0)

    def as_tuple(self) -> tuple:
        return tuple(self)


def _device_vec(t: torch.Tensor, n: int, device: torch.device) -> torch.Tensor:
    t = torch.as_tensor(t, dtype=torch.float32)
    if t.device != device or not t.is_contiguous() or t.data_ptr() % 16 != 0:
        t = t.to(device=device, dtype=torch.float32).contiguous().clone()
    if t.numel() != n:
        raise RuntimeError(f'expected {n} floats, got shape {tuple(t.shape)}')
    return t


def _c_settings(s: RasterizerSettings, device: torch.device) -> tuple[_lib.Settings, tuple]:
    w2c = _device_vec(s.w2c, 16, device)
    cam = _device_vec(s.cam_position, 3, device)
    bg = _device_vec(s.bg_color, 3, device)
    cs = _lib.Settings(w2c.data_ptr(), cam.data_ptr(), bg.data_ptr(), int(s.appearance_degree), int(s.width), int(s.height),
                       float(s.focal_x), float(s.focal_y), float(s.center_x), float(s.center_y), float(s.near_plane),
                       float(s.far_plane), int(bool(s.proper_antialiasing)), int(bool(s.render_base)), int(bool(s.render_residual)))
    return cs, (w2c, cam, bg)


def _check_input(t: torch.Tensor | None, name: str) -> None:
    if t is None or t.numel() == 0:
        return
    if not t.is_cuda or t.dtype != torch.float32 or not t.is_contiguous():
        raise RuntimeError(f'{name} must be a contiguous CUDA float32 tensor')


def _check_sizes(n: int, scales, rotations, opacities, precomputed, base, residual, mlp, rasterizer: 'Rasterizer | None') -> None:
    """Rejects tensors whose sizes do not match N and the configured appearance (the kernels index them by N)."""
    def need(t, count, name):
        if t is not None and t.numel() > 0 and t.numel() != count:
            raise ValueError(f'{name} has {t.numel()} elements, expected {count}')
    need(scales, 3 * n, 'scales')
    need(rotations, 4 * n, 'rotations')
    need(opacities, n, 'opacities')
    need(precomputed, 3 * n, 'precomputed_colors')
    if precomputed is not None and precomputed.numel() > 0:
        return
    need(base, 3 * n, 'base_colors')
    if rasterizer is not None and rasterizer.model is not None:
        need(residual, rasterizer.residual_stride * n, 'residual_params')
        if rasterizer.mlp is not None:
            need(mlp, rasterizer.n_mlp_params, 'mlp_weights')


def _c_primitives(means, scales, rotations, opacities, precomputed, base, residual, mlp) -> _lib.Primitives:
    for t, name in ((means, 'means'), (scales, 'scales'), (rotations, 'rotations'), (opacities, 'opacities'),
                    (precomputed, 'precomputed_colors'), (base, 'base_colors'), (residual, 'residual_params'), (mlp, 'mlp_weights')):
        _check_input(t, name)
    if means.numel() % 3:
        raise ValueError('means must have shape [N, 3]')
    _check_sizes(means.numel() // 3, scales, rotations, opacities, precomputed, base, residual, mlp, _rasterizer)
    if rotations.numel() > 0 and rotations.data_ptr() % 16 != 0:
        raise RuntimeError('rotations must be 16-byte aligned')
    return _lib.Primitives(ptr(means), ptr(scales), ptr(rotations), ptr(opacities), ptr(precomputed), ptr(base), ptr(residual), ptr(mlp),
                           means.shape[0])


def _stream() -> int:
    return torch.cuda.current_stream().cuda_stream


def _workspace(nbytes: int, device: torch.device) -> torch.Tensor:
    return torch.empty(max(int(nbytes), 1), dtype=torch.uint8, device=device)


class ForwardState:
    """Workspaces and frame record of one forward pass (kept by autograd for the backward)."""

    def __init__(self, rasterizer: Rasterizer, prims: _lib.Primitives, settings: RasterizerSettings, device: torch.device,
                 training: bool = True) -> None:
        """`training`: a backward follows, so the primitive workspace also holds the tensor-core MLP's activations
        (Neural appearance), which the backward then reads instead of recomputing them."""
        self.rasterizer = rasterizer
        self.settings = settings
        self.device = device
        self.c_settings, self.keep = _c_settings(settings, device)
        self.frame = _lib.Frame()
        n = prims.n_primitives
        self.prim_ws = _workspace(size_out(lib.fgs_primitive_workspace_bytes, rasterizer.handle if training else None, n), device)
        self.tile_ws = _workspace(size_out(lib.fgs_tile_workspace_bytes, int(settings.width), int(settings.height)), device)
        self.inst_ws = None
        self.bucket_ws = None

    def preprocess(self, prims: _lib.Primitives) -> None:
        check(lib.fgs_forward_preprocess(self.rasterizer.handle, ctypes.byref(prims), ctypes.byref(self.c_settings), self.prim_ws.data_ptr(),
                                         self.prim_ws.numel(), _stream(), ctypes.byref(self.frame)))
        f = self.frame
        self.inst_ws = _workspace(size_out(lib.fgs_instance_workspace_bytes, f.n_instances, f.width, f.height), self.device)

    def render_train(self, image: torch.Tensor) -> None:
        f = self.frame
        n_tiles = ((f.width + 15) // 16) * ((f.height + 11) // 12)
        self.bucket_ws = _workspace(size_out(lib.fgs_bucket_workspace_bytes, f.n_instances // 32 + n_tiles), self.device)
        check(lib.fgs_forward_render(self.rasterizer.handle, ctypes.byref(self.c_settings), ctypes.byref(f), self.prim_ws.data_ptr(),
                                     self.tile_ws.data_ptr(), self.tile_ws.numel(), self.inst_ws.data_ptr(), self.inst_ws.numel(),
                                     self.bucket_ws.data_ptr(), self.bucket_ws.numel(), image.data_ptr(), _stream()))

    def render_inference(self, image: torch.Tensor, to_chw: bool, clamp_output: bool) -> None:
        f = self.frame
        check(lib.fgs_inference_render(self.rasterizer.handle, ctypes.byref(self.c_settings), ctypes.byref(f), self.prim_ws.data_ptr(),
                                       self.tile_ws.data_ptr(), self.tile_ws.numel(), self.inst_ws.data_ptr(), self.inst_ws.numel(),
                                       image.data_ptr(), int(bool(to_chw)), int(bool(clamp_output)), _stream()))

    def backward(self, prims: _lib.Primitives, image: torch.Tensor, grad_image: torch.Tensor, grads: _lib.Gradients,
                 densification_info: torch.Tensor | None, accumulate: bool = False, grad_ws: torch.Tensor | None = None) -> None:
        """`grad_ws`: a caller-owned gradient workspace (uint8, at least fgs_gradient_workspace_bytes) that keeps the
        per-primitive blend sums of this backward (48-byte records in depth-rank order at its start) for inspection."""
        f = self.frame
        need = size_out(lib.fgs_gradient_workspace_bytes, self.rasterizer.handle, f.n_visible)
        if grad_ws is None:
            grad_ws = _workspace(need, self.device)
        elif grad_ws.numel() < need:
            raise ValueError('gradient workspace too small')
        dens = ptr(densification_info)
        rows = densification_info.shape[0] if dens is not None else 0
        check(lib.fgs_backward(self.rasterizer.handle, ctypes.byref(prims), ctypes.byref(self.c_settings), ctypes.byref(f),
                               self.prim_ws.data_ptr(), self.tile_ws.data_ptr(), self.inst_ws.data_ptr(), self.bucket_ws.data_ptr(),
                               grad_ws.data_ptr(), grad_ws.numel(), image.data_ptr(), grad_image.data_ptr(), ctypes.byref(grads), dens,
                               rows, int(bool(accumulate)), _stream()))

    def pruning_scores(self, image: torch.Tensor, scores: torch.Tensor) -> None:
        check(lib.fgs_pruning_scores(ctypes.byref(self.c_settings), ctypes.byref(self.frame), self.prim_ws.data_ptr(), self.tile_ws.data_ptr(),
                                     self.inst_ws.data_ptr(), image.data_ptr(), scores.data_ptr(), _stream()))

    def views(self) -> _lib.FrameViews:
        out = _lib.FrameViews()
        check(lib.fgs_frame_buffers(ctypes.byref(self.frame), self.prim_ws.data_ptr(), self.tile_ws.data_ptr(),
                                    self.inst_ws.data_ptr() if self.inst_ws is not None else None, ctypes.byref(out)))
        return out


def _empty(device) -> torch.Tensor:
    return torch.empty(0, dtype=torch.float32, device=device)


class _Rasterize(torch.autograd.Function):
    @staticmethod
    def forward(
        ctx: Any,
        means: torch.Tensor,
        scales: torch.Tensor,
        rotations: torch.Tensor,
        opacities: torch.Tensor,
        precomputed_colors: torch.Tensor,
        base_colors: torch.Tensor,
        residual_params: torch.Tensor,
        mlp_weights: torch.Tensor,
        densification_info: torch.Tensor,
        rasterizer_settings: RasterizerSettings,
    ) -> torch.Tensor:
        device = means.device
        prims = _c_primitives(means, scales, rotations, opacities, precomputed_colors, base_colors, residual_params, mlp_weights)
        state = ForwardState(_rasterizer, prims, rasterizer_settings, device)
        state.preprocess(prims)
        image = torch.empty((3, int(rasterizer_settings.height), int(rasterizer_settings.width)), dtype=torch.float32, device=device)
        state.render_train(image)
        ctx.state = state
        ctx.densification_info = densification_info
        ctx.save_for_backward(image, means, scales, rotations, opacities, precomputed_colors, base_colors, residual_params, mlp_weights)
        ctx.mark_non_differentiable(densification_info)
        return image

    @staticmethod
    @once_differentiable
    def backward(ctx: Any, grad_image: torch.Tensor):
        image, means, scales, rotations, opacities, precomputed_colors, base_colors, residual_params, mlp_weights = ctx.saved_tensors
        state: ForwardState = ctx.state
        prims = _c_primitives(means, scales, rotations, opacities, precomputed_colors, base_colors, residual_params, mlp_weights)
        grad_image = grad_image.contiguous().float()
        g_means = torch.empty_like(means)
        g_scales = torch.empty_like(scales)
        g_rotations = torch.empty_like(rotations)
        g_opacities = torch.empty_like(opacities)
        g_pre = torch.empty_like(precomputed_colors)
        g_base = torch.empty_like(base_colors)
        g_res = torch.empty_like(residual_params)
        g_mlp = torch.empty_like(mlp_weights)
        grads = _lib.Gradients(ptr(g_means), ptr(g_scales), ptr(g_rotations), ptr(g_opacities), ptr(g_pre), ptr(g_base), ptr(g_res), ptr(g_mlp))
        dens = ctx.densification_info if ctx.densification_info is not None and ctx.densification_info.numel() > 0 else None
        state.backward(prims, image, grad_image, grads, dens)
        return (
            g_means, g_scales, g_rotations, g_opacities,
            g_pre if g_pre.numel() > 0 else None,
            g_base if g_base.numel() > 0 else None,
            g_res if g_res.numel() > 0 else None,
            g_mlp if g_mlp.numel() > 0 else None,
            None,  # densification_info
            None,  # rasterizer_settings
        )


def diff_rasterize(
    means: torch.Tensor,
    scales: torch.Tensor,
    rotations: torch.Tensor,
    opacities: torch.Tensor,
    densification_info: torch.Tensor,
    rasterizer_settings: RasterizerSettings,
    precomputed_colors: torch.Tensor | None = None,
    base_colors: torch.Tensor | None = None,
    residual_params: torch.Tensor | None = None,
    mlp_weights: torch.Tensor | None = None,
) -> torch.Tensor:
    device = means.device
    return _Rasterize.apply(
        means,
        scales,
        rotations,
        opacities,
        precomputed_colors if precomputed_colors is not None else _empty(device),
        base_colors if base_colors is not None else _empty(device),
        residual_params if residual_params is not None else _empty(device),
        mlp_weights if mlp_weights is not None else _empty(device),
        densification_info,
        rasterizer_settings,
    )


@torch.no_grad()
def rasterize(
    means: torch.Tensor,
    scales: torch.Tensor,
    rotations: torch.Tensor,
    opacities: torch.Tensor,
    rasterizer_settings: RasterizerSettings,
    to_chw: bool,
    clamp_output: bool,
    precomputed_colors: torch.Tensor | None = None,
    base_colors: torch.Tensor | None = None,
    residual_params: torch.Tensor | None = None,
    mlp_weights: torch.Tensor | None = None,
) -> torch.Tensor:
    device = means.device
    mlp = mlp_weights.detach() if mlp_weights is not None else None
    prims = _c_primitives(means.detach(), scales.detach(), rotations.detach(), opacities.detach(),
                          precomputed_colors.detach() if precomputed_colors is not None else None,
                          base_colors.detach() if base_colors is not None else None,
                          residual_params.detach() if residual_params is not None else None, mlp)
    state = ForwardState(_rasterizer, prims, rasterizer_settings, device, training=False)
    state.preprocess(prims)
    h, w = int(rasterizer_settings.height), int(rasterizer_settings.width)
    image = torch.empty((3, h, w) if to_chw else (h, w, 3), dtype=torch.float32, device=device)
    state.render_inference(image, to_chw, clamp_output)
    return image


@torch.no_grad()
def update_pruning_scores(
    scores: torch.Tensor,
    means: torch.Tensor,
    scales: torch.Tensor,
    rotations: torch.Tensor,
    opacities: torch.Tensor,
    rasterizer_settings: RasterizerSettings,
    precomputed_colors: torch.Tensor | None = None,
    base_colors: torch.Tensor | None = None,
    residual_params: torch.Tensor | None = None,
    mlp_weights: torch.Tensor | None = None,
) -> None:
    """Adds the view's Speedy-Splat pruning scores to `scores` [N] (contiguous CUDA float32, updated in place):
    per primitive, the sum over its accepted fragments of (opacity * dL/dalpha)^2 for an all-ones image gradient.
    Mirrors torch_bindings/rasterization.py:227-251 (returns None like the reference's binding)."""
    device = means.device
    n = means.shape[0]
    if not scores.is_cuda or scores.dtype != torch.float32 or not scores.is_contiguous() or scores.numel() != n:
        raise RuntimeError('scores must be a contiguous CUDA float32 tensor with one element per Gaussian')
    mlp = mlp_weights.detach() if mlp_weights is not None else None
    prims = _c_primitives(means.detach(), scales.detach(), rotations.detach(), opacities.detach(),
                          precomputed_colors.detach() if precomputed_colors is not None else None,
                          base_colors.detach() if base_colors is not None else None,
                          residual_params.detach() if residual_params is not None else None, mlp)
    state = ForwardState(_rasterizer, prims, rasterizer_settings, device, training=False)
    state.preprocess(prims)
    image = torch.empty((3, int(rasterizer_settings.height), int(rasterizer_settings.width)), dtype=torch.float32, device=device)
    state.render_train(image)
    state.pruning_scores(image, scores)
