"""Viewer export: the `.ngsplat` file the reference's web viewer loads, written from this library's parameter tensors.

Format (defined by the reference's viewer/export_ngsplat.py, whose docstring documents it; little-endian):
  magic "NGSPLAT\\n"; eleven u32 (splat count, texture width 2048, texture height, model dims, frequencies, degree mask,
  colour activation code, residual activation code, neurons, hidden layers, flags); f32 base scale and offset; for SH
  three f32 per-level quantisation scales; f32x3 orbit centre, f32x3 up, f32 distance; u32 test-camera count and
  f32x18 per camera; u32 weight-texel count and the fp16 weight texels (Neural); one RGBA32UI geometry texel per
  splat (rgb8 base code + opacity8, fp16 position, 24-bit octahedral rotation code, three 8-bit log-scale codes),
  padded to whole texture rows; then the per-splat residual textures of the appearance model.

Per model the residual payload is what the viewer evaluates per frame without further activation: SH keeps the raw
coefficients, quantised per degree level (7/8/6-bit signed fields bit-packed into 2/4/4 words); SV stores unit site
directions, exp'd temperatures (capped at 60000) and activated site colours; NASG and NASGabor store the baked lobe
frame (x and z axes), 2*lambda, anisotropy, (NASGabor: frequency,) normalisation and activated colours; Neural stores
either the view-independent share of layer 0 per splat ("baked", with only the direction columns of layer 0 in the
weight stream) or the encoded features and the whole network. The appearance schedule position (active_degree)
trims SH degrees and lobes, gates the not-yet-enabled direction degrees of the Neural input layer, and zeroes the
Neural output layer before any degree is enabled.

Splats whose opacity is below 1/255 are dropped. The numbers are produced with the same float32 numpy operations as
the reference exporter, so the file is byte-identical to the reference's for the same parameters (tests against
files exported by the reference: tests/golden/ngsplat_*.npz). Test cameras can be passed in; PPISP is not part of
this library, so its block is never written.
"""
from __future__ import annotations

import math
import struct
from dataclasses import dataclass
from pathlib import Path

import numpy as np

MAGIC = b'NGSPLAT\n'
ROW_TEXELS = 2048
MIN_OPACITY = 1.0 / 255.0
SH_C0 = 0.28209479177387814
LOG_SCALE_LO, LOG_SCALE_HI = -12.0, 9.0
LOG_SCALE_STEP = 254.0 / (LOG_SCALE_HI - LOG_SCALE_LO)
MODEL_IDS = {'neural': 0, 'sh': 1, 'sv': 2, 'nasg': 3, 'nasgabor': 4}
COLOR_CODES = {'relu': 0, 'softplus': 1, 'sigmoid': 2, 'satexp': 3, 'hardsigmoid': 4, 'none': 5}
RESIDUAL_CODES = {'none': 0, 'tanh': 1, 'softplus': 2}
GRAY_SHIFTED = ('none', 'relu', 'softplus', 'hardsigmoid')  # colour activations of the form act(x + 0.5)
SH_LEVEL_FIELDS = {1: (7, 2), 2: (8, 4), 3: (6, 4)}  # degree -> (bits per field, u32 words per splat)
MAX_HALF_VALUES = 64  # the viewer reads at most 8 textures of 8 fp16 values
TEMPERATURE_CAP = 60000.0
SITE_EPS = 1e-12
LOBE_COS_LIMIT = 0.999999
LOBE_SHAPE_LIMIT = 1e4
LOBE_NORM_EPS = 1e-8
GABOR_FREQUENCY_SCALE = 20.0


@dataclass
class ViewerAppearance:
    """Appearance configuration of the exported scene (the reference's MODEL.APPEARANCE fields)."""
    model: str
    base_activation: str = 'none'
    residual_activation: str = 'none'
    color_activation: str = 'relu'
    active_degree: int | None = None  # appearance schedule position; None: every degree / lobe enabled
    # Neural only
    feature_frequencies: int = 1
    sh_degrees: tuple = (0, 1, 2, 3)
    n_neurons: int = 16
    n_hidden_layers: int = 2
    base_input: bool = False


def _f32(x) -> np.ndarray:
    if hasattr(x, 'detach'):
        x = x.detach().cpu().numpy()
    return np.asarray(x, dtype=np.float32)


def _half_words(a: np.ndarray) -> np.ndarray:
    return a.astype(np.float16).view(np.uint16).astype(np.uint32)


def _residual_act(x: np.ndarray, name: str) -> np.ndarray:
    if name == 'tanh':
        return np.tanh(x)
    if name == 'softplus':  # beta 10, linear above 2
        return np.where(x > 2.0, x, np.log1p(np.exp(10.0 * np.minimum(x, 2.0))) / 10.0)
    return x


# ---- geometry texel -------------------------------------------------------------------------------------------

def _log_scale_codes(scales: np.ndarray) -> np.ndarray:
    """8-bit codes of log(scale) over [LOG_SCALE_LO, LOG_SCALE_HI]: 1..255, 0 for a zero scale."""
    level = np.maximum(0.0, (np.log(np.maximum(scales, 1e-30)) - LOG_SCALE_LO) * LOG_SCALE_STEP)
    codes = np.minimum(255, np.round(level) + 1).astype(np.uint32)
    codes[scales == 0.0] = 0
    return codes


def _rotation_codes(q: np.ndarray) -> np.ndarray:
    """24-bit codes of unit quaternions (x, y, z, w): rotation angle in bits 16-23, the rotation axis as a folded
    octahedral point (u in bits 0-7, v in bits 8-15)."""
    q = np.where(q[:, 3:4] < 0.0, -q, q)
    half = np.arccos(np.clip(q[:, 3], -1.0, 1.0))
    angle = 2.0 * half
    s = np.sin(half)
    tiny = np.abs(s) < 1e-6
    axis = q[:, :3] / np.where(tiny, 1.0, s)[:, None]
    axis[tiny] = (1.0, 0.0, 0.0)
    l1 = np.abs(axis).sum(axis=1)
    u, v = axis[:, 0] / l1, axis[:, 1] / l1
    lower = axis[:, 2] < 0.0
    u_fold = (1.0 - np.abs(v)) * np.where(u >= 0.0, 1.0, -1.0)
    v_fold = (1.0 - np.abs(u)) * np.where(v >= 0.0, 1.0, -1.0)
    u, v = np.where(lower, u_fold, u), np.where(lower, v_fold, v)

    def byte(x):
        return np.round(np.clip(x, 0.0, 255.0)).astype(np.uint32)

    return byte(angle / math.pi * 255.0) << 16 | byte((v * 0.5 + 0.5) * 255.0) << 8 | byte((u * 0.5 + 0.5) * 255.0)


def _geometry_texels(means, scales, quats_xyzw, base_codes, opacity_codes, padded: int) -> np.ndarray:
    n = means.shape[0]
    rot = _rotation_codes(quats_xyzw)
    sc = _log_scale_codes(scales)
    out = np.zeros((padded, 4), np.uint32)
    out[:n, 0] = base_codes[:, 0] | base_codes[:, 1] << 8 | base_codes[:, 2] << 16 | opacity_codes << 24
    out[:n, 1] = _half_words(means[:, 0]) | _half_words(means[:, 1]) << 16
    out[:n, 2] = _half_words(means[:, 2]) | (rot & 0xFF) << 16 | (rot >> 8 & 0xFF) << 24
    out[:n, 3] = sc[:, 0] | sc[:, 1] << 8 | sc[:, 2] << 16 | (rot >> 16) << 24
    return out


def _half_textures(values: np.ndarray, padded: int) -> list:
    """[n, V] floats -> ceil(V / 8) RGBA32UI textures of 8 fp16 values (two per channel, low half first)."""
    n, count = values.shape
    tex = (count + 7) // 8
    full = np.zeros((padded, 8 * tex), np.float32)
    full[:n, :count] = values
    bits = _half_words(full)
    return [(bits[:, 8 * t:8 * t + 8:2] | bits[:, 8 * t + 1:8 * t + 8:2] << 16).astype(np.uint32) for t in range(tex)]


def _weight_texels(layers: list) -> np.ndarray:
    """fp16 texel stream of the MLP: per layer W [out x in] (in a multiple of 4), texel j * out + o = W[o, 4j:4j+4]."""
    blocks = []
    for w in layers:
        rows, cols = w.shape
        if cols % 4:
            raise ValueError(f'layer input width {cols} is not a multiple of 4')
        blocks.append(w.reshape(rows, cols // 4, 4).transpose(1, 0, 2).reshape(-1, 4))
    return np.concatenate(blocks).astype(np.float32).astype(np.float16).view(np.uint16)


# ---- residual payloads ----------------------------------------------------------------------------------------

def _sh_payload(coef: np.ndarray, padded: int, active: int | None):
    """Raw SH coefficients [n, C, 3] -> (textures, level scales, degree mask); degrees beyond the schedule dropped."""
    n, count, _ = coef.shape
    degree = int(round(math.sqrt(count + 1))) - 1
    if (degree + 1) ** 2 - 1 != count or degree > 3:
        raise ValueError(f'{count} SH coefficients are not complete degrees 1..3')
    degree = min(degree if active is None else active, degree)
    coef = coef[:, :(degree + 1) ** 2 - 1, :].astype(np.float32)
    textures, level_scales, first = [], [], 0
    for level, (bits, words) in SH_LEVEL_FIELDS.items():
        width = 2 * level + 1
        if first + width > coef.shape[1]:
            level_scales.append(0.0)
            continue
        vals = coef[:, first:first + width, :].reshape(n, -1)
        scale = max(float(np.abs(vals).max(initial=0.0)), 1e-8)
        top = (1 << (bits - 1)) - 1
        codes = np.clip(np.round(vals / scale * top), -top, top).astype(np.int32)
        codes = (codes & ((1 << bits) - 1)).astype(np.uint32)
        packed = np.zeros((padded, words), np.uint32)
        for k in range(codes.shape[1]):
            pos = bits * k
            w, shift = divmod(pos, 32)
            packed[:n, w] |= codes[:, k] << shift
            if shift + bits > 32:
                packed[:n, w + 1] |= codes[:, k] >> (32 - shift)
        textures.append(packed)
        level_scales.append(scale)
        first += width
    return textures, level_scales, sum(1 << d for d in range(1, degree + 1))


def _sv_values(params: np.ndarray, residual_act: str) -> np.ndarray:
    """[n, S, 7] (site xyz, log temperature, rgb) -> [n, 7S] unit sites, capped temperatures, activated colours."""
    sites = params[..., 0:3]
    length = np.maximum(np.linalg.norm(sites, axis=-1, keepdims=True), SITE_EPS)
    temperature = np.minimum(np.exp(params[..., 3:4]), TEMPERATURE_CAP)
    return np.concatenate([sites / length, temperature, _residual_act(params[..., 4:7], residual_act)],
                          axis=-1).reshape(params.shape[0], -1).astype(np.float32)


def _lobe_values(params: np.ndarray, residual_act: str, gabor: bool) -> np.ndarray:
    """[n, L, 8 | 9] raw lobes -> [n, 12L | 13L]: frame x axis, frame z axis, 2 lambda, anisotropy, (Gabor
    frequency,) normalisation, activated colour."""
    c = np.clip(np.tanh(params[..., 0:3]), -LOBE_COS_LIMIT, LOBE_COS_LIMIT)
    s = np.sqrt(1.0 - c * c)
    ct, cp, cu = c[..., 0], c[..., 1], c[..., 2]
    st, sp, su = s[..., 0], s[..., 1], s[..., 2]
    x_axis = np.stack([ct * cp * cu - st * su, st * cp * cu + ct * su, -sp * cu], axis=-1)
    z_axis = np.stack([ct * sp, st * sp, cp], axis=-1)
    lam = np.minimum(np.exp(params[..., 3]), LOBE_SHAPE_LIMIT)
    aniso = np.minimum(np.exp(params[..., 4]), LOBE_SHAPE_LIMIT)
    norm = lam * np.sqrt(1.0 + aniso) / (2.0 * math.pi * (1.0 + LOBE_NORM_EPS - np.exp(-2.0 * lam)))
    cols = [x_axis, z_axis, (2.0 * lam)[..., None], aniso[..., None]]
    if gabor:
        cols.append(((np.tanh(params[..., 5]) + 1.0) * GABOR_FREQUENCY_SCALE)[..., None])
    cols += [norm[..., None], _residual_act(params[..., 6:9] if gabor else params[..., 5:8], residual_act)]
    return np.concatenate(cols, axis=-1).reshape(params.shape[0], -1).astype(np.float32)


def _neural_payload(features: np.ndarray, base: np.ndarray, weights: np.ndarray, a: ViewerAppearance, padded: int):
    """Returns (textures, weight texels, header dims, degree mask, flag bits)."""
    degrees = list(a.sh_degrees)
    if degrees != sorted(set(degrees)) or not any(d > 0 for d in degrees) or any(d < 0 or d > 6 for d in degrees):
        raise ValueError(f'SH degrees {degrees} must ascend in [0, 6] and include a direction degree')
    if a.n_neurons % 4 or a.n_neurons < 4:
        raise ValueError('the viewer needs a multiple of 4 neurons')
    raw = np.concatenate([features, base], axis=-1) if a.base_input else features
    freqs = a.feature_frequencies
    enc_dim = raw.shape[1] * (2 * freqs if freqs else 1)
    with_c0 = 0 in degrees
    direction = [d for d in degrees if d > 0]
    n_dir = sum(2 * d + 1 for d in direction)
    n_in = enc_dim + sum(2 * d + 1 for d in degrees)
    nn, nh = a.n_neurons, a.n_hidden_layers
    shapes = [(nn, n_in)] + [(nn, nn)] * (nh - 1) + [(16, nn)]
    w16 = np.asarray(weights, np.float32).astype(np.float16).astype(np.float32).reshape(-1)
    if w16.size != sum(r * c for r, c in shapes):
        raise ValueError(f'{w16.size} MLP weights do not match a {n_in}-input network (the input must fill a multiple of 16)')
    layers, at = [], 0
    for r, c in shapes:
        layers.append(w16[at:at + r * c].reshape(r, c))
        at += r * c
    layers[-1] = layers[-1][:3]
    active = len(direction) if a.active_degree is None else a.active_degree
    if active == 0:  # the rasterizer skips the MLP: no residual at all
        if a.residual_activation == 'softplus':
            raise ValueError('softplus maps a zero MLP output to a non-zero residual; export a checkpoint with a direction degree enabled')
        layers[-1][:] = 0.0
    elif active < len(direction):  # input columns of the not-yet-enabled direction degrees
        col, rank = enc_dim, 0
        for d in degrees:
            if d > 0:
                if rank >= active:
                    layers[0][:, col:col + 2 * d + 1] = 0.0
                rank += 1
            col += 2 * d + 1
    if freqs:
        arg = raw[..., None] * np.exp2(np.arange(freqs, dtype=np.float32))
        encoded = np.stack([np.sin(arg), np.cos(arg)], axis=-1).reshape(raw.shape[0], -1).astype(np.float32)
    else:
        encoded = raw
    baked = nn <= 16 and -(-nn // 8) <= -(-enc_dim // 8)
    if baked:
        w0 = layers[0]
        static = encoded @ w0[:, :enc_dim].T
        if with_c0:
            static = static + SH_C0 * w0[:, enc_dim]
        static = static.astype(np.float16).astype(np.float32)
        w0_dir = np.zeros((nn, (n_dir + 3) // 4 * 4), np.float32)
        w0_dir[:, :n_dir] = w0[:, enc_dim + (1 if with_c0 else 0):]
        textures, texels = _half_textures(static, padded), _weight_texels([w0_dir] + layers[1:])
    else:
        if enc_dim > 16:
            raise ValueError(f'{enc_dim} encoded features exceed the viewer\'s two feature textures')
        textures, texels = _half_textures(encoded, padded), _weight_texels(layers)
    flags = (0 if with_c0 else 2) | (4 if baked else 0)
    return textures, texels, enc_dim, sum(1 << d for d in direction), flags


# ---- writer ---------------------------------------------------------------------------------------------------

def export_ngsplat(path, means, scales, rotations, opacities, base_colors, residual_params, appearance: ViewerAppearance,
                   mlp_weights=None, proper_antialiasing: bool = False, center=None, up=None, distance=None,
                   test_cameras=None) -> dict:
    """Writes a .ngsplat file from raw (pre-activation) parameters: means [N,3], log-scales [N,3], quaternions (w, x,
    y, z) [N,4], opacity logits [N] or [N,1], base colours [N,3], residual parameters (SH [N,15,3], SV [N,S,7], NASG
    [N,L,8], NASGabor [N,L,9], Neural [N,F], flat rows accepted), and for Neural the flat MLP weights in the
    tiny-cuda-nn layout. `center` / `up` / `distance` override the orbit hint (median of the means, -y, 1.5x the
    median distance to the centre); `test_cameras` [V,18] are the viewer's benchmark viewpoints. Returns a summary."""
    a = appearance
    if a.model not in MODEL_IDS or a.color_activation not in COLOR_CODES or a.residual_activation not in RESIDUAL_CODES \
            or a.base_activation not in ('none', 'exp'):
        raise ValueError(f'unsupported appearance {a}')
    q = _f32(rotations)
    q /= np.linalg.norm(q, axis=1, keepdims=True)
    op = 1.0 / (1.0 + np.exp(-_f32(opacities).reshape(-1)))
    keep = op >= MIN_OPACITY
    mu = _f32(means)[keep]
    sc = np.exp(_f32(scales))[keep]
    qx = q[:, [1, 2, 3, 0]][keep]
    op = op[keep]
    base_raw = _f32(base_colors)[keep]
    res = _f32(residual_params)
    res = res[keep]
    n = mu.shape[0]

    shift = 0.5 if a.color_activation in GRAY_SHIFTED and a.base_activation == 'none' else 0.0
    base = (shift + base_raw).astype(np.float32)
    lo, hi = float(base.min()), float(base.max())
    step = max(hi - lo, 1e-6) / 255.0
    base_codes = np.round((base - lo) / step).clip(0, 255).astype(np.uint32)
    opacity_codes = np.round(op * 255.0).clip(0, 255).astype(np.uint32)
    rows = (n + ROW_TEXELS - 1) // ROW_TEXELS
    padded = rows * ROW_TEXELS
    geometry = _geometry_texels(mu, sc, qx, base_codes, opacity_codes, padded)

    texels = np.zeros((0, 4), np.uint16)
    level_scales = None
    dims = freqs = neurons = hidden = mask = extra_flags = 0
    if a.model == 'neural':
        if mlp_weights is None:
            raise ValueError('the Neural appearance needs mlp_weights')
        textures, texels, dims, mask, extra_flags = _neural_payload(res.reshape(n, -1), base_raw, _f32(mlp_weights), a, padded)
        freqs, neurons, hidden = a.feature_frequencies, a.n_neurons, a.n_hidden_layers
    elif a.model == 'sh':
        textures, level_scales, mask = _sh_payload(res.reshape(n, -1, 3), padded, a.active_degree)
    else:
        per = {'sv': 7, 'nasg': 8, 'nasgabor': 9}[a.model]
        res = res.reshape(n, -1, per)
        if a.model == 'sv':
            values, dims = _sv_values(res, a.residual_activation), res.shape[1]
        else:
            lobes = res.shape[1] if a.active_degree is None else min(a.active_degree, res.shape[1])
            values, dims = _lobe_values(res[:, :lobes], a.residual_activation, a.model == 'nasgabor'), lobes
        if values.shape[1] > MAX_HALF_VALUES:
            raise ValueError(f'{values.shape[1]} residual values per splat exceed the viewer\'s {MAX_HALF_VALUES}')
        textures = _half_textures(values, padded)

    ctr = np.asarray(center, np.float32) if center is not None else np.median(mu, axis=0).astype(np.float32)
    radius = float(np.median(np.linalg.norm(mu - ctr, axis=1))) if n else 1.0
    upv = np.asarray(up if up is not None else (0.0, -1.0, 0.0), np.float32)
    upv = upv / np.linalg.norm(upv)
    dist = float(distance) if distance is not None else 1.5 * radius
    model_id = MODEL_IDS[a.model]
    flags = (1 if proper_antialiasing else 0) | (model_id & 3) << 3 | (model_id >> 2) << 6 | extra_flags
    if a.base_activation == 'exp':
        flags |= 32
    cams = np.zeros((0, 18), np.float32) if test_cameras is None else np.asarray(test_cameras, np.float32).reshape(-1, 18)

    parts = [MAGIC, struct.pack('<11I', n, ROW_TEXELS, rows, dims, freqs, mask, COLOR_CODES[a.color_activation],
                                RESIDUAL_CODES[a.residual_activation], neurons, hidden, flags), struct.pack('<2f', step, lo)]
    if level_scales is not None:
        parts.append(struct.pack('<3f', *level_scales))
    parts += [struct.pack('<3f', *ctr.tolist()), struct.pack('<3f', *upv.tolist()), struct.pack('<f', dist),
              struct.pack('<I', cams.shape[0]), cams.astype('<f4').tobytes(), struct.pack('<I', texels.shape[0]),
              texels.astype('<u2').tobytes(), geometry.astype('<u4').tobytes()]
    parts += [t.astype('<u4').tobytes() for t in textures]
    Path(path).write_bytes(b''.join(parts))
    return {'splats': n, 'culled': int((~keep).sum()), 'bytes_per_splat': 16 + 4 * sum(t.shape[1] for t in textures),
            'weight_texels': int(texels.shape[0])}


# ---- reader ---------------------------------------------------------------------------------------------------

def read_ngsplat(path) -> dict:
    """Parses a .ngsplat file into its header fields and raw payload arrays (geometry [P,4] u32, weight texels [T,4]
    u16, residual textures [P,c] u32)."""
    return read_ngsplat_bytes(Path(path).read_bytes())


def read_ngsplat_bytes(raw: bytes) -> dict:
    """read_ngsplat on the file's bytes."""
    if raw[:8] != MAGIC:
        raise ValueError('not an .ngsplat file')
    at = 8
    names = ('n', 'tex_width', 'tex_height', 'model_dims', 'frequencies', 'degree_mask', 'color_activation',
             'residual_activation', 'n_neurons', 'n_hidden_layers', 'flags')
    out = dict(zip(names, struct.unpack_from('<11I', raw, at)))
    at += 44
    out['base_scale'], out['base_offset'] = struct.unpack_from('<2f', raw, at)
    at += 8
    model_id = (out['flags'] >> 3 & 3) | (out['flags'] >> 6 & 1) << 2
    model = {v: k for k, v in MODEL_IDS.items()}[model_id]
    out['model'] = model
    if model == 'sh':
        out['sh_level_scales'] = struct.unpack_from('<3f', raw, at)
        at += 12
    out['center'] = struct.unpack_from('<3f', raw, at)
    out['up'] = struct.unpack_from('<3f', raw, at + 12)
    out['distance'] = struct.unpack_from('<f', raw, at + 24)[0]
    at += 28
    n_cams = struct.unpack_from('<I', raw, at)[0]
    at += 4
    out['test_cameras'] = np.frombuffer(raw, '<f4', 18 * n_cams, at).reshape(n_cams, 18)
    at += 72 * n_cams
    if out['flags'] & 128:
        raise ValueError('PPISP blocks are not read')
    n_texels = struct.unpack_from('<I', raw, at)[0]
    at += 4
    out['weight_texels'] = np.frombuffer(raw, '<u2', 4 * n_texels, at).reshape(n_texels, 4)
    at += 8 * n_texels
    padded = out['tex_width'] * out['tex_height']
    out['geometry'] = np.frombuffer(raw, '<u4', 4 * padded, at).reshape(padded, 4)
    at += 16 * padded
    if model == 'sh':
        widths = [SH_LEVEL_FIELDS[d][1] for d in (1, 2, 3) if out['degree_mask'] >> d & 1]
    elif model == 'neural':
        count = out['n_neurons'] if out['flags'] & 4 else out['model_dims']
        widths = [4] * ((count + 7) // 8)
    else:
        count = out['model_dims'] * {'sv': 7, 'nasg': 12, 'nasgabor': 13}[model]
        widths = [4] * ((count + 7) // 8)
    textures = []
    for c in widths:
        textures.append(np.frombuffer(raw, '<u4', c * padded, at).reshape(padded, c))
        at += 4 * c * padded
    out['textures'] = textures
    if at != len(raw):
        raise ValueError(f'{len(raw) - at} trailing bytes')
    return out
