"""PLY export of a Gaussian scene in the layout the reference writes (Model.py:502-531, Appearance/Base.py:230-236,
Appearance/SH.py:59-70) and that common 3DGS viewers read: one binary little-endian `vertex` element of float32
properties x, y, z, the appearance columns, opacity (logit), scale_0..2 (log-space), rot_0..3 (normalised quaternion).

Appearance columns: SH appearance with the default activations (base none, residual none, colour relu) stores its
coefficients, f_dc_0..2 = base / C0 and f_rest_i = the degree-1..3 coefficients channel-major (all of red, then green,
then blue). Every other configuration stores only the view-independent colour baked into degree 0,
f_dc = (colour_activation(base_activation(base)) - 0.5) / C0 (viewers reconstruct max(0.5 + C0 f_dc, 0)); the
view-dependent residual is not representable in the format. The writer and reader are this library's own, for the
standard PLY header grammar (format, element, property, comment, end_header).
"""
from __future__ import annotations

from pathlib import Path

import numpy as np
import torch

SH_C0 = 0.28209479177387814


def base_activation(x: torch.Tensor, name: str) -> torch.Tensor:
    return {'none': lambda v: v, 'exp': lambda v: torch.exp(3.0 * v)}[name](x)


def color_activation(x: torch.Tensor, name: str) -> torch.Tensor:
    fns = {
        'none': lambda v: v + 0.5,
        'relu': lambda v: torch.relu(v + 0.5),
        'softplus': lambda v: torch.nn.functional.softplus(v + 0.5, beta=10.0),
        'sigmoid': lambda v: torch.sigmoid(4.0 * v),
        'hardsigmoid': lambda v: torch.nn.functional.hardsigmoid(6.0 * v),
        'satexp': lambda v: -torch.expm1(-v),
    }
    return fns[name](x)


def appearance_columns(model: str, base_colors: torch.Tensor, residual_params: torch.Tensor | None, base_act: str = 'none',
                       residual_act: str = 'none', color_act: str = 'relu') -> tuple[np.ndarray, list[str]]:
    """(columns [N, C], names) of the appearance part of a vertex (rules in the module docstring)."""
    base = base_colors.detach().float().reshape(-1, 3)
    if model == 'sh' and base_act == 'none' and residual_act == 'none' and color_act == 'relu' and residual_params is not None:
        rest = residual_params.detach().float().reshape(base.shape[0], -1, 3).transpose(1, 2).reshape(base.shape[0], -1)
        cols = torch.cat([base / SH_C0, rest], dim=1).cpu().numpy()
        return cols, ['f_dc_0', 'f_dc_1', 'f_dc_2'] + [f'f_rest_{i}' for i in range(rest.shape[1])]
    rgb = color_activation(base_activation(base, base_act), color_act)
    return ((rgb - 0.5) / SH_C0).cpu().numpy(), ['f_dc_0', 'f_dc_1', 'f_dc_2']


def scene_vertices(means: torch.Tensor, scales: torch.Tensor, rotations: torch.Tensor, opacities: torch.Tensor, appearance: np.ndarray,
                   appearance_names: list[str]) -> np.ndarray:
    """Structured float32 vertex array from raw (pre-activation) parameters: means [N,3], log-scales [N,3],
    quaternions [N,4] (normalised here), opacity logits [N,1]."""
    n = means.shape[0]
    q = torch.nn.functional.normalize(rotations.detach().float().reshape(n, 4), dim=1)
    cols = [means.detach().float().reshape(n, 3).cpu().numpy(), appearance.reshape(n, -1),
            opacities.detach().float().reshape(n, 1).cpu().numpy(), scales.detach().float().reshape(n, 3).cpu().numpy(), q.cpu().numpy()]
    names = (['x', 'y', 'z'] + list(appearance_names) + ['opacity'] + ['scale_0', 'scale_1', 'scale_2']
             + ['rot_0', 'rot_1', 'rot_2', 'rot_3'])
    data = np.concatenate(cols, axis=1).astype(np.float32)
    out = np.empty(n, dtype=[(name, '<f4') for name in names])
    for k, name in enumerate(names):
        out[name] = data[:, k]
    return out


def write_ply(path: str | Path, vertices: np.ndarray, comments: list[str] = ()) -> None:
    """Writes one binary little-endian `vertex` element with the structured array's float32 fields."""
    lines = ['ply', 'format binary_little_endian 1.0'] + [f'comment {c}' for c in comments]
    lines.append(f'element vertex {vertices.shape[0]}')
    for name in vertices.dtype.names:
        if vertices.dtype[name] != np.dtype('<f4'):
            raise ValueError(f'property {name} is not float32')
        lines.append(f'property float {name}')
    lines.append('end_header')
    with open(path, 'wb') as f:
        f.write(('\n'.join(lines) + '\n').encode('ascii'))
        f.write(np.ascontiguousarray(vertices).tobytes())


_PLY_TYPES = {'float': '<f4', 'float32': '<f4', 'double': '<f8', 'float64': '<f8', 'uchar': 'u1', 'uint8': 'u1', 'char': 'i1', 'int8': 'i1',
              'short': '<i2', 'int16': '<i2', 'ushort': '<u2', 'uint16': '<u2', 'int': '<i4', 'int32': '<i4', 'uint': '<u4', 'uint32': '<u4'}


def read_ply(path: str | Path) -> tuple[np.ndarray, list[str]]:
    """Reads a binary little-endian PLY whose only element is `vertex` with scalar properties; returns the structured
    array and the comments."""
    raw = Path(path).read_bytes()
    end = raw.index(b'end_header\n') + len(b'end_header\n')
    header = raw[:end].decode('ascii').splitlines()
    if header[0] != 'ply' or header[1] != 'format binary_little_endian 1.0':
        raise ValueError('only binary little-endian PLY files are read')
    comments, fields, count = [], [], None
    for line in header[2:]:
        tok = line.split()
        if tok[0] == 'comment':
            comments.append(line[len('comment '):])
        elif tok[0] == 'element':
            if tok[1] != 'vertex' or count is not None:
                raise ValueError('only a single vertex element is read')
            count = int(tok[2])
        elif tok[0] == 'property':
            if tok[1] == 'list':
                raise ValueError('list properties are not read')
            fields.append((tok[2], _PLY_TYPES[tok[1]]))
    dt = np.dtype(fields)
    return np.frombuffer(raw, dtype=dt, count=count, offset=end).copy(), comments
