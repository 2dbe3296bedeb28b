"""Test and baseline infrastructure only: a PyTorch (CPU) restatement of the reference's unfused appearance path for
spherical harmonics, the computation its `USE_FUSED_APPEARANCE=false` mode runs in PyTorch (Appearance/Base.py:83-108
forward, Appearance/SH.py:33-55 residual_colors, Appearance/utils.py:130-200 activations). Its backward is PyTorch
autograd, as in the reference. The reference's modules need the absent NeRFICG framework and cannot be imported where
the benchmark runs, so bench.py times this restatement as the reference's CPU path (configuration c0); the tests pin it
against fixtures the reference's own modules produced (tests/golden/appearance_*.npz, tests/test_oracle_golden.py)."""
from __future__ import annotations

import torch

SH_C1 = 0.48860251190291987
SH_C2 = (1.0925484305920792, 0.94617469575755997, 0.31539156525251999, 0.54627421529603959)
SH_C3 = (0.59004358992664352, 1.7701307697799304, 2.8906114426405538, 0.45704579946446572, 2.2852289973223288, 1.865881662950577,
         1.1195289977703462, 1.4453057213202769)


def base_activation(x: torch.Tensor, act: str) -> torch.Tensor:
    return x if act == 'none' else torch.exp(3.0 * x)


def residual_activation(x: torch.Tensor, act: str) -> torch.Tensor:
    if act == 'none':
        return x
    if act == 'tanh':
        return torch.tanh(x)
    return torch.nn.functional.softplus(x, beta=10.0)


def color_activation(x: torch.Tensor, act: str) -> torch.Tensor:
    if act == 'none':
        return x + 0.5
    if act == 'relu':
        return torch.relu(x + 0.5)
    if act == 'softplus':
        return torch.nn.functional.softplus(x + 0.5, beta=10.0)
    if act == 'sigmoid':
        return torch.sigmoid(4.0 * x)
    if act == 'hardsigmoid':
        return torch.nn.functional.hardsigmoid(6.0 * x)
    return -torch.expm1(-x)


def sh_residual(d: torch.Tensor, rest: torch.Tensor, degree: int) -> torch.Tensor:
    """Sum of the SH bands 1..degree of unit directions d [N,3] with coefficients rest [N, bases, 3] -> [N,3]."""
    x, y, z = d[:, 0:1], d[:, 1:2], d[:, 2:3]
    r = -SH_C1 * y * rest[:, 0] + SH_C1 * z * rest[:, 1] - SH_C1 * x * rest[:, 2]
    if degree > 1:
        xx, yy, zz, xy, xz, yz = x * x, y * y, z * z, x * y, x * z, y * z
        a, b, c, e = SH_C2
        r = r + a * xy * rest[:, 3] - a * yz * rest[:, 4] + (b * zz - c) * rest[:, 5] - a * xz * rest[:, 6] + e * (xx - yy) * rest[:, 7]
        if degree > 2:
            k0, k1, k2, k3, k4, k5, k6, k7 = SH_C3
            r = (r + y * (k0 * yy - k1 * xx) * rest[:, 8] + k2 * xy * z * rest[:, 9] + y * (k3 - k4 * zz) * rest[:, 10]
                 + z * (k5 * zz - k6) * rest[:, 11] + x * (k3 - k4 * zz) * rest[:, 12] + k7 * z * (xx - yy) * rest[:, 13]
                 + x * (k1 * yy - k0 * xx) * rest[:, 14])
    return r


def sh_colors(means: torch.Tensor, cam: torch.Tensor, base: torch.Tensor, rest: torch.Tensor, degree: int, base_act: str = 'none',
              residual_act: str = 'none', color_act: str = 'relu') -> torch.Tensor:
    """color_activation(base_activation(base) + residual_activation(SH bands of the unit view direction))."""
    d = torch.nn.functional.normalize(means - cam)
    return color_activation(base_activation(base, base_act) + residual_activation(sh_residual(d, rest, degree), residual_act), color_act)
