"""Seeded synthetic scenes with the shapes and value distributions of the benchmark configurations.

There is no dataset in this environment (the reference trains on Mip-NeRF 360 scenes), so these scenes stand in
for it. All tensors are generated on the CPU with torch.Generator (seed 0 geometry, 1 appearance, 2 upstream
gradients / targets, 3 MLP weights) in fp32, so the GPU path and the CPU checker see identical bits.

Geometry (configs c1-c4): 80% of the means from 8 isotropic clusters (sigma 1) whose centres are uniform in a
radius-6 ball, 20% uniform in a radius-6..20 shell; log-scales ~ N(-4.5, 0.6); uniform random unit quaternions
(normalised N(0, I4), stored as (w, x, y, z)); opacity logits ~ N(0, 1.5). Cameras: pinhole, 60 degree horizontal
field of view, principal point at the image centre, on a ring of radius 10 in the y = 0 plane looking at the
origin, near 0.2, far 1e4, black background.
"""
from __future__ import annotations

import math
from dataclasses import dataclass, field

import torch


@dataclass
class Camera:
    w2c: torch.Tensor          # [4,4] row-major world-to-camera (x right, y down, z forward)
    position: torch.Tensor     # [3]
    width: int
    height: int
    focal_x: float
    focal_y: float
    center_x: float
    center_y: float
    near_plane: float = 0.2
    far_plane: float = 1e4
    bg: torch.Tensor = field(default_factory=lambda: torch.zeros(3))


def look_at(position: torch.Tensor, width: int, height: int, fov_x_deg: float = 60.0) -> Camera:
    c = position.double()
    f = -c / c.norm()
    down0 = torch.tensor([0.0, -1.0, 0.0], dtype=torch.float64)
    r = torch.linalg.cross(down0, f)
    if r.norm() < 1e-9:
        r = torch.tensor([1.0, 0.0, 0.0], dtype=torch.float64)
    r = r / r.norm()
    d = torch.linalg.cross(f, r)
    Rm = torch.stack([r, d, f])
    t = -Rm @ c
    w2c = torch.eye(4, dtype=torch.float64)
    w2c[:3, :3] = Rm
    w2c[:3, 3] = t
    fx = width / (2.0 * math.tan(math.radians(fov_x_deg) / 2.0))
    return Camera(w2c.float(), position.float(), width, height, fx, fx, width / 2.0, height / 2.0)


def ring_cameras(n_views: int, width: int, height: int, radius: float = 10.0) -> list[Camera]:
    cams = []
    for k in range(n_views):
        a = 2.0 * math.pi * k / max(n_views, 1)
        cams.append(look_at(torch.tensor([radius * math.sin(a), 0.0, radius * math.cos(a)]), width, height))
    return cams


def geometry(n: int, seed: int = 0) -> dict[str, torch.Tensor]:
    g = torch.Generator().manual_seed(seed)
    n_cluster = int(round(0.8 * n))
    n_shell = n - n_cluster
    centres = torch.randn(8, 3, generator=g)
    centres = centres / centres.norm(dim=1, keepdim=True) * 6.0 * torch.rand(8, 1, generator=g).pow(1.0 / 3.0)
    which = torch.randint(0, 8, (n_cluster,), generator=g)
    cl = centres[which] + torch.randn(n_cluster, 3, generator=g)
    dirs = torch.randn(n_shell, 3, generator=g)
    dirs = dirs / dirs.norm(dim=1, keepdim=True).clamp_min(1e-12)
    u = torch.rand(n_shell, 1, generator=g)
    rad = (6.0 ** 3 + u * (20.0 ** 3 - 6.0 ** 3)).pow(1.0 / 3.0)
    means = torch.cat([cl, dirs * rad])
    means = means[torch.randperm(n, generator=g)]
    scales = torch.randn(n, 3, generator=g) * 0.6 - 4.5
    q = torch.randn(n, 4, generator=g)
    q = q / q.norm(dim=1, keepdim=True).clamp_min(1e-12)
    opac = torch.randn(n, 1, generator=g) * 1.5
    return {'means': means.contiguous(), 'scales': scales.contiguous(), 'rotations': q.contiguous(), 'opacities': opac.contiguous()}


def sh_appearance(n: int, degree: int = 3, seed: int = 1) -> dict[str, torch.Tensor]:
    g = torch.Generator().manual_seed(seed)
    base = torch.randn(n, 3, generator=g)
    rest = torch.randn(n, (degree + 1) ** 2 - 1, 3, generator=g) * 0.3
    return {'base_colors': base.contiguous(), 'residual_params': rest.contiguous()}


def sv_appearance(n: int, sites: int = 8, seed: int = 1) -> dict[str, torch.Tensor]:
    g = torch.Generator().manual_seed(seed)
    base = torch.randn(n, 3, generator=g)
    p = torch.empty(n, sites, 7)
    s = torch.randn(n, sites, 3, generator=g)
    p[..., 0:3] = s / s.norm(dim=-1, keepdim=True).clamp_min(1e-12)
    p[..., 3] = torch.randn(n, sites, generator=g) * 0.5 + 2.0
    p[..., 4:7] = torch.randn(n, sites, 3, generator=g) * 0.2
    return {'base_colors': base.contiguous(), 'residual_params': p.contiguous()}


def nasg_appearance(n: int, lobes: int = 8, seed: int = 1, gabor: bool = False) -> dict[str, torch.Tensor]:
    g = torch.Generator().manual_seed(seed)
    base = torch.randn(n, 3, generator=g)
    stride = 9 if gabor else 8
    p = torch.empty(n, lobes, stride)
    p[..., 0:3] = torch.randn(n, lobes, 3, generator=g)  # raw frame angles (tanh -> cosines), a random frame
    p[..., 3] = torch.randn(n, lobes, generator=g) * 0.5 + 1.0  # log sharpness
    p[..., 4] = torch.randn(n, lobes, generator=g) * 0.5  # log anisotropy
    w0 = 5
    if gabor:
        p[..., 5] = torch.randn(n, lobes, generator=g) * 0.5 - 1.6
        w0 = 6
    p[..., w0:w0 + 3] = torch.randn(n, lobes, 3, generator=g) * 0.2
    return {'base_colors': base.contiguous(), 'residual_params': p.contiguous()}


def neural_appearance(n: int, feature_dim: int = 32, n_params: int = 0, seed: int = 1, mlp_seed: int = 3,
                      layer_shapes: list[tuple[int, int]] | None = None) -> dict[str, torch.Tensor]:
    """Latents ~ N(0, 0.1); MLP weights Kaiming-uniform per layer (bound sqrt(6 / fan_in)), all layers random."""
    g = torch.Generator().manual_seed(seed)
    base = torch.randn(n, 3, generator=g)
    lat = torch.randn(n, feature_dim, generator=g) * 0.1
    out = {'base_colors': base.contiguous(), 'residual_params': lat.contiguous()}
    if layer_shapes:
        gm = torch.Generator().manual_seed(mlp_seed)
        parts = []
        for rows, cols in layer_shapes:
            bound = math.sqrt(6.0 / cols)
            parts.append((torch.rand(rows * cols, generator=gm) * 2.0 - 1.0) * bound)
        w = torch.cat(parts)
        assert n_params == 0 or w.numel() == n_params
        out['mlp_weights'] = w.contiguous()
    return out


def mlp_layer_shapes(n_input_pad: int, n_neurons: int, n_hidden: int) -> list[tuple[int, int]]:
    return [(n_neurons, n_input_pad)] + [(n_neurons, n_neurons)] * (n_hidden - 1) + [(16, n_neurons)]
