"""Generates the appearance golden vectors from the reference's own PyTorch modules.

Imports Appearance/SH.py, SV.py, NASG.py and NASGabor.py from the reference checkout ($FGS_REFERENCE) unmodified,
with small stand-ins for the NeRFICG framework modules they import but that are absent from the checkout
(Framework, Logging, Datasets.utils, Optim.*, Thirdparty.TinyCudaNN and the backend package). For each model it
evaluates AppearanceModel.forward (color_activation(base_activation(base) + residual(dir))) on seeded inputs on the
CPU in float64 and records the colors and the autograd gradients for a seeded upstream gradient. The fixtures are
written to tests/golden/appearance_<model>.npz and committed; the tests never read the reference at run time.

Run: python tests/golden/make_golden.py <reference checkout>   (or set $FGS_REFERENCE)
"""
import importlib
import os
import sys
import types
from pathlib import Path

import numpy as np
import torch

REF = Path(sys.argv[1] if len(sys.argv) > 1 else os.environ.get('FGS_REFERENCE', ''))
if not str(REF) or not (REF / 'Appearance').is_dir():
    raise SystemExit('pass the reference checkout (the directory holding Appearance/) as the first argument or in $FGS_REFERENCE')
OUT = Path(__file__).resolve().parent


def _install_shims() -> None:
    class ConfigParameterList(dict):
        def __getattr__(self, k):
            try:
                return self[k]
            except KeyError as e:
                raise AttributeError(k) from e

    fw = types.ModuleType('Framework')
    fw.ConfigParameterList = ConfigParameterList
    fw.ModelError = RuntimeError
    fw.ExtensionError = RuntimeError
    sys.modules['Framework'] = fw
    log = types.ModuleType('Logging')
    log.Logger = type('Logger', (), {'log_warning': staticmethod(lambda *a, **k: None), 'log_info': staticmethod(lambda *a, **k: None)})
    sys.modules['Logging'] = log
    ds = types.ModuleType('Datasets')
    dsu = types.ModuleType('Datasets.utils')
    dsu.View = object
    sys.modules['Datasets'] = ds
    sys.modules['Datasets.utils'] = dsu
    optim = types.ModuleType('Optim')
    for name, attrs in (('Optim.adam_utils', ('extend_param_groups', 'prune_param_groups', 'reset_state', 'sort_param_groups')),
                        ('Optim.lr_utils', ('CosineDecayPolicy', 'LRDecayPolicy')), ('Optim.knn_utils', ('compute_knn_distances',))):
        m = types.ModuleType(name)
        for a in attrs:
            setattr(m, a, None)
        sys.modules[name] = m
    sys.modules['Optim'] = optim
    tp = types.ModuleType('Thirdparty')
    tcnn = types.ModuleType('Thirdparty.TinyCudaNN')
    sys.modules['Thirdparty'] = tp
    sys.modules['Thirdparty.TinyCudaNN'] = tcnn
    # package alias Methods.FasterGSVDA -> reference root, with a stub backend
    methods = types.ModuleType('Methods')
    methods.__path__ = []
    fg = types.ModuleType('Methods.FasterGSVDA')
    fg.__path__ = [str(REF)]
    backend = types.ModuleType('Methods.FasterGSVDA.FasterGSVDACudaBackend')
    backend.FusedAdam = None
    backend.initialize_appearance = lambda *a, **k: None
    backend.initialize_residual_mlp = lambda *a, **k: None
    sys.modules['Methods'] = methods
    sys.modules['Methods.FasterGSVDA'] = fg
    sys.modules['Methods.FasterGSVDA.FasterGSVDACudaBackend'] = backend
    app_pkg = types.ModuleType('Methods.FasterGSVDA.Appearance')
    app_pkg.__path__ = [str(REF / 'Appearance')]
    sys.modules['Methods.FasterGSVDA.Appearance'] = app_pkg


def _config(model: str, degree: int, base: str, residual: str, color: str):
    fw = sys.modules['Framework']
    C = fw.ConfigParameterList
    return C(TYPE=model, BASE_ACTIVATION=base, RESIDUAL_ACTIVATION=residual, COLOR_ACTIVATION=color, DIRECTION_GRADIENT=True,
             SH=C(SH_DEGREE=degree), SV=C(N_SITES=degree), NASG=C(N_LOBES=degree), NASGABOR=C(N_LOBES=degree))


def _inputs(model: str, n: int, degree: int, seed: int):
    g = torch.Generator().manual_seed(seed)
    base = torch.randn(n, 3, generator=g, dtype=torch.float64)
    if model == 'SH':
        res = torch.randn(n, (degree + 1) ** 2 - 1, 3, generator=g, dtype=torch.float64) * 0.3
    elif model == 'SV':
        res = torch.empty(n, degree, 7, dtype=torch.float64)
        s = torch.randn(n, degree, 3, generator=g, dtype=torch.float64)
        res[..., :3] = s / s.norm(dim=-1, keepdim=True)
        res[..., 3] = torch.randn(n, degree, generator=g, dtype=torch.float64) * 0.5 + 2.0
        res[..., 4:] = torch.randn(n, degree, 3, generator=g, dtype=torch.float64) * 0.2
    else:
        stride = 9 if model == 'NASGabor' else 8
        res = torch.randn(n, degree, stride, generator=g, dtype=torch.float64) * 0.5
        res[..., 3] += 1.0
    means = torch.randn(n, 3, generator=g, dtype=torch.float64) * 3.0
    cam = torch.tensor([0.5, -1.0, 9.0], dtype=torch.float64)
    grad = torch.randn(n, 3, generator=g, dtype=torch.float64)
    return base, res, means, cam, grad


CASES = [
    ('SH', 3, 'none', 'none', 'relu'),
    ('SH', 2, 'exp', 'tanh', 'satexp'),
    ('SV', 8, 'none', 'none', 'relu'),
    ('SV', 5, 'none', 'softplus', 'sigmoid'),
    ('NASG', 8, 'none', 'tanh', 'relu'),
    ('NASG', 3, 'none', 'none', 'softplus'),
    ('NASGabor', 4, 'none', 'tanh', 'relu'),
    ('NASGabor', 2, 'exp', 'softplus', 'hardsigmoid'),
]


def main() -> None:
    _install_shims()
    torch.set_default_dtype(torch.float64)
    for k, (model, degree, base_act, res_act, col_act) in enumerate(CASES):
        module = importlib.import_module(f'Methods.FasterGSVDA.Appearance.{model}')
        cls = getattr(module, model)
        app = cls(_config(model, degree, base_act, res_act, col_act))
        app.active_degree = degree
        n = 64
        base, res, means, cam, grad = _inputs(model, n, degree, seed=100 + k)
        app._base_colors = torch.nn.Parameter(base.clone())
        app._residual_params = torch.nn.Parameter(res.clone())
        means_p = torch.nn.Parameter(means.clone())
        view = types.SimpleNamespace(position=cam)
        colors = app(means_p, view)
        (colors * grad).sum().backward()
        np.savez(OUT / f'appearance_{k}_{model.lower()}.npz', model=model.lower(), degree=degree, base_act=base_act, residual_act=res_act,
                 color_act=col_act, base=base.numpy(), residual=res.numpy(), means=means.numpy(), cam=cam.numpy(), upstream=grad.numpy(),
                 colors=colors.detach().numpy(), grad_base=app._base_colors.grad.numpy(), grad_residual=app._residual_params.grad.numpy(),
                 grad_means=means_p.grad.numpy())
        print(f'wrote appearance_{k}_{model.lower()}.npz', tuple(colors.shape))


if __name__ == '__main__':
    main()
