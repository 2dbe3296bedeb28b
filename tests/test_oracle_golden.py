"""Pins the oracle's appearance math to the reference's own PyTorch modules (Appearance/SH.py, SV.py, NASG.py,
NASGabor.py run on the CPU by tests/golden/make_golden.py): colors and gradients for base, residual parameters and
the view-direction path of the means, across activation triples."""
import glob
from pathlib import Path

import numpy as np
import pytest

from oracle import oracle as O
from fgs_testutil import ACT

FILES = sorted(glob.glob(str(Path(__file__).resolve().parent / 'golden' / 'appearance_*.npz')))


@pytest.mark.parametrize('path', FILES, ids=[Path(f).stem for f in FILES])
@pytest.mark.parametrize('double', [True, False])
def test_appearance_matches_reference_modules(path, double):
    z = np.load(path)
    a = O.make_appearance(str(z['model']), int(z['degree']), ACT['base'][str(z['base_act'])], ACT['res'][str(z['residual_act'])],
                          ACT['color'][str(z['color_act'])])
    o = O.appearance(a, z['means'], z['cam'], z['base'], z['residual'], int(z['degree']), z['upstream'], double=double)
    tol = 1e-7 if double else 1e-5
    for key in ('colors', 'grad_base', 'grad_residual', 'grad_means'):
        ref = z[key]
        got = o[key].reshape(ref.shape)
        assert np.abs(got - ref).max() <= tol * max(1.0, np.abs(ref).max()), key


def test_golden_files_present():
    assert len(FILES) == 8


@pytest.mark.parametrize('path', [f for f in FILES if '_sh' in Path(f).stem], ids=lambda f: Path(f).stem)
def test_torch_restatement_matches_reference_modules(path):
    """The PyTorch restatement of the reference's unfused SH path (the CPU baseline of configuration c0) reproduces
    the reference modules' colours and autograd gradients."""
    import torch
    from oracle import appearance_torch as AT
    z = np.load(path)
    t = {k: torch.tensor(z[k], dtype=torch.float64, requires_grad=k in ('base', 'residual', 'means')) for k in ('base', 'residual', 'means')}
    col = AT.sh_colors(t['means'], torch.tensor(z['cam'], dtype=torch.float64), t['base'], t['residual'], int(z['degree']), str(z['base_act']),
                       str(z['residual_act']), str(z['color_act']))
    col.backward(torch.tensor(z['upstream'], dtype=torch.float64))
    for got, key in ((col.detach(), 'colors'), (t['base'].grad, 'grad_base'), (t['residual'].grad, 'grad_residual'), (t['means'].grad, 'grad_means')):
        ref = z[key]
        assert np.abs(got.numpy().reshape(ref.shape) - ref).max() <= 1e-9 * max(1.0, np.abs(ref).max()), key
