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
