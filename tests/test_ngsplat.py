"""Viewer export (.ngsplat): the library's writer reproduces, byte for byte, the files the reference's own exporter
wrote for the same parameters (tests/golden/ngsplat_*.npz, made by tests/golden/make_ngsplat_golden.py): every
appearance model, trimmed SH degrees and NASG lobes, baked and full Neural layouts, gated and inactive Neural
direction degrees, base colours as MLP inputs, opacity culling, a zero scale and degenerate / negative-w rotations.
The reader parses every file completely."""
import json
from pathlib import Path

import numpy as np
import pytest

import ngsplat

GOLDEN = Path(__file__).resolve().parent / 'golden'
CASES = sorted(p.stem[len('ngsplat_'):] for p in GOLDEN.glob('ngsplat_*.npz'))


def _appearance(meta: dict) -> ngsplat.ViewerAppearance:
    app = meta['appearance']
    model = meta['model']
    kw = dict(model=model, base_activation=app['BASE_ACTIVATION'].lower(), residual_activation=app['RESIDUAL_ACTIVATION'].lower(),
              color_activation=app['COLOR_ACTIVATION'].lower(), active_degree=meta['active_degree'])
    if model == 'neural':
        nr = app['NEURAL']
        kw.update(feature_frequencies=nr['FEATURE_N_FREQUENCIES'], sh_degrees=tuple(nr['SH_DEGREES']), n_neurons=nr['N_NEURONS'],
                  n_hidden_layers=nr['N_HIDDEN_LAYERS'], base_input=nr['BASE_INPUT'])
    return ngsplat.ViewerAppearance(**kw)


def test_golden_cases_present():
    assert len(CASES) >= 9
    assert {'sh', 'sv', 'nasg', 'nasgabor', 'neural'} <= {json.loads(str(np.load(GOLDEN / f'ngsplat_{c}.npz')['meta']))['model'] for c in CASES}


@pytest.mark.parametrize('case', CASES)
def test_export_matches_reference_bytes(case, tmp_path):
    z = np.load(GOLDEN / f'ngsplat_{case}.npz')
    meta = json.loads(str(z['meta']))
    out = tmp_path / 'scene.ngsplat'
    summary = ngsplat.export_ngsplat(out, z['means'], z['scales'], z['rotations'], z['opacities'], z['base_colors'], z['residual_params'],
                                     _appearance(meta), mlp_weights=z['mlp_weights'] if 'mlp_weights' in z.files else None)
    got = np.frombuffer(out.read_bytes(), np.uint8)
    ref = z['ngsplat']
    assert got.size == ref.size, (got.size, ref.size)
    f = ngsplat.read_ngsplat(out)
    if not np.array_equal(got, ref):
        # The baked Neural layer-0 share is a float32 matrix product (BLAS); on another CPU its summation order may
        # move one fp16 rounding. Everything else must still be identical, those values within one fp16 unit.
        r = ngsplat.read_ngsplat_bytes(ref.tobytes())
        assert f['model'] == 'neural' and f['flags'] & 4, 'bytes differ outside the baked Neural payload'
        for k in f:
            if k != 'textures':
                np.testing.assert_array_equal(np.asarray(f[k]), np.asarray(r[k]), err_msg=k)
        for a, b in zip(f['textures'], r['textures']):
            ha, hb = (t.view(np.uint16).astype(np.int32) for t in (a, b))
            assert np.abs(ha - hb).max() <= 1
    assert f['model'] == meta['model']
    assert f['n'] == summary['splats'] == z['means'].shape[0] - summary['culled']
    assert summary['culled'] >= 6  # the six planted ones and any drawn below 1/255
    assert f['geometry'].shape == (f['tex_width'] * f['tex_height'], 4)
    # the geometry texels decode back to the kept Gaussians: fp16 positions, opacity codes
    keep = 1.0 / (1.0 + np.exp(-z['opacities'].reshape(-1).astype(np.float32))) >= 1.0 / 255.0
    mu = z['means'][keep]
    g = f['geometry'][:f['n']]
    x = (g[:, 1] & 0xFFFF).astype(np.uint16).view(np.float16).astype(np.float32)
    zc = (g[:, 2] & 0xFFFF).astype(np.uint16).view(np.float16).astype(np.float32)
    np.testing.assert_allclose(x, mu[:, 0], rtol=1e-3, atol=1e-3)
    np.testing.assert_allclose(zc, mu[:, 2], rtol=1e-3, atol=1e-3)
    assert np.all(g[:, 0] >> 24 >= 1)


def test_rejects_unrepresentable_neural_configs(tmp_path):
    z = np.load(GOLDEN / 'ngsplat_neural_baked.npz')
    a = ngsplat.ViewerAppearance('neural', residual_activation='softplus', active_degree=0)
    with pytest.raises(ValueError, match='softplus'):
        ngsplat.export_ngsplat(tmp_path / 'x.ngsplat', z['means'], z['scales'], z['rotations'], z['opacities'], z['base_colors'],
                               z['residual_params'], a, mlp_weights=z['mlp_weights'])
    with pytest.raises(ValueError, match='multiple of 16'):
        ngsplat.export_ngsplat(tmp_path / 'x.ngsplat', z['means'], z['scales'], z['rotations'], z['opacities'], z['base_colors'],
                               z['residual_params'], ngsplat.ViewerAppearance('neural', residual_activation='tanh'),
                               mlp_weights=z['mlp_weights'][:-16])


def test_header_options_and_test_cameras(tmp_path):
    """Proper-antialiasing flag, orbit-hint overrides and baked test cameras land in the header; the splat and
    residual payloads stay those of the reference file for the same parameters."""
    z = np.load(GOLDEN / 'ngsplat_sv3.npz')
    meta = json.loads(str(z['meta']))
    cams = np.arange(2 * 18, dtype=np.float32).reshape(2, 18)
    out = tmp_path / 'opts.ngsplat'
    ngsplat.export_ngsplat(out, z['means'], z['scales'], z['rotations'], z['opacities'], z['base_colors'], z['residual_params'],
                           _appearance(meta), proper_antialiasing=True, center=(1.0, 2.0, 3.0), up=(0.0, 0.0, 2.0), distance=7.5,
                           test_cameras=cams)
    f = ngsplat.read_ngsplat(out)
    r = ngsplat.read_ngsplat_bytes(z['ngsplat'].tobytes())
    assert f['flags'] == r['flags'] | 1
    assert f['center'] == (1.0, 2.0, 3.0) and f['up'] == (0.0, 0.0, 1.0) and f['distance'] == 7.5
    np.testing.assert_array_equal(f['test_cameras'], cams)
    np.testing.assert_array_equal(f['geometry'], r['geometry'])
    for a, b in zip(f['textures'], r['textures']):
        np.testing.assert_array_equal(a, b)
