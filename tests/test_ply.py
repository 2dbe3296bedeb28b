"""PLY export (efficient-gaussian-appearance_b200/ply.py) in the reference's layout (Model.py:502-531,
Appearance/SH.py:59-70, Appearance/Base.py:230-236): a write / read round trip is exact, SH coefficients are stored
as f_dc = base / C0 and channel-major f_rest, other appearance setups bake the activated base colour into f_dc, the
quaternion is normalised and opacity and scales stay pre-activation."""
import numpy as np
import torch

import ply as P


def _scene(n=257):
    g = torch.Generator().manual_seed(0)
    return dict(means=torch.randn(n, 3, generator=g), scales=torch.randn(n, 3, generator=g) - 4.0, rotations=torch.randn(n, 4, generator=g),
                opacities=torch.randn(n, 1, generator=g), base=torch.randn(n, 3, generator=g), rest=torch.randn(n, 15, 3, generator=g))


def test_sh_layout_and_round_trip(tmp_path):
    s = _scene()
    cols, names = P.appearance_columns('sh', s['base'], s['rest'])
    assert names[:3] == ['f_dc_0', 'f_dc_1', 'f_dc_2'] and names[3:] == [f'f_rest_{i}' for i in range(45)]
    # f_rest_i: channel c, coefficient j at i = c * 15 + j
    np.testing.assert_allclose(cols[:, 3 + 1 * 15 + 4], s['rest'][:, 4, 1].numpy(), rtol=0, atol=0)
    np.testing.assert_allclose(cols[:, 0], (s['base'][:, 0] / P.SH_C0).numpy(), rtol=1e-7)
    v = P.scene_vertices(s['means'], s['scales'], s['rotations'], s['opacities'], cols, names)
    assert list(v.dtype.names) == ['x', 'y', 'z'] + names + ['opacity', 'scale_0', 'scale_1', 'scale_2', 'rot_0', 'rot_1', 'rot_2', 'rot_3']
    q = np.stack([v[f'rot_{i}'] for i in range(4)], 1)
    np.testing.assert_allclose(np.linalg.norm(q, axis=1), 1.0, rtol=1e-6)
    np.testing.assert_array_equal(v['opacity'], s['opacities'][:, 0].numpy())
    np.testing.assert_array_equal(v['scale_2'], s['scales'][:, 2].numpy())
    path = tmp_path / 'scene.ply'
    P.write_ply(path, v, ['SplatRenderMode: default', 'Generated with the B200 backend'])
    back, comments = P.read_ply(path)
    assert comments == ['SplatRenderMode: default', 'Generated with the B200 backend']
    assert back.dtype == v.dtype
    assert back.tobytes() == v.tobytes()


def test_other_setups_bake_the_base_colour():
    s = _scene()
    cols, names = P.appearance_columns('nasg', s['base'], None, base_act='exp', color_act='sigmoid')
    assert names == ['f_dc_0', 'f_dc_1', 'f_dc_2']
    rgb = torch.sigmoid(4.0 * torch.exp(3.0 * s['base']))
    np.testing.assert_allclose(cols, ((rgb - 0.5) / P.SH_C0).numpy(), rtol=1e-6)
    # a viewer's diffuse colour max(0.5 + C0 f_dc, 0) is the activated base colour
    np.testing.assert_allclose(np.maximum(0.5 + P.SH_C0 * cols, 0.0), rgb.numpy(), rtol=1e-5, atol=1e-6)
