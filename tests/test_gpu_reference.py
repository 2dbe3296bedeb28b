"""GPU parity against the reference's own rasterizer: its unmodified forward.cu / backward.cu / inference.cu host code
and AOT kernels, and its NVRTC preprocess kernels, compiled from the reference checkout by oracle/ref_build.py into
oracle/_ref (test infrastructure; see oracle/reference.py). Both run on the same device tensors.

Asserted (fgs_testutil.assert_matches_reference): counts, tiles touched per primitive, screen means, conics and
opacities bit for bit; every tile's primitive list bit for bit once the reference's order of equal-depth primitives
(scheduling-dependent in its compaction) is made canonical; contributor counts and final transmittance bit for bit
outside tiles that such a tie reordered; images bit for bit for precomputed colours and within 2e-6 otherwise (the
appearance is evaluated in another operation order); every parameter gradient within 1e-4 relative L2 of the
reference's. The measured figures are printed. Skipped when the harness is not built (no reference checkout was
available where the repository was built)."""
import numpy as np
import pytest
import torch

import synthetic as S
from oracle import reference as REF
from fgs_testutil import scene, to_dev, settings_for, gpu_forward_stages, rel_err, assert_matches_reference

pytestmark = pytest.mark.gpu

CASES = [
    # model, degree, base, residual, color
    ('precomputed', 0, 'none', 'none', 'relu'),
    ('sh', 3, 'none', 'none', 'relu'),
    ('sh', 1, 'none', 'none', 'none'),
    ('sh', 2, 'exp', 'tanh', 'satexp'),
    ('sv', 8, 'none', 'none', 'relu'),
    ('nasg', 8, 'none', 'tanh', 'relu'),
    ('nasgabor', 4, 'none', 'tanh', 'sigmoid'),
]


def require_reference():
    if not REF.available():
        pytest.skip('reference harness not built (oracle/ref_build.py needs the reference checkout)')


def forward_and_gradients(F, ref, dev, settings, grad_image, exact_image, label):
    """Forward stages against the reference, then both backward passes for the same upstream gradient; returns the
    measured differences."""
    g = gpu_forward_stages(F, dev, settings)
    img_ref = ref.forward(dev, settings)
    r = ref.buffers()
    ties, _ = assert_matches_reference(g, r, img_ref, exact_image=exact_image)
    d = np.abs(g['image'] - img_ref.cpu().numpy())
    m = {'label': label, 'n_visible': g['n_visible'], 'n_instances': g['n_instances'], 'tie_tiles': ties,
         'image_max_abs': float(d.max()), 'image_mean_abs': float(d.mean())}
    del g
    gr = ref.backward(dev, img_ref, grad_image)
    leaves = {k: v.clone().requires_grad_(True) for k, v in dev.items()}
    img = F.diff_rasterize(leaves['means'], leaves['scales'], leaves['rotations'], leaves['opacities'], torch.empty(0, device=dev['means'].device),
                           settings, precomputed_colors=leaves.get('precomputed_colors'), base_colors=leaves.get('base_colors'),
                           residual_params=leaves.get('residual_params'))
    img.backward(grad_image)
    for k, t in leaves.items():
        if gr.get(k) is not None:
            m[f'grad_{k}_rel'] = rel_err(t.grad.cpu().numpy().reshape(-1), gr[k].cpu().numpy().reshape(-1))
    print('\n[reference]', m)
    for k, v in m.items():
        if k.startswith('grad_'):
            assert v <= 1e-4, (k, v)
    return m


@pytest.mark.parametrize('case', CASES, ids=[f'{c[0]}{c[1]}-{c[2]}-{c[3]}-{c[4]}' for c in CASES])
def test_against_reference_kernels(cuda, case):
    require_reference()
    import FasterGSVDACudaBackend as F
    model, degree, base, res, col = case
    if model == 'precomputed':
        F.initialize_appearance('sh', 3, 'none', 'none', 'relu', True)
    else:
        F.initialize_appearance(model, degree, base, res, col, True)
    ref = REF.Reference(REF.tag_of(model, degree, base, res, col))
    n, W, H = 20000, 256, 192
    settings = settings_for(F, S.ring_cameras(3, W, H)[1], degree, cuda)
    dev = to_dev(scene(model, n, degree, seed=0, scale_shift=1.0), cuda)
    grad_image = (torch.randn(3, H, W, generator=torch.Generator().manual_seed(2)) * 0.01).to(cuda)
    forward_and_gradients(F, ref, dev, settings, grad_image, model == 'precomputed', f'{model}{degree}')
    ref.close()


def test_c1_full_size_against_reference(cuda):
    """Configuration c1 (SH-3, 1,000,000 Gaussians, 1280x720): forward stages, image and gradients."""
    require_reference()
    import FasterGSVDACudaBackend as F
    F.initialize_appearance('sh', 3, 'none', 'none', 'relu', True)
    ref = REF.Reference('sh3_none_none_relu')
    n, W, H = 1_000_000, 1280, 720
    settings = settings_for(F, S.ring_cameras(8, W, H)[0], 3, cuda)
    dev = to_dev({**S.geometry(n), **S.sh_appearance(n, 3)}, cuda)
    grad_image = (torch.randn(3, H, W, generator=torch.Generator().manual_seed(2)) * 0.01).to(cuda)
    m = forward_and_gradients(F, ref, dev, settings, grad_image, False, 'c1')
    assert m['n_visible'] > 400_000 and m['n_instances'] > 1_000_000
    ref.close()


@pytest.mark.parametrize('to_chw,clamp', [(False, True), (True, False)])
def test_inference_against_reference(cuda, to_chw, clamp):
    """The inference render (clamp, HWC / CHW) against the reference's inference path, precomputed colours: bit for bit
    outside the tiles whose lists a depth tie reordered (found from the training forward of the same view)."""
    require_reference()
    import FasterGSVDACudaBackend as F
    F.initialize_appearance('sh', 3, 'none', 'none', 'relu', True)
    ref = REF.Reference('precomputed')
    n, W, H = 30000, 250, 130
    settings = settings_for(F, S.ring_cameras(4, W, H)[3], 3, cuda)
    dev = to_dev(scene('precomputed', n, 0, seed=9, scale_shift=1.0), cuda)
    g = gpu_forward_stages(F, dev, settings)
    img_train_ref = ref.forward(dev, settings)
    _, mask = assert_matches_reference(g, ref.buffers(), img_train_ref, exact_image=True)
    img = F.rasterize(dev['means'], dev['scales'], dev['rotations'], dev['opacities'], settings, to_chw, clamp,
                      precomputed_colors=dev['precomputed_colors']).cpu().numpy()
    img_ref = ref.inference(dev, settings, to_chw, clamp).cpu().numpy()
    if not to_chw:
        img, img_ref = img.transpose(2, 0, 1), img_ref.transpose(2, 0, 1)
    np.testing.assert_array_equal(img[:, mask], img_ref[:, mask])
    ref.close()
