"""Helpers shared by the tests: scene construction, GPU runs with stage views, and error metrics."""
from __future__ import annotations

import numpy as np
import torch

import synthetic as S
from oracle import oracle as O

ACT = {'base': {'none': 0, 'exp': 1}, 'res': {'none': 0, 'tanh': 1, 'softplus': 2},
       'color': {'none': 0, 'relu': 1, 'softplus': 2, 'sigmoid': 3, 'hardsigmoid': 4, 'satexp': 5}}


def scene(model: str, n: int, degree: int, seed: int = 0, scale_shift: float = 0.0):
    geo = S.geometry(n, seed=seed)
    if scale_shift:
        geo['scales'] = geo['scales'] + scale_shift
    if model in ('sh', 'precomputed'):
        app = S.sh_appearance(n, max(degree, 1) if model == 'sh' else 3, seed=seed + 1)
    elif model == 'sv':
        app = S.sv_appearance(n, degree, seed=seed + 1)
    elif model == 'nasg':
        app = S.nasg_appearance(n, degree, seed=seed + 1)
    elif model == 'nasgabor':
        app = S.nasg_appearance(n, degree, seed=seed + 1, gabor=True)
    else:
        raise ValueError(model)
    prims = {**geo, **app}
    if model == 'precomputed':
        g = torch.Generator().manual_seed(seed + 7)
        prims = {**geo, 'precomputed_colors': torch.rand(n, 3, generator=g)}
    return prims


def to_dev(prims: dict, device) -> dict:
    return {k: v.to(device).contiguous() for k, v in prims.items()}


def settings_for(F, cam, degree: int, device, proper_aa=False, render_base=True, render_residual=True):
    return F.RasterizerSettings(cam.w2c.to(device), cam.position.to(device), cam.bg.to(device), degree, cam.width, cam.height,
                                cam.focal_x, cam.focal_y, cam.center_x, cam.center_y, cam.near_plane, cam.far_plane, proper_aa,
                                render_base, render_residual)


def view_tensor(ws: torch.Tensor, ptr: int, count: int, dtype: torch.dtype) -> torch.Tensor:
    """Slices `count` elements of `dtype` at device address `ptr` out of workspace tensor `ws`."""
    off = ptr - ws.data_ptr()
    nbytes = count * torch.empty(0, dtype=dtype).element_size()
    assert 0 <= off and off + nbytes <= ws.numel()
    return ws[off:off + nbytes].view(dtype)


def gpu_forward_stages(F, prims_dev: dict, settings, grad_image=None, densification_info=None):
    """Runs the training forward through the library and returns CPU copies of every stage buffer."""
    from FasterGSVDACudaBackend import rasterization as R, _lib
    empty = torch.empty(0, device=prims_dev['means'].device)
    get = lambda k: prims_dev.get(k, empty)
    cp = R._c_primitives(prims_dev['means'], prims_dev['scales'], prims_dev['rotations'], prims_dev['opacities'], get('precomputed_colors'),
                         get('base_colors'), get('residual_params'), get('mlp_weights'))
    st = R.ForwardState(R._rasterizer, cp, settings, prims_dev['means'].device)
    st.preprocess(cp)
    image = torch.empty((3, settings.height, settings.width), device=prims_dev['means'].device)
    st.render_train(image)
    torch.cuda.synchronize()
    f = st.frame
    v = st.views()
    n, V, I = f.n_primitives, f.n_visible, f.n_instances
    T = f.grid_w * f.grid_h
    out = {'n_visible': V, 'n_instances': I, 'image': image.cpu().numpy(), 'state': st}
    out['n_touched'] = view_tensor(st.prim_ws, v.n_touched, n, torch.int32).cpu().numpy().view(np.uint32)
    out['depth_key'] = view_tensor(st.prim_ws, v.depth_keys, n, torch.int32).cpu().numpy().view(np.uint32)
    out['sorted_idx'] = view_tensor(st.prim_ws, v.sorted_indices, V, torch.int32).cpu().numpy().view(np.uint32) if V else np.zeros(0, np.uint32)
    out['rank_of'] = view_tensor(st.prim_ws, v.rank_of, n, torch.int32).cpu().numpy().view(np.uint32)
    out['records'] = view_tensor(st.prim_ws, v.sorted_records, V * 12, torch.float32).cpu().numpy().reshape(V, 12) if V else np.zeros((0, 12), np.float32)
    out['instance_offsets'] = view_tensor(st.prim_ws, v.instance_offsets, V, torch.int32).cpu().numpy().view(np.uint32) if V else np.zeros(0, np.uint32)
    if I:
        kd = torch.int32 if f.wide_keys else torch.int16
        keys = view_tensor(st.inst_ws, v.instance_keys, I, kd).cpu().numpy()
        out['tile_keys'] = keys.view(np.uint32) if f.wide_keys else keys.view(np.uint16).astype(np.uint32)
        out['ranks'] = view_tensor(st.inst_ws, v.instance_ranks, I, torch.int32).cpu().numpy().view(np.uint32)
    else:
        out['tile_keys'] = np.zeros(0, np.uint32)
        out['ranks'] = np.zeros(0, np.uint32)
    out['ranges'] = view_tensor(st.tile_ws, v.tile_ranges, 2 * T, torch.int32).cpu().numpy().view(np.uint32).reshape(T, 2)
    ft = view_tensor(st.tile_ws, v.final_transmittance, T * 192, torch.float32).cpu().numpy().reshape(f.grid_h, f.grid_w, 12, 16)
    nc = view_tensor(st.tile_ws, v.n_contributors, T * 192, torch.int32).cpu().numpy().view(np.uint32).reshape(f.grid_h, f.grid_w, 12, 16)
    H, W = settings.height, settings.width
    out['final_T'] = ft.transpose(0, 2, 1, 3).reshape(f.grid_h * 12, f.grid_w * 16)[:H, :W]
    out['n_contrib'] = nc.transpose(0, 2, 1, 3).reshape(f.grid_h * 12, f.grid_w * 16)[:H, :W]
    out['tile_max'] = view_tensor(st.tile_ws, v.tile_max_contributors, T, torch.int32).cpu().numpy().view(np.uint32)
    out['bucket_off'] = view_tensor(st.tile_ws, v.bucket_offsets, T, torch.int32).cpu().numpy().view(np.uint32)
    return out


def rel_err(a, b) -> float:
    """||a - b|| / ||b|| over all elements (0 when both vanish)."""
    a = np.asarray(a, np.float64)
    b = np.asarray(b, np.float64)
    nb = np.linalg.norm(b)
    na = np.linalg.norm(a - b)
    return float(na / nb) if nb > 0 else float(na)


def oracle_records_in_rank_order(o: dict) -> np.ndarray:
    return o['records'][o['sorted_idx']]


def compare_forward(g, o, image_max=5e-2, flips=1e-3):
    """Every forward stage of a GPU run (gpu_forward_stages) against the oracle's C restatement. The kernels evaluate
    the projection, tile test and fragment acceptance with the reference build's fast-math arithmetic (approximate
    division, square root, exp, log and exp2; bit for bit the reference's, tests/test_gpu_reference.py), which a C
    program cannot reproduce, while the restatement uses IEEE arithmetic; the two agree within rounding, and a decision
    that sits within a rounding of its threshold (a culled primitive, a tile at the edge of a footprint, a fragment at
    alpha = 1/255) can go either way, which changes a pixel by up to the fragment's share of it. Bounds: visible and
    instance counts and tiles touched per primitive differ on at most a fraction `flips` of the primitives; for
    primitives visible on both sides the screen means agree within 1e-3 px, conics within 1e-3 of their magnitude,
    opacities within 1e-5, colours within 1e-4 relative; the depth order agrees wherever the depth keys and visibility
    do; contributor counts differ on at most a fraction `flips` of the pixels; the image within 5e-6 mean-abs, with at
    most a fraction `flips` of the pixels off by more than 1e-4 and none by more than `image_max` (a flipped fragment
    has alpha near 1/255 and moves its pixel by at most that share of a colour difference). Returns the measured
    figures."""
    n = len(o['n_touched'])
    tol = 2 + flips * n
    m = {'visible': (g['n_visible'], o['n_visible']), 'instances': (g['n_instances'], o['n_instances']),
         'touched_mismatch': int((g['n_touched'] != o['n_touched']).sum())}
    assert abs(g['n_visible'] - o['n_visible']) <= tol, m
    assert abs(g['n_instances'] - o['n_instances']) <= 10 + flips * max(o['n_instances'], 1), m
    assert m['touched_mismatch'] <= tol, m
    both = (g['n_touched'] > 0) & (o['n_touched'] > 0)
    if both.any():
        rec_g = np.zeros((n, 12), np.float32)
        rec_g[g['sorted_idx']] = g['records']
        rec_o = o['records']
        m['mean2d'] = float(np.abs(rec_g[both, 0:2] - rec_o[both, 0:2]).max())
        cg, co = rec_g[both, 4:7].astype(np.float64), rec_o[both, 4:7]
        m['conic'] = float((np.abs(cg - co).max(1) / np.maximum(np.abs(co[:, 0]), np.abs(co[:, 2]))).max())
        m['opacity'] = float(np.abs(rec_g[both, 2] - rec_o[both, 2]).max())
        colo = rec_o[both, 7:10]
        m['colour'] = float(np.abs(rec_g[both, 8:11].astype(np.float64) - colo).max() / max(1.0, np.abs(colo).max()))
        assert m['mean2d'] <= 1e-3 and m['conic'] <= 1e-3 and m['opacity'] <= 1e-5 and m['colour'] <= 1e-4, m
    if np.array_equal(g['depth_key'][both], o['depth_key'][both]) and np.array_equal(g['n_touched'] > 0, o['n_touched'] > 0):
        np.testing.assert_array_equal(g['sorted_idx'], o['sorted_idx'])
    # bucket offsets: inclusive scan of ceil(tile list length / 32) of this run's own ranges (kernels_forward.cuh:14-24)
    lengths = g['ranges'][:, 1].astype(np.int64) - g['ranges'][:, 0].astype(np.int64)
    np.testing.assert_array_equal(g['bucket_off'], np.cumsum((lengths + 31) // 32).astype(np.uint32))
    m['contrib_mismatch'] = float((g['n_contrib'] != o['n_contrib']).mean())
    d = np.abs(g['image'] - o['image'])
    m['image_mean'], m['image_max'], m['pixels_over_1e-4'] = float(d.mean()), float(d.max()), float((d.max(0) > 1e-4).mean())
    print('\n[vs oracle]', m)
    assert m['contrib_mismatch'] <= flips and m['pixels_over_1e-4'] <= flips, m
    assert m['image_mean'] <= 5e-6 and m['image_max'] <= image_max, m
    return m


def assert_matches_reference(g, r, img_ref, exact_image=False, image_max=2e-6):
    """This library's forward stages (gpu_forward_stages) against the reference's own kernels run on the same inputs
    (oracle/reference.py buffers()): visible and instance counts, tiles touched per primitive, screen means, conics and
    opacities bit for bit; every tile's list of primitives bit for bit once the reference's order of equal-depth
    primitives is made canonical (its compaction orders depth ties by atomic scheduling; this library by primitive
    index); contributor counts and final transmittance bit for bit outside the tiles where such a tie reordered the
    list; the image bit for bit there (`exact_image`, identical colours) or within `image_max` (colours evaluated in
    another order). Returns the number of tiles whose raw lists differ only in the order of depth ties, and the [H, W]
    mask of the pixels outside them."""
    n = len(g['n_touched'])
    assert g['n_visible'] == r['n_visible'] and g['n_instances'] == r['n_instances'], \
        ((g['n_visible'], r['n_visible']), (g['n_instances'], r['n_instances']))
    np.testing.assert_array_equal(g['n_touched'], r['n_touched'], err_msg='tiles touched per primitive')
    vis = g['n_touched'] > 0
    rec = np.zeros((n, 12), np.float32)
    rec[g['sorted_idx']] = g['records']
    np.testing.assert_array_equal(rec[vis, 0:2], r['mean2d'][vis], err_msg='screen means')
    np.testing.assert_array_equal(rec[vis, 4:7], r['conic_opacity'][vis, 0:3], err_msg='conics')
    np.testing.assert_array_equal(rec[vis, 2], r['conic_opacity'][vis, 3], err_msg='opacities')
    np.testing.assert_array_equal(g['ranges'], r['ranges'], err_msg='tile ranges')
    mine = g['sorted_idx'][g['ranks']] if g['n_instances'] else np.zeros(0, np.uint32)
    theirs = r['instance_prims']
    key = g['depth_key'].astype(np.uint64)
    tie_tiles = []
    for t, (a, b) in enumerate(g['ranges']):
        if a == b or np.array_equal(mine[a:b], theirs[a:b]):
            continue
        lst = theirs[a:b]
        canon = lst[np.lexsort((lst, key[lst]))]
        np.testing.assert_array_equal(mine[a:b], canon, err_msg=f'tile {t}')
        tie_tiles.append(t)
    H, W = g['image'].shape[1:]
    gw = (W + 15) // 16
    mask = np.ones((H, W), bool)
    for t in tie_tiles:
        ty, tx = divmod(t, gw)
        mask[ty * 12:(ty + 1) * 12, tx * 16:(tx + 1) * 16] = False
    np.testing.assert_array_equal(g['n_contrib'][mask], r['n_contrib'][mask], err_msg='contributor counts')
    np.testing.assert_array_equal(g['final_T'][mask], r['final_T'][mask], err_msg='final transmittance')
    ref = img_ref.cpu().numpy() if hasattr(img_ref, 'cpu') else img_ref
    if exact_image:
        np.testing.assert_array_equal(g['image'][:, mask], ref[:, mask], err_msg='image')
    else:
        assert np.abs(g['image'][:, mask] - ref[:, mask]).max() <= image_max
    return len(tie_tiles), mask


def gpu_colors_by_primitive(g: dict, n: int) -> np.ndarray:
    """The blended colors of a GPU run (record fields 8-10, depth-rank order) scattered back to primitive order
    [n, 3]; zero for culled primitives. Fed to the oracle as precomputed colors, they make its blend see the GPU's
    inputs exactly."""
    out = np.zeros((n, 3), np.float32)
    out[g['sorted_idx']] = g['records'][:, 8:11]
    return out
