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


def compare_forward(g, o, exact_image):
    """Every forward stage of a GPU run (gpu_forward_stages) against an oracle run: integer stages, geometry fields
    and contributor counts bit for bit; colors, image and transmittance bit for bit when `exact_image`, else within
    1e-5 relative (colors), 1e-4 max abs (image) and 1e-6 (transmittance)."""
    assert g['n_visible'] == o['n_visible']
    assert g['n_instances'] == o['n_instances']
    np.testing.assert_array_equal(g['n_touched'], o['n_touched'])
    vis = o['n_touched'] > 0
    np.testing.assert_array_equal(g['depth_key'][vis], o['depth_key'][vis])
    np.testing.assert_array_equal(g['sorted_idx'], o['sorted_idx'])
    np.testing.assert_array_equal(g['instance_offsets'], o['instance_offsets'])
    np.testing.assert_array_equal(g['tile_keys'], o['tile_keys'])
    np.testing.assert_array_equal(g['ranks'], o['ranks'])
    np.testing.assert_array_equal(g['ranges'], o['ranges'])
    # bucket offsets: inclusive scan of ceil(tile list length / 32) (kernels_forward.cuh:14-24, forward.cu:204-219)
    lengths = o['ranges'][:, 1].astype(np.int64) - o['ranges'][:, 0].astype(np.int64)
    np.testing.assert_array_equal(g['bucket_off'], np.cumsum((lengths + 31) // 32).astype(np.uint32))
    rec_o = oracle_records_in_rank_order(o)
    rec_g = g['records']
    # geometry fields bit-exact: mean2d, opacity, power threshold, conic, bounds
    for gi, oi in ((0, 0), (1, 1), (2, 2), (3, 3), (4, 4), (5, 5), (6, 6)):
        np.testing.assert_array_equal(rec_g[:, gi], rec_o[:, oi].astype(np.float32))
    bx = rec_g[:, 7].view(np.uint32)
    by = rec_g[:, 11].view(np.uint32)
    np.testing.assert_array_equal(bx & 0xffff, rec_o[:, 10].astype(np.uint32))
    np.testing.assert_array_equal(bx >> 16, rec_o[:, 11].astype(np.uint32))
    np.testing.assert_array_equal(by & 0xffff, rec_o[:, 12].astype(np.uint32))
    np.testing.assert_array_equal(by >> 16, rec_o[:, 13].astype(np.uint32))
    np.testing.assert_array_equal(g['n_contrib'], o['n_contrib'])
    colors_g = rec_g[:, 8:11]
    colors_o = rec_o[:, 7:10].astype(np.float32)
    if exact_image:
        np.testing.assert_array_equal(colors_g, colors_o)
        np.testing.assert_array_equal(g['image'], o['image'])
        np.testing.assert_array_equal(g['final_T'], o['final_T'])
    else:
        assert np.abs(colors_g - colors_o).max() <= 1e-5 * max(1.0, np.abs(colors_o).max())
        assert np.abs(g['image'] - o['image']).max() <= 1e-4
        assert np.abs(g['final_T'] - o['final_T']).max() <= 1e-6


def gpu_colors_by_primitive(g: dict, n: int) -> np.ndarray:
    """The blended colors of a GPU run (record fields 8-10, depth-rank order) scattered back to primitive order
    [n, 3]; zero for culled primitives. Fed to the oracle as precomputed colors, they make its blend see the GPU's
    inputs exactly."""
    out = np.zeros((n, 3), np.float32)
    out[g['sorted_idx']] = g['records'][:, 8:11]
    return out
