"""The oracle's OpenMP loops (oracle/fgs_oracle.c, orc_set_threads): with eight threads the whole restated pipeline
gives the same image, tile lists and ranges bit for bit, and gradients equal to rounding (the per-thread sums of the
blend backward and of the MLP weight gradient are combined in a different order)."""
import numpy as np
import torch

import synthetic as S
from oracle import oracle as O


def test_threads_reproduce_the_single_thread_pipeline():
    feat, nf, nn, nh = 8, 1, 16, 2
    n_in = feat * 2 * nf + 16
    pad = (n_in + 15) // 16 * 16
    neural = dict(feature_dim=feat, base_input=0, n_freq=nf, sh_mask=15, n_input=n_in, n_input_pad=pad, n_neurons=nn, n_hidden=nh,
                  hidden_act=1)
    n, W, H = 3000, 128, 96
    geo = S.geometry(n)
    geo['scales'] = geo['scales'] + 2.0
    prims = {k: v.numpy() for k, v in {**geo, **S.neural_appearance(n, feature_dim=feat, layer_shapes=S.mlp_layer_shapes(pad, nn, nh))}.items()}
    cam = S.look_at(torch.tensor([0.0, 0.0, 12.0]), W, H)
    v = O.make_view(cam, 3)
    a = O.make_appearance('neural', 0, 0, 1, 1, True, neural=neural)
    G = torch.randn(3, H, W, generator=torch.Generator().manual_seed(2)).numpy()
    out = {}
    try:
        for th in (1, 8):
            O.set_threads(th)
            out[th] = O.run(a, v, prims, grad_image=G)
    finally:
        O.set_threads(1)
    for k in ('image', 'final_T', 'n_contrib', 'tile_keys', 'ranks', 'ranges', 'sorted_idx'):
        np.testing.assert_array_equal(out[1][k], out[8][k])
    for k, x in out[1]['grads'].items():
        if x is not None:
            np.testing.assert_allclose(out[8]['grads'][k], x, rtol=1e-10, atol=1e-14 * max(np.abs(x).max(), 1e-30))
