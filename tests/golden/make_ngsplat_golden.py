"""Generates golden .ngsplat files with the reference's own viewer exporter (viewer/export_ngsplat.py).

For each case below it writes a small synthetic checkpoint (raw Gaussian parameters, appearance parameters, the
tiny-cuda-nn style MLP parameter vector for Neural, and the MODEL.APPEARANCE mapping plus the appearance schedule
position the exporter looks up), runs the unmodified exporter on it as a bare checkpoint (no test cameras, no PPISP,
so no dataset or NeRFICG framework is needed) and stores the inputs together with the exported bytes in
tests/golden/ngsplat_<case>.npz. The tests compare this library's writer (ngsplat.py) with those bytes and never read
the reference at run time.

Run: python tests/golden/make_ngsplat_golden.py <reference checkout>   (or set $FGS_REFERENCE)
"""
import json
import os
import subprocess
import sys
import tempfile
from pathlib import Path

import numpy as np
import torch

REF = Path(sys.argv[1] if len(sys.argv) > 1 else os.environ.get('FGS_REFERENCE', ''))
if not str(REF) or not (REF / 'Appearance').is_dir():
    raise SystemExit('pass the reference checkout (the directory holding Appearance/) as the first argument or in $FGS_REFERENCE')
OUT = Path(__file__).resolve().parent
N = 300

# name: (TYPE, appearance mapping, active_degree or None, residual shape per Gaussian, neural dims or None)
CASES = {
    'sh3': ('sh', {'BASE_ACTIVATION': 'none', 'RESIDUAL_ACTIVATION': 'none', 'COLOR_ACTIVATION': 'relu', 'SH': {'SH_DEGREE': 3}},
            None, (15, 3), None),
    'sh3_trim2': ('sh', {'BASE_ACTIVATION': 'exp', 'RESIDUAL_ACTIVATION': 'tanh', 'COLOR_ACTIVATION': 'sigmoid', 'SH': {'SH_DEGREE': 3}},
                  2, (15, 3), None),
    'sv3': ('sv', {'BASE_ACTIVATION': 'none', 'RESIDUAL_ACTIVATION': 'tanh', 'COLOR_ACTIVATION': 'softplus', 'SV': {'N_SITES': 3}},
            None, (3, 7), None),
    'nasg2_trim1': ('nasg', {'BASE_ACTIVATION': 'none', 'RESIDUAL_ACTIVATION': 'none', 'COLOR_ACTIVATION': 'hardsigmoid',
                             'NASG': {'N_LOBES': 2}}, 1, (2, 8), None),
    'nasgabor2': ('nasgabor', {'BASE_ACTIVATION': 'none', 'RESIDUAL_ACTIVATION': 'softplus', 'COLOR_ACTIVATION': 'satexp',
                               'NASGABOR': {'N_LOBES': 2}}, None, (2, 9), None),
    # Neural: (feature dims, frequencies, SH degrees, neurons, hidden layers, base input)
    'neural_baked': ('neural', {'BASE_ACTIVATION': 'none', 'RESIDUAL_ACTIVATION': 'tanh', 'COLOR_ACTIVATION': 'relu'},
                     None, (8,), (8, 1, [0, 1, 2, 3], 16, 2, False)),
    'neural_raw_nodeg0_gated': ('neural', {'BASE_ACTIVATION': 'none', 'RESIDUAL_ACTIVATION': 'softplus', 'COLOR_ACTIVATION': 'none'},
                                2, (17,), (17, 0, [1, 2, 3], 16, 1, False)),
    'neural_full_inactive': ('neural', {'BASE_ACTIVATION': 'exp', 'RESIDUAL_ACTIVATION': 'tanh', 'COLOR_ACTIVATION': 'relu'},
                             0, (8,), (8, 1, [0, 1, 2, 3], 32, 2, False)),
    'neural_base_input': ('neural', {'BASE_ACTIVATION': 'none', 'RESIDUAL_ACTIVATION': 'tanh', 'COLOR_ACTIVATION': 'softplus'},
                          None, (5,), (5, 1, [0, 1, 2, 3], 16, 2, True)),
}


def scene(seed: int, residual_shape: tuple) -> dict:
    g = torch.Generator().manual_seed(seed)
    means = torch.randn(N, 3, generator=g) * 2.0
    scales = torch.randn(N, 3, generator=g) - 3.0
    scales[0, 1] = float('-inf')  # an exactly zero scale (sentinel code 0)
    rotations = torch.randn(N, 4, generator=g)
    rotations[1] = torch.tensor([1.0, 0.0, 0.0, 0.0])  # identity: degenerate rotation axis
    rotations[2, 0] = -abs(float(rotations[2, 0]))  # w < 0: the exporter flips the sign
    opacities = torch.randn(N, 1, generator=g) * 2.0
    opacities[3:9] = -7.0  # below alpha 1/255: culled
    base = torch.randn(N, 3, generator=g) * 0.5
    residual = torch.randn(N, *residual_shape, generator=g) * 0.3
    return dict(means=means, scales=scales, rotations=rotations, opacities=opacities, base_colors=base, residual_params=residual)


def mlp_params(seed: int, n_in: int, neurons: int, hidden: int) -> torch.Tensor:
    g = torch.Generator().manual_seed(seed)
    n = n_in * neurons + (hidden - 1) * neurons * neurons + 16 * neurons
    return (torch.rand(n, generator=g) * 2.0 - 1.0) * 0.4


def main() -> None:
    exporter = REF / 'viewer' / 'export_ngsplat.py'
    for k, (name, (model, appearance, active, rshape, neural)) in enumerate(CASES.items()):
        params = scene(100 + k, rshape)
        app = {'TYPE': model.upper() if model != 'nasgabor' else 'NASGabor', **appearance}
        mlp = None
        if neural is not None:
            feat, nfreq, degrees, neurons, hidden, base_input = neural
            raw = feat + (3 if base_input else 0)
            n_in = raw * (2 * nfreq if nfreq else 1) + sum(2 * d + 1 for d in degrees)
            app['NEURAL'] = {'FEATURE_DIM': raw, 'FEATURE_N_FREQUENCIES': nfreq, 'SH_DEGREES': degrees, 'N_NEURONS': neurons,
                             'N_HIDDEN_LAYERS': hidden, 'HIDDEN_ACTIVATION': 'relu', 'BASE_INPUT': base_input}
            mlp = mlp_params(200 + k, n_in, neurons, hidden)
        ckpt = {'model': {'_means': params['means'], '_scales': params['scales'], '_rotations': params['rotations'],
                          '_opacities': params['opacities'],
                          'appearance': {'_base_colors': params['base_colors'], '_residual_params': params['residual_params']}},
                'config': {'MODEL': {'APPEARANCE': app}}}
        if mlp is not None:
            ckpt['model']['residual_mlp'] = {'params': mlp}
        if active is not None:
            ckpt['schedule'] = {'active_degree': active}
        with tempfile.TemporaryDirectory() as tmp:
            path = Path(tmp) / 'ckpt.pt'
            torch.save(ckpt, path)
            out = Path(tmp) / 'scene.ngsplat'
            res = subprocess.run([sys.executable, str(exporter), str(path), '--out', str(out), '--no-test-cameras', '--no-ppisp'],
                                 capture_output=True, text=True)
            if res.returncode != 0:
                raise RuntimeError(f'{name}: exporter failed\n{res.stdout}\n{res.stderr}')
            data = np.frombuffer(out.read_bytes(), dtype=np.uint8)
        arrays = {key: value.numpy() for key, value in params.items()}
        if mlp is not None:
            arrays['mlp_weights'] = mlp.numpy()
        meta = {'model': model, 'appearance': app, 'active_degree': active}
        np.savez_compressed(OUT / f'ngsplat_{name}.npz', ngsplat=data, meta=np.array(json.dumps(meta)), **arrays)
        print(f'{name}: {data.size} bytes')


if __name__ == '__main__':
    main()
