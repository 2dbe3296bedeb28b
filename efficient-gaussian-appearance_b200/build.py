"""Builds libfgs_b200.so (all CUDA sources of csrc/) for sm_100a with nvcc, in parallel, in-tree.

Usage: python build.py [--force]. The shared library lands in FasterGSVDACudaBackend/lib/ so that it
travels with the source tree; objects go to _build/ next to this file.
"""
import concurrent.futures
import hashlib
import os
import subprocess
import sys
from pathlib import Path

HERE = Path(__file__).resolve().parent
CSRC = HERE / 'csrc'
BUILD = HERE / '_build'
LIB = HERE / 'FasterGSVDACudaBackend' / 'lib' / 'libfgs_b200.so'
NVCC = os.environ.get('NVCC', '/usr/local/cuda/bin/nvcc')
ARCH = ['-gencode', 'arch=compute_100a,code=sm_100a']
# Default for the remaining sources (sort, adam, densification, the C ABI): -fmad=false, no implicit contraction of
# a*b+c, with nvcc's IEEE division, square root and denormals.
FLAGS = ['-O3', '-std=c++17', '-lineinfo', '-fmad=false', '-Xcompiler', '-fPIC', '--expt-relaxed-constexpr',
         '-Xptxas', '-warn-spills']
# Sources whose outputs are checked against the CPU restatement within a tolerance rather than bit for bit (the fp16
# tensor-core MLP of the neural appearance, whose backward also carries the geometry chain rule; the photometric loss,
# checked against its fp32 PyTorch definition): contraction allowed. Their deterministic parts (the frequency encoding,
# the view direction, the SH band values) are written with explicit single-rounding operations.
CONTRACTED = {'neural.cu', 'neural_tc.cu', 'loss.cu'}
# Sources that evaluate the rasterizer's forward decisions (projection, culling, tile bounds and overlap, fragment
# acceptance, transmittance) and must compute them exactly as the reference's own build does: its kernels are
# compiled with -use_fast_math (FasterGSVDACudaBackend/setup.py:125-129, and tiny-cuda-nn's runtime compiler with
# fast math for the preprocess), so these are too, with the reference's expressions.
FAST_MATH = {'preprocess.cu', 'binning.cu', 'blend.cu', 'blend_bwd.cu'}


def _digest(paths):
    h = hashlib.sha256()
    for p in sorted(paths):
        h.update(p.name.encode())
        h.update(p.read_bytes())
    h.update(' '.join(FLAGS + ARCH + sorted(CONTRACTED) + sorted(FAST_MATH)).encode())
    return h.hexdigest()


def _compile(src: Path, headers_digest: str) -> Path:
    obj = BUILD / (src.stem + '.o')
    stamp = BUILD / (src.stem + '.stamp')
    key = headers_digest + hashlib.sha256(src.read_bytes()).hexdigest()
    if obj.exists() and stamp.exists() and stamp.read_text() == key:
        return obj
    flags = [f if not (f == '-fmad=false' and src.name in CONTRACTED) else '-fmad=true' for f in FLAGS]
    if src.name in FAST_MATH:
        flags = [f for f in flags if f != '-fmad=false'] + ['-use_fast_math']
    cmd = [NVCC, *ARCH, *flags, '-c', str(src), '-o', str(obj)]
    res = subprocess.run(cmd, capture_output=True, text=True)
    if res.returncode != 0:
        raise RuntimeError(f'nvcc failed for {src.name}:\n{res.stdout}\n{res.stderr}')
    if res.stderr.strip():
        sys.stderr.write(res.stderr)
    stamp.write_text(key)
    return obj


def build(force: bool = False) -> Path:
    BUILD.mkdir(exist_ok=True)
    LIB.parent.mkdir(parents=True, exist_ok=True)
    sources = sorted(CSRC.glob('*.cu'))
    headers = sorted(list(CSRC.glob('*.cuh')) + list(CSRC.glob('*.h')) + list((HERE.parent / 'include').glob('*.h')))
    hd = _digest(headers)
    if force:
        for f in BUILD.glob('*.stamp'):
            f.unlink()
    with concurrent.futures.ThreadPoolExecutor(max_workers=min(8, os.cpu_count() or 1)) as ex:
        objs = list(ex.map(lambda s: _compile(s, hd), sources))
    cmd = [NVCC, *ARCH, '-shared', '-o', str(LIB), *map(str, objs), '-lcudart']
    res = subprocess.run(cmd, capture_output=True, text=True)
    if res.returncode != 0:
        raise RuntimeError(f'link failed:\n{res.stdout}\n{res.stderr}')
    return LIB


if __name__ == '__main__':
    print(build(force='--force' in sys.argv))
