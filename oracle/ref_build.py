"""Builds the reference harness (test infrastructure only): the reference's own rasterizer, compiled from its unmodified
sources where they lie in the reference checkout, with outputs only in oracle/_ref/.

What is compiled, and how:
- The JIT preprocess kernels (FasterGSVDACudaBackend/FasterGSVDACudaBackend/rasterization/rtc/preprocess_forward.cu
  and preprocess_backward.cu with preprocess_common.cuh, include/tile_culling.cuh, include/appearance_params.h and the
  appearance chunk of the configuration) are assembled into one source in the order the reference's loader uses
  (rasterization/src/appearance.cu:85-145: the JIT_* token preamble and the generated config namespace, then
  appearance_params.h, tile_culling.cuh, preprocess_common.cuh, the appearance chunk, the kernel file) and compiled
  with NVRTC for sm_100a with fast math, as tiny-cuda-nn's runtime compiler does for the reference build
  (setup.py:125-129 defines TCNN_RTC_USE_FAST_MATH). tiny-cuda-nn's own NVRTC preamble is absent from the checkout;
  the one used here only declares the fixed-width integer types and includes cuda_fp16.h, which is all the non-neural
  sources use. One cubin per (kernel, configuration) in CONFIGS; the Neural model is not built (its source splices
  tiny-cuda-nn device functions that are absent).
- The host stage code and the AOT kernels (rasterization/src/forward.cu, backward.cu, inference.cu, which include
  include/kernels_forward.cuh, kernels_backward.cuh, kernels_inference.cuh, kernels_common.cuh, buffer_utils.h and
  utils/helper_math.h) together with oracle/ref_harness.cu (the C-ABI, this repository's code) are compiled by nvcc
  with the reference's flags (setup.py:112-129: -O3 -use_fast_math -std=c++17 --extended-lambda
  --expt-relaxed-constexpr and the half-operator undefines) into oracle/_ref/libfgsref.so. oracle/ref/ holds the
  stand-in for tiny-cuda-nn's CudaRtcKernel (a cuLaunchKernel wrapper).

Run: python oracle/ref_build.py [reference checkout]   (default: $FGS_REFERENCE, else a checkout named `reference`
next to this repository). Skips with a message when the checkout is absent.
"""
from __future__ import annotations

import ctypes
import hashlib
import json
import os
import subprocess
import sys
from pathlib import Path

HERE = Path(__file__).resolve().parent
OUT = HERE / '_ref'
CUDA = Path(os.environ.get('CUDA_HOME', '/usr/local/cuda'))
NVCC = str(CUDA / 'bin' / 'nvcc')

# (tag, model id, base act, residual act, color act, max degree) -- ids as in torch_bindings/rasterization.py:21-24
CONFIGS = [
    ('precomputed', 0, 0, 0, 0, 0),
    ('sh3_none_none_relu', 1, 0, 0, 1, 3),
    ('sh1_none_none_none', 1, 0, 0, 0, 1),
    ('sh2_exp_tanh_satexp', 1, 1, 1, 5, 2),
    ('sv8_none_none_relu', 2, 0, 0, 1, 8),
    ('nasg8_none_tanh_relu', 3, 0, 1, 1, 8),
    ('nasg8_none_none_relu', 3, 0, 0, 1, 8),
    ('nasgabor4_none_tanh_sigmoid', 4, 0, 1, 3, 4),
]
SUFFIX = {0: 'precomputed', 1: 'sh', 2: 'sv', 3: 'nasg', 4: 'nasgabor'}
CHUNK = {1: 'appearance_sh.cuh', 2: 'appearance_sv.cuh', 3: 'appearance_nasg.cuh', 4: 'appearance_nasgabor.cuh'}

TYPES_PRELUDE = """#include <cuda_fp16.h>
typedef unsigned char uint8_t;
typedef unsigned short uint16_t;
typedef unsigned int uint32_t;
typedef unsigned long long uint64_t;
typedef int int32_t;
typedef long long int64_t;
"""


def _reference(argv: list[str]) -> Path | None:
    cand = argv[1] if len(argv) > 1 else os.environ.get('FGS_REFERENCE', str(HERE.parent.parent / 'reference'))
    p = Path(cand)
    bk = p / 'FasterGSVDACudaBackend' / 'FasterGSVDACudaBackend'
    return p if (bk / 'rasterization' / 'rtc' / 'preprocess_forward.cu').is_file() else None


def _preamble(kernel_base: str, model: int, base: int, res: int, col: int, degree: int, with_backward: bool) -> str:
    """The token preamble of rasterization/src/appearance.cu:89-126 for a non-neural configuration (config values of
    rasterization/include/rasterization_config.h:10-61, written as exact float literals)."""
    pre = model == 0
    lines = [
        f'#define JIT_KERNEL_NAME {kernel_base}_{SUFFIX[model]}_cu',
        f'#define JIT_APPEARANCE_MODEL {model}',
        f'#define JIT_BASE_ACTIVATION {0 if pre else base}',
        f'#define JIT_RESIDUAL_ACTIVATION {0 if pre else res}',
        f'#define JIT_COLOR_ACTIVATION {0 if pre else col}',
        f'#define JIT_SH_REST_BASES {((degree + 1) ** 2 - 1) if model == 1 else 0}u',
        '#define JIT_N_INPUT_DIMS 0',
        '#define JIT_N_FEATURE_DIMS 0u',
        '#define JIT_LOSS_SCALE 128.000000f',
        '#define JIT_BASE_INPUT false',
        '#define JIT_N_FREQUENCIES 0u',
        '#define JIT_CTX_BYTES 0',
        f'#define JIT_WITH_BACKWARD {1 if with_backward else 0}',
        '#define JIT_SH_DEGREE_MASK 0u',
        f'#define JIT_NASG_N_LOBES {degree if model == 3 else 0}u',
        f'#define JIT_NASGABOR_N_LOBES {degree if model == 4 else 0}u',
        f'#define JIT_SV_N_SITES {degree if model == 2 else 0}u',
        f'#define JIT_DIRECTION_GRADIENT {"false" if pre else "true"}',
        'namespace faster_gs { namespace config {',
        'constexpr float dilation = 0.300000012f;',
        'constexpr float dilation_proper_antialiasing = 0.100000001f;',
        'constexpr bool detach_dilation_proper_antialiasing_from_cov2d = true;',
        'constexpr float min_cov2d_determinant = 9.99999997e-07f;',
        'constexpr bool original_opacity_interpretation = true;',
        'constexpr float min_alpha_threshold_rcp = 255.000000f;',
        'constexpr float min_alpha_threshold = 0.00392156886f;',
        'constexpr float max_power_threshold = 5.54126358f;',
        'constexpr uint32_t tile_width = 16u;',
        'constexpr uint32_t tile_height = 12u;',
        'constexpr uint32_t n_sequential_threshold = 4u;',
        'constexpr uint32_t block_size_preprocess = 128u;',
        '} }',
    ]
    return '\n'.join(lines) + '\n'


def _source(ref: Path, kernel_file: str, cfg: tuple) -> tuple[str, str]:
    _, model, base, res, col, degree = cfg
    ras = ref / 'FasterGSVDACudaBackend' / 'FasterGSVDACudaBackend' / 'rasterization'
    kernel_base = kernel_file[:-3]
    src = TYPES_PRELUDE + _preamble(kernel_base, model, base, res, col, degree, kernel_base.endswith('backward')) + '\n'
    src += (ras / 'include' / 'appearance_params.h').read_text() + '\n'
    src += (ras / 'include' / 'tile_culling.cuh').read_text() + '\n'
    src += (ras / 'rtc' / 'preprocess_common.cuh').read_text() + '\n'
    if model in CHUNK:
        src += (ras / 'rtc' / CHUNK[model]).read_text() + '\n'
    src += (ras / 'rtc' / kernel_file).read_text()
    return src, f'{kernel_base}_{SUFFIX[model]}_cu'


def _nvrtc():
    for name in ('libnvrtc.so', 'libnvrtc.so.12'):
        try:
            return ctypes.CDLL(str(CUDA / 'lib64' / name))
        except OSError:
            continue
    return ctypes.CDLL('libnvrtc.so')


def _nvrtc_compile(lib, src: str, name: str, tag: str) -> tuple[bytes, str]:
    prog = ctypes.c_void_p()
    r = lib.nvrtcCreateProgram(ctypes.byref(prog), src.encode(), f'{tag}.cu'.encode(), 0, None, None)
    if r:
        raise RuntimeError(f'nvrtcCreateProgram: {r}')
    lib.nvrtcAddNameExpression(prog, name.encode())
    opts = [b'--gpu-architecture=sm_100a', b'--std=c++17', b'--use_fast_math', f'-I{CUDA / "include"}'.encode()]
    arr = (ctypes.c_char_p * len(opts))(*opts)
    r = lib.nvrtcCompileProgram(prog, len(opts), arr)
    size = ctypes.c_size_t()
    lib.nvrtcGetProgramLogSize(prog, ctypes.byref(size))
    log = ctypes.create_string_buffer(size.value)
    lib.nvrtcGetProgramLog(prog, log)
    if r:
        raise RuntimeError(f'NVRTC failed for {tag}:\n{log.value.decode(errors="replace")}')
    lowered = ctypes.c_char_p()
    lib.nvrtcGetLoweredName(prog, name.encode(), ctypes.byref(lowered))
    lowered_name = lowered.value.decode()
    lib.nvrtcGetCUBINSize(prog, ctypes.byref(size))
    cubin = ctypes.create_string_buffer(size.value)
    lib.nvrtcGetCUBIN(prog, cubin)
    data = cubin.raw
    lib.nvrtcDestroyProgram(ctypes.byref(prog))
    return data, lowered_name


def build(argv: list[str] | None = None) -> bool:
    argv = sys.argv if argv is None else argv
    ref = _reference(argv)
    if ref is None:
        print('oracle/ref_build.py: no reference checkout found; the reference harness is not built')
        return False
    OUT.mkdir(exist_ok=True)
    bk = ref / 'FasterGSVDACudaBackend' / 'FasterGSVDACudaBackend'
    ras = bk / 'rasterization'
    # preprocess cubins
    lib = _nvrtc()
    index = {}
    for cfg in CONFIGS:
        for kernel_file in ('preprocess_forward.cu', 'preprocess_backward.cu'):
            src, name = _source(ref, kernel_file, cfg)
            key = hashlib.sha256(src.encode()).hexdigest()[:16]
            stem = f'{kernel_file[:-3]}_{cfg[0]}'
            cubin_path = OUT / f'{stem}.cubin'
            meta_path = OUT / f'{stem}.json'
            if cubin_path.exists() and meta_path.exists() and json.loads(meta_path.read_text()).get('key') == key:
                index[stem] = json.loads(meta_path.read_text())
                continue
            data, lowered = _nvrtc_compile(lib, src, name, stem)
            cubin_path.write_bytes(data)
            meta = {'key': key, 'kernel': lowered, 'cubin': cubin_path.name, 'config': cfg}
            meta_path.write_text(json.dumps(meta))
            index[stem] = meta
    (OUT / 'index.json').write_text(json.dumps(index, indent=1))
    # host code + AOT kernels + harness
    sources = [ras / 'src' / 'forward.cu', ras / 'src' / 'backward.cu', ras / 'src' / 'inference.cu', HERE / 'ref_harness.cu']
    flags = ['-gencode', 'arch=compute_100a,code=sm_100a', '-O3', '-use_fast_math', '-std=c++17', '--extended-lambda', '--expt-relaxed-constexpr',
             '-U__CUDA_NO_HALF_OPERATORS__', '-U__CUDA_NO_HALF_CONVERSIONS__', '-U__CUDA_NO_HALF2_OPERATORS__', '-Xcompiler=-fno-strict-aliasing',
             '-Xcompiler', '-fPIC', f'-I{HERE / "ref"}', f'-I{ras / "include"}', f'-I{bk / "utils"}']
    digest = hashlib.sha256(' '.join(flags).encode())
    for s in sources + [HERE / 'ref' / 'tiny-cuda-nn' / 'rtc_kernel.h']:
        digest.update(s.read_bytes())
    for h in sorted((ras / 'include').glob('*')) + sorted((bk / 'utils').glob('*')):
        digest.update(h.read_bytes())
    lib_path = OUT / 'libfgsref.so'
    stamp = OUT / 'libfgsref.stamp'
    if lib_path.exists() and stamp.exists() and stamp.read_text() == digest.hexdigest():
        return True
    objs = []
    for s in sources:
        obj = OUT / (s.stem + '.o')
        res = subprocess.run([NVCC, *flags, '-c', str(s), '-o', str(obj)], capture_output=True, text=True)
        if res.returncode:
            raise RuntimeError(f'nvcc failed for {s.name}:\n{res.stdout}\n{res.stderr}')
        objs.append(str(obj))
    res = subprocess.run([NVCC, '-gencode', 'arch=compute_100a,code=sm_100a', '-shared', '-o', str(lib_path), *objs, '-lcuda', '-lcudart'],
                         capture_output=True, text=True)
    if res.returncode:
        raise RuntimeError(f'link failed:\n{res.stdout}\n{res.stderr}')
    stamp.write_text(digest.hexdigest())
    return True


if __name__ == '__main__':
    print('built' if build() else 'skipped')
