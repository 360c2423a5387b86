"""Build the in-tree native libraries of trpg_b200.

    python -m trpg_b200.build            # builds what is out of date

Products (next to this file, so they travel with the source tree):

* ``libtrpg_ckv.so``  -- CUDA kernels + the C ABI of ``include/ckv.h``
  (nvcc, ``-gencode arch=compute_100a,code=sm_100a``, static cudart);
* ``_ckv_torch.so``   -- ``torch.library`` registration of the ``ckv`` ops,
  linked against ``libtrpg_ckv.so`` through ``$ORIGIN``.

nvcc cross-compiles for sm_100a without a GPU, so this runs on any machine
with CUDA 12.8+ and the torch headers.
"""
from __future__ import annotations

import os
import subprocess
import sys
from concurrent.futures import ThreadPoolExecutor
from pathlib import Path

PKG = Path(__file__).resolve().parent
ROOT = PKG.parent
CSRC = PKG / 'csrc'
INCLUDE = ROOT / 'include'
BUILD = PKG / '_build'
LIB = PKG / 'libtrpg_ckv.so'
TORCH_LIB = PKG / '_ckv_torch.so'

CUDA_HOME = Path(os.environ.get('CUDA_HOME', '/usr/local/cuda'))
NVCC = str(CUDA_HOME / 'bin' / 'nvcc')
ARCH = ['-gencode', 'arch=compute_100a,code=sm_100a']
NVCC_FLAGS = ['-O3', '-std=c++17', '-lineinfo', '-Xcompiler', '-fPIC', '--expt-relaxed-constexpr',
              f'-I{INCLUDE}', f'-I{CSRC}']

CU_SOURCES = ['ckv_capi.cu', 'ckv_pack.cu', 'ckv_attn.cu', 'ckv_static.cu', 'ckv_prefill.cu',
              'ckv_exchange.cu']
HEADERS = sorted(p.name for p in CSRC.glob('*.cuh'))


def _run(cmd):
    proc = subprocess.run(cmd, stdout=subprocess.PIPE, stderr=subprocess.STDOUT, text=True)
    if proc.returncode != 0:
        raise RuntimeError('command failed:\n' + ' '.join(cmd) + '\n' + proc.stdout)
    return proc.stdout


def _stale(target: Path, deps) -> bool:
    if not target.exists():
        return True
    t = target.stat().st_mtime
    return any(Path(d).stat().st_mtime > t for d in deps)


def build_cuda(verbose: bool = False) -> Path:
    BUILD.mkdir(exist_ok=True)
    headers = [CSRC / h for h in HEADERS] + [INCLUDE / 'ckv.h']
    objects = []
    jobs = []
    for src in CU_SOURCES:
        obj = BUILD / (Path(src).stem + '.o')
        objects.append(obj)
        if _stale(obj, [CSRC / src, *headers]):
            cmd = [NVCC, *ARCH, *NVCC_FLAGS, '-c', str(CSRC / src), '-o', str(obj)]
            if verbose:
                cmd += ['-Xptxas', '-v']
            jobs.append(cmd)
    with ThreadPoolExecutor(max_workers=max(1, min(len(jobs), os.cpu_count() or 1))) as ex:
        for out in ex.map(_run, jobs):
            if verbose and out:
                print(out)
    if _stale(LIB, objects):
        _run([NVCC, *ARCH, '-shared', '-o', str(LIB), *map(str, objects), '-lcudart_static',
              '-Xlinker', '--no-undefined', '-lrt', '-ldl', '-lpthread'])
    return LIB


def build_torch_binding() -> Path:
    import torch
    from torch.utils import cpp_extension

    src = CSRC / 'ckv_torch.cpp'
    if not _stale(TORCH_LIB, [src, INCLUDE / 'ckv.h', LIB]):
        return TORCH_LIB
    includes = cpp_extension.include_paths(device_type='cuda')
    libdirs = cpp_extension.library_paths(device_type='cuda')
    abi = int(torch._C._GLIBCXX_USE_CXX11_ABI)
    cmd = ['g++', '-O2', '-std=c++17', '-shared', '-fPIC', f'-D_GLIBCXX_USE_CXX11_ABI={abi}',
           f'-I{INCLUDE}', *[f'-I{p}' for p in includes], str(src), '-o', str(TORCH_LIB),
           f'-L{PKG}', '-ltrpg_ckv', *[f'-L{p}' for p in libdirs],
           '-lc10', '-lc10_cuda', '-ltorch', '-ltorch_cpu', '-ltorch_cuda',
           '-Wl,-rpath,$ORIGIN']
    _run(cmd)
    return TORCH_LIB


def build(verbose: bool = False):
    build_cuda(verbose)
    build_torch_binding()


if __name__ == '__main__':
    build(verbose='-v' in sys.argv)
    print('built', LIB.name, TORCH_LIB.name)
