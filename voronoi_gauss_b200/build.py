"""Builds libvgb200.so (the CUDA kernels + the C ABI of include/vgb200.h) in-tree for sm_100a.

    python -m voronoi_gauss_b200.build [--verbose]

Every .cu under csrc/ is compiled by nvcc to an object with -gencode arch=compute_100a,code=sm_100a
(static CUDA runtime, no torch headers) and linked into voronoi_gauss_b200/_lib/libvgb200.so, which
the package loads with ctypes. Objects are rebuilt only when a source or header is newer.
"""

from __future__ import annotations

import argparse
import concurrent.futures as cf
import glob
import os
import shutil
import subprocess

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(HERE)
CSRC = os.path.join(HERE, 'csrc')
OUT = os.path.join(HERE, '_lib')
OBJ = os.path.join(OUT, 'obj')
LIB = os.path.join(OUT, 'libvgb200.so')
ARCH = ['-gencode', 'arch=compute_100a,code=sm_100a']
FLAGS = ['-O3', '-std=c++17', '-lineinfo', '--expt-relaxed-constexpr', '-Xcompiler', '-fPIC,-O3',
         '-I', os.path.join(ROOT, 'include')]


def nvcc():
    path = shutil.which('nvcc') or '/usr/local/cuda/bin/nvcc'
    if not os.path.exists(path):
        raise RuntimeError('nvcc not found: the CUDA toolkit is required to build libvgb200')
    return path


def _compile(src, headers_mtime, verbose):
    obj = os.path.join(OBJ, os.path.basename(src)[:-3] + '.o')
    if os.path.exists(obj) and os.path.getmtime(obj) >= max(os.path.getmtime(src), headers_mtime):
        return obj
    cmd = [nvcc(), *ARCH, *FLAGS, '-c', src, '-o', obj]
    if verbose:
        cmd += ['-Xptxas', '-v']
    res = subprocess.run(cmd, capture_output=True, text=True)
    if res.returncode != 0:
        raise RuntimeError(f'nvcc failed on {src}:\n{res.stderr}')
    if verbose and res.stderr:
        print(res.stderr)
    return obj


def build(verbose=False):
    os.makedirs(OBJ, exist_ok=True)
    sources = sorted(glob.glob(os.path.join(CSRC, '*.cu')))
    headers = glob.glob(os.path.join(CSRC, '*.cuh')) + glob.glob(os.path.join(ROOT, 'include', '*.h'))
    hm = max(os.path.getmtime(h) for h in headers)
    with cf.ThreadPoolExecutor(max_workers=min(8, len(sources))) as ex:
        objs = list(ex.map(lambda s: _compile(s, hm, verbose), sources))
    if not os.path.exists(LIB) or os.path.getmtime(LIB) < max(os.path.getmtime(o) for o in objs):
        tmp = LIB + f'.{os.getpid()}.tmp'
        res = subprocess.run([nvcc(), *ARCH, '-shared', '-Xcompiler', '-fPIC', '-o', tmp, *objs],
                             capture_output=True, text=True)
        if res.returncode != 0:
            raise RuntimeError(f'link failed:\n{res.stderr}')
        os.replace(tmp, LIB)
    return LIB


if __name__ == '__main__':
    ap = argparse.ArgumentParser()
    ap.add_argument('--verbose', action='store_true')
    print(build(ap.parse_args().verbose))
