"""Builds libvgb200.so (the CUDA kernels + the C ABI of include/vgb200.h) in-tree for sm_100a.

    python -m voronoi_gauss_b200.build [--verbose]
    python -m voronoi_gauss_b200.build --define VG_INFER_UNROLL=4 --out DIR   # a variant library

Every .cu under csrc/ is compiled by nvcc to an object with -gencode arch=compute_100a,code=sm_100a
(static CUDA runtime, no torch headers) and linked into voronoi_gauss_b200/_lib/libvgb200.so, which
the package loads with ctypes. Objects are rebuilt when a source or header is newer, or when the
compiler flags or knob defines differ from the ones recorded beside the objects (`flags.txt`). A
variant with other values of the kernels' build knobs (the VG_* macros of csrc/) goes to its own
directory; setting VG_LIB_PATH to its libvgb200.so makes the package load it instead of the in-tree one.
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


def compile_command(src, obj, defines=()):
    """nvcc command line of one source; `defines` are NAME=VALUE strings passed as -D."""
    return [nvcc(), *ARCH, *FLAGS, *(f'-D{d}' for d in defines), '-c', src, '-o', obj]


def flag_signature(defines=()):
    """The compile flags and sorted knob defines an object directory was built with (one per line)."""
    return '\n'.join([*ARCH, *FLAGS, *sorted(f'-D{d}' for d in defines)]) + '\n'


def _sync_flags(obj_dir, defines):
    """Removes the objects of `obj_dir` when they were compiled with other flags or defines than these,
    and records the new signature, so that a rebuild with other knobs never reuses stale objects."""
    stamp = os.path.join(obj_dir, 'flags.txt')
    want = flag_signature(defines)
    have = open(stamp).read() if os.path.exists(stamp) else None
    if have != want:
        for o in glob.glob(os.path.join(obj_dir, '*.o')):
            os.remove(o)
        with open(stamp, 'w') as f:
            f.write(want)


def _compile(src, headers_mtime, verbose, obj_dir=OBJ, defines=()):
    obj = os.path.join(obj_dir, os.path.basename(src)[:-3] + '.o')
    if os.path.exists(obj) and os.path.getmtime(obj) >= max(os.path.getmtime(src), headers_mtime):
        return obj
    cmd = compile_command(src, obj, defines)
    if verbose:
        cmd += ['-Xptxas', '-v']
    res = subprocess.run(cmd, capture_output=True, text=True)
    if res.returncode != 0:
        raise RuntimeError(f'nvcc failed on {src}:\n{res.stderr}')
    if verbose and res.stderr:
        print(res.stderr)
    return obj


def build(verbose=False, defines=(), out=None):
    """Builds the library (in-tree by default; with `defines`, a variant into `out`). -> its path."""
    if defines and out is None:
        raise ValueError('a variant build (defines) needs its own output directory')
    out_dir = OUT if out is None else os.path.abspath(out)
    obj_dir, lib = os.path.join(out_dir, 'obj'), os.path.join(out_dir, 'libvgb200.so')
    os.makedirs(obj_dir, exist_ok=True)
    _sync_flags(obj_dir, defines)
    sources = sorted(glob.glob(os.path.join(CSRC, '*.cu')))
    headers = glob.glob(os.path.join(CSRC, '*.cuh')) + glob.glob(os.path.join(ROOT, 'include', '*.h'))
    hm = max(os.path.getmtime(h) for h in headers)
    with cf.ThreadPoolExecutor(max_workers=min(8, len(sources))) as ex:
        objs = list(ex.map(lambda s: _compile(s, hm, verbose, obj_dir, tuple(defines)), sources))
    if not os.path.exists(lib) or os.path.getmtime(lib) < max(os.path.getmtime(o) for o in objs):
        tmp = lib + f'.{os.getpid()}.tmp'
        res = subprocess.run([nvcc(), *ARCH, '-shared', '-Xcompiler', '-fPIC', '-o', tmp, *objs],
                             capture_output=True, text=True)
        if res.returncode != 0:
            raise RuntimeError(f'link failed:\n{res.stderr}')
        os.replace(tmp, lib)
    knobs = os.path.join(out_dir, 'defines.txt')
    if defines:
        with open(knobs, 'w') as f:
            f.write('\n'.join(defines) + '\n')
    elif os.path.exists(knobs):
        os.remove(knobs)
    return lib


if __name__ == '__main__':
    ap = argparse.ArgumentParser()
    ap.add_argument('--verbose', action='store_true')
    ap.add_argument('--define', action='append', default=[], help='NAME=VALUE of a VG_* build knob (repeatable)')
    ap.add_argument('--out', default=None, help='output directory of a variant build')
    a = ap.parse_args()
    print(build(a.verbose, a.define, a.out))
