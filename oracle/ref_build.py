"""TEST INFRASTRUCTURE ONLY — builds the reference's own CUDA extensions, unchanged, into oracle/_ref/.

    python oracle/ref_build.py            (needs the reference checkout, see reference_root())

Each of csrc/foam.cu, csrc/march.cu, csrc/foam_infer.cu and csrc/vgf.cu is compiled from where it lies
in the reference checkout by torch.utils.cpp_extension (the same tool the reference's ext.py:11-27
uses) for sm_100a, with the reference's flags (-O3 -lineinfo), into oracle/_ref/<name>/<name>.so. The
built modules travel to the GPU box, where tests/ load them with `load_reference(name)` to compare
the product with the reference's kernels on identical inputs. Nothing else in the repository uses them.
"""

from __future__ import annotations

import importlib.util
import os
import sys

HERE = os.path.dirname(os.path.abspath(__file__))
OUT = os.path.join(HERE, '_ref')
MODULES = {'vgf_foam': 'foam.cu', 'vgf_march': 'march.cu', 'vgf_foam_infer': 'foam_infer.cu', 'vgf_ext': 'vgf.cu'}


def reference_root():
    """The reference checkout: the directory named by VG_REFERENCE, else a directory `reference` beside
    this repository's own directory (where the build machine keeps it); None when neither holds csrc/."""
    env = os.environ.get('VG_REFERENCE')
    cands = [env] if env else [os.path.join(os.path.dirname(os.path.dirname(HERE)), 'reference')]
    for c in cands:
        if c and os.path.isdir(os.path.join(c, 'csrc')):
            return os.path.abspath(c)
    return None


def build(names=None, verbose=False):
    """Builds the named modules (default all). Several modules build at once, one child process each
    (every module has its own build directory)."""
    todo = [n for n in MODULES if not names or n in names]
    if len(todo) > 1:
        import subprocess
        procs = [(n, subprocess.Popen([sys.executable, os.path.abspath(__file__), n] + (['-v'] if verbose else []),
                                      stdout=subprocess.PIPE, stderr=subprocess.STDOUT, text=True)) for n in todo]
        failed = []
        for n, p in procs:
            out, _ = p.communicate()
            if p.returncode != 0:
                failed.append(f'{n}: {out[-2000:]}')
        if failed:
            raise RuntimeError('reference extension build failed:\n' + '\n'.join(failed))
        return [os.path.join(OUT, n, n + '.so') for n in todo]
    import torch  # noqa: F401  (the build needs torch's headers)
    from torch.utils.cpp_extension import load

    os.environ['TORCH_CUDA_ARCH_LIST'] = '10.0a'
    ref = reference_root()
    if ref is None:
        raise FileNotFoundError('reference checkout not found: set VG_REFERENCE to its directory')
    built = []
    for name, src in MODULES.items():
        if name not in todo:
            continue
        source = os.path.join(ref, 'csrc', src)
        if not os.path.exists(source):
            raise FileNotFoundError(source)
        bdir = os.path.join(OUT, name)
        os.makedirs(bdir, exist_ok=True)
        load(name=name, sources=[source], build_directory=bdir, verbose=verbose,
             extra_cuda_cflags=['-O3', '-lineinfo', '-gencode=arch=compute_100a,code=sm_100a'],
             extra_cflags=['-O3'])
        built.append(os.path.join(bdir, name + '.so'))
    return built


def available(name):
    return os.path.exists(os.path.join(OUT, name, name + '.so'))


def load_reference(name):
    """Imports a prebuilt reference extension module (no rebuild, no access to the reference sources)."""
    import torch  # noqa: F401  (resolves the extension's libtorch symbols)

    path = os.path.join(OUT, name, name + '.so')
    if not os.path.exists(path):
        raise FileNotFoundError(path)
    if name in sys.modules:
        return sys.modules[name]
    spec = importlib.util.spec_from_file_location(name, path)
    mod = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(mod)
    sys.modules[name] = mod
    return mod


if __name__ == '__main__':
    for p in build([a for a in sys.argv[1:] if a != '-v'] or None, verbose='-v' in sys.argv):
        print(p)
