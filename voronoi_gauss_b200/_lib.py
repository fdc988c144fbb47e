"""ctypes binding of libvgb200.so (include/vgb200.h).

The library is built in-tree by ``python -m voronoi_gauss_b200.build`` (or ``__graft_entry__.build()``).
There is no fallback: every render call goes through this library, and a missing or unloadable
library raises at the first call.
"""

from __future__ import annotations

import ctypes
import os

HERE = os.path.dirname(os.path.abspath(__file__))
# VG_LIB_PATH: load a variant of the library (python -m voronoi_gauss_b200.build --define ... --out DIR)
LIB_PATH = os.environ.get('VG_LIB_PATH') or os.path.join(HERE, '_lib', 'libvgb200.so')

_lib = None

P = ctypes.c_void_p
I64 = ctypes.c_int64
I32 = ctypes.c_int
F32 = ctypes.c_float
F64 = ctypes.c_double
SZ = ctypes.c_size_t

# entry point -> (restype, argtypes); mirrors include/vgb200.h
SIGNATURES = {
    'vg_version': (I32, []),
    'vg_last_error': (ctypes.c_char_p, []),
    'vg_status': (I32, [P]),
    'vg_status_reset': (I32, []),
    'vg_graph_pack_bytes': (SZ, [I64, I64]),
    'vg_graph_pack': (I32, [P, P, P, I64, I64, P, SZ, P]),
    'vg_foam_workspace_bytes': (SZ, [I64, I32, I64, I32, I32]),
    'vg_foam_forward': (I32, [P, I64, I64, P, P, P, P, I32, P, P, P, P, P, I64, F32, F32, I32, P, P, P, P, P, P, SZ,
                              P]),
    'vg_foam_forward_noalloc': (I32, [P, I64, I64, P, P, P, P, I32, P, P, P, P, P, I64, F32, F32, I32, P, P, P, P,
                                      P, P]),
    'vg_foam_backward': (I32, [P, I64, I64, P, P, P, P, I32, P, P, P, P, P, I64, F32, F32, P, P, P, P, P, I32, P, P, P,
                               P, P, P, SZ, P]),
    'vg_foam_counts_bytes': (SZ, [I64, I64, I32]),
    'vg_foam_forward_counted': (I32, [P, I64, I64, P, P, P, P, I32, P, P, P, P, P, I64, F32, F32, I32, P, P, P, P, P,
                                      P, P, SZ, P]),
    'vg_foam_backward_counted': (I32, [P, I64, I64, P, P, P, P, I32, P, P, P, P, P, I64, F32, F32, P, P, P, P, P, I32,
                                       P, P, P, P, P, P, P, SZ, P]),
    'vg_foam_backward_packed': (I32, [P, I64, I64, P, P, P, P, I32, P, P, P, P, P, I64, F32, F32, P, P, P, P, P, I32,
                                      P, P, I32, P, SZ, P]),
    'vg_grad_unpack': (I32, [P, I64, I64, P, I32, P, P, P, P, P]),
    'vg_march_forward': (I32, [P, I64, I64, P, P, P, P, I32, P, P, P, P, P, P, I64, F32, I32, F32, F32, P, P, P, P, P,
                               SZ, P]),
    'vg_march_backward': (I32, [P, I64, I64, P, P, P, P, I32, P, P, P, P, P, P, I64, F32, I32, F32, F32, P, P, P, P,
                                P, P, P, P, P, SZ, P]),
    'vg_conic_forward': (I32, [P, P, I64, F64, P, P]),
    'vg_conic_backward': (I32, [P, P, I64, F64, P, P, P, P]),
    'vg_walk': (I32, [P, I64, I64, P, P, P, P, I64, I64, P, P, P]),
    'vg_field_workspace_bytes': (SZ, [I64, I32, I32, I64]),
    'vg_density_forward': (I32, [P, I64, I64, P, P, P, P, P, I64, F64, P, P, SZ, P]),
    'vg_density_backward': (I32, [P, I64, I64, P, P, P, P, P, I64, P, P, P, P, P, SZ, P]),
    'vg_color_forward': (I32, [P, I64, I64, P, P, P, I32, P, P, P, I64, P, P, SZ, P]),
    'vg_color_backward': (I32, [P, I64, I64, P, P, P, I32, P, P, P, I64, P, P, P, P, P, P, SZ, P]),
    'vg_infer_pack_workspace_bytes': (SZ, [I64]),
    'vg_infer_pack': (I32, [P, I64, I64, P, P, P, P, P, P, P, P, P, F64, F64, I32, I32, P, P, P, P, P, P, P, P, P, SZ,
                            P]),
    'vg_bake_colors': (I32, [P, P, I32, I64, F32, F32, F32, P, P]),
    'vg_camera_rays': (I32, [P, P, P, I32, I32, I32, I32, P, P, P]),
    'vg_nearest_sites': (I32, [P, I64, I64, P, I64, P, P]),
    'vg_foam_infer': (I32, [P, P, P, P, P, P, I32, I32, I64, I64, P, P, P, P, P, I64, F32, F32, F32, I32, I32, P, P, P,
                            P, P, P, P]),
    'vg_foam_infer_workspace_bytes': (SZ, [I64, I64]),
    'vg_infer_trace_records': (I32, [P, P, P, I64, I64, P, P]),
    'vg_foam_infer_deferred': (I32, [P, P, P, P, P, P, I32, I32, I64, I64, P, P, P, P, P, I64, F32, F32, F32, I32, I32,
                                     P, P, P, P, P, P, P, P, SZ, P]),
    'vg_prof_enable': (I32, [I32]),
    'vg_prof_read': (I32, [I32, P, P]),
}

# kernel classes of vg_prof_read (VG_PROF_* of include/vgb200.h)
PROF = {'traversal': 0, 'color': 1, 'replay': 2, 'scatter': 3, 'infer': 4, 'march_fwd': 5, 'march_items': 6,
        'infer_color': 7}


def prof_enable(on):
    """Starts (forgetting earlier records) or stops recording kernel times (vg_prof_enable)."""
    check(lib().vg_prof_enable(1 if on else 0), 'vg_prof_enable')


def prof_read(kernel):
    """-> (summed device ms, launches) of one kernel class since prof_enable(True); waits for its events."""
    ms, n = ctypes.c_double(), ctypes.c_int64()
    check(lib().vg_prof_read(PROF[kernel], ctypes.byref(ms), ctypes.byref(n)), 'vg_prof_read')
    return ms.value, n.value


def lib():
    """The loaded library (raises if it has not been built)."""
    global _lib
    if _lib is None:
        if not os.path.exists(LIB_PATH):
            raise RuntimeError(f'{LIB_PATH} is missing: build it with `python -m voronoi_gauss_b200.build`')
        handle = ctypes.CDLL(LIB_PATH)
        for name, (res, args) in SIGNATURES.items():
            fn = getattr(handle, name)
            fn.restype, fn.argtypes = res, args
        _lib = handle
    return _lib


def check(rc, what):
    if rc != 0:
        msg = lib().vg_last_error().decode(errors='replace')
        raise RuntimeError(f'{what}: {msg}')


def call(name, *args):
    """Calls entry point `name` and raises RuntimeError with the library's message on failure."""
    check(getattr(lib(), name)(*args), name)
