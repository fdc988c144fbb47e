"""The C ABI (include/vgb200.h) without a GPU: the in-tree library loads, exports every declared entry
point, and rejects bad arguments on the host with the reference's error categories."""

import ctypes
import os
import re

import pytest

from conftest import ROOT

HEADER = os.path.join(ROOT, 'include', 'vgb200.h')


def declared():
    src = open(HEADER).read()
    src = re.sub(r'/\*.*?\*/', '', src, flags=re.S)
    return sorted(set(re.findall(r'\b(vg_\w+)\s*\(', src)))


@pytest.fixture(scope='module')
def lib():
    from voronoi_gauss_b200 import _lib
    if not os.path.exists(_lib.LIB_PATH):
        from voronoi_gauss_b200 import build
        build.build()
    return _lib.lib()


def test_library_exports_every_declared_symbol(lib):
    names = declared()
    assert len(names) >= 14
    for n in names:
        assert hasattr(lib, n), n


def test_python_signatures_cover_the_header():
    from voronoi_gauss_b200 import _lib
    assert sorted(_lib.SIGNATURES) == declared()


def test_version(lib):
    assert lib.vg_version() == 100


def test_host_side_argument_errors(lib):
    """Null scene / bad degree / workspace too small are rejected before any device work."""
    null = None
    rc = lib.vg_foam_forward(null, 10, 10, null, null, null, null, 3, null, null, null, null, null, 0, 1e-4, 1e-4, 0,
                             null, null, null, null, null, null, 0, null)
    assert rc == 1 and b'graph pack is null' in lib.vg_last_error()
    buf = ctypes.create_string_buffer(64)
    p = ctypes.addressof(buf)
    rc = lib.vg_foam_forward(p, 10, 10, p, p, p, p, 4, p, p, p, p, p, 1, 1e-4, 1e-4, 0, p, p, p, p, null, p, 0, null)
    assert rc == 1 and b'sh_deg' in lib.vg_last_error()
    rc = lib.vg_foam_forward(p, 10, 10, p, p, p, p, 3, p, p, p, p, p, 1, 1e-4, 1e-4, -1, p, p, p, p, null, p, 0, null)
    assert rc == 1 and b'record_cap' in lib.vg_last_error()
    rc = lib.vg_foam_infer(p, p, p, p, p, p, 0, 3, 10, 20, p, p, p, p, p, 1, 1e-4, 1e-4, 1.0, 5, 2, null, null, p, p, p,
                           p, null)
    assert rc == 1 and b'color_mode' in lib.vg_last_error()
    rc = lib.vg_conic_forward(null, null, -1, 0.0, null, null)
    assert rc == 1


def test_python_layer_rejects_cpu_tensors():
    """ext raises the reference's CHECK_INPUT messages (foam.cu:34-37) before touching the library."""
    import torch
    from voronoi_gauss_b200 import ext
    x = torch.zeros(4, 3)
    with pytest.raises(RuntimeError, match='must be a CUDA tensor'):
        ext.extension().conic_forward(x, torch.zeros(4, 4), 0.0)


def test_host_side_argument_errors_of_the_field_packing_and_scene_entry_points(lib):
    """The field, packing and scene-preparation entry points validate on the host too."""
    null = None
    buf = ctypes.create_string_buffer(256)
    p = ctypes.addressof(buf)
    rc = lib.vg_walk(null, 10, 10, p, p, p, p, 1, 4, p, p, null)
    assert rc == 1 and b'graph pack is null' in lib.vg_last_error()
    assert lib.vg_field_workspace_bytes(10, 3, 7, 0) == 0
    assert lib.vg_field_workspace_bytes(10, 3, 3, 1000) > lib.vg_field_workspace_bytes(10, 3, 3, 0) > 0
    rc = lib.vg_density_forward(p, 10, 10, p, p, p, p, p, 5, 1.0, p, null, 0, null)
    assert rc == 2 and b'workspace' in lib.vg_last_error()
    rc = lib.vg_color_forward(p, 10, 10, p, p, p, 4, p, p, p, 5, p, p, 1 << 20, null)
    assert rc == 1 and b'sh_deg' in lib.vg_last_error()
    k = (ctypes.c_float * 9)(1, 0, 0, 0.5, 1, 0, 0, 0, 1)  # not the inverse of a pinhole intrinsic matrix
    r = (ctypes.c_float * 9)(1, 0, 0, 0, 1, 0, 0, 0, 1)
    c = (ctypes.c_float * 3)(0, 0, 0)
    rc = lib.vg_camera_rays(k, r, c, 4, 4, 4, 8, p, p, null)
    assert rc == 1 and b'K_inv' in lib.vg_last_error()
    rc = lib.vg_nearest_sites(null, 10, 10, p, 3, p, null)
    assert rc == 1 and b'graph pack is null' in lib.vg_last_error()
    ws = lib.vg_infer_pack_workspace_bytes(10)
    rc = lib.vg_infer_pack(null, 10, 10, p, p, p, p, p, p, p, p, p, 0.0, 0.0, 0, 1, p, p, p, p, p, p, p, p, p, ws,
                           null)
    assert rc == 1 and b'reorder' in lib.vg_last_error()
    rc = lib.vg_bake_colors(p, p, 5, 10, 0.0, 0.0, 0.0, p, null)
    assert rc == 1 and b'sh_deg' in lib.vg_last_error()


def test_workspace_sizes_are_aligned_and_monotone(lib):
    """The host-side size queries: every size is a multiple of 256 bytes, grows with the work it covers,
    and the cell-major march backward (backward = 3) asks for at least the per-sample scatter's size."""
    ws = lib.vg_foam_workspace_bytes
    sizes = []
    for n_sites, n_rays, cap, bwd in [(1000, 4096, 256, 0), (1000, 4096, 256, 1), (1000, 4096, 256, 2),
                                      (1000, 4096, 0, 3), (3_000_000, 2_073_600, 256, 0),
                                      (3_000_000, 2_073_600, 256, 1), (8_000_000, 8_294_400, 256, 1)]:
        b = ws(n_sites, 3, n_rays, cap, bwd)
        assert b > 0 and b % 256 == 0, (n_sites, n_rays, cap, bwd)
        sizes.append(b)
    assert ws(3_000_000, 3, 2_073_600, 256, 1) >= ws(1000, 3, 4096, 256, 1)
    assert ws(1000, 3, 4096, 0, 3) >= ws(1000, 3, 4096, 0, 1)
    assert ws(1000, 3, 8192, 0, 3) >= ws(1000, 3, 4096, 0, 3)
    assert ws(8_000_000, 3, 8_294_400, 256, 1) < 180 * 2 ** 30  # fits a B200 next to the records
    g = lib.vg_graph_pack_bytes
    assert g(1000, 15000) % 256 == 0 and g(2000, 30000) > g(1000, 15000)
    f = lib.vg_field_workspace_bytes
    assert f(1000, 3, 1, 10 ** 6) >= f(1000, 3, 1, 0) and f(1000, 3, 1, 0) % 256 == 0
    assert lib.vg_infer_pack_workspace_bytes(10 ** 6) >= 4 * 10 ** 6


def test_variant_builds_pass_their_knobs_and_need_their_own_directory():
    """`build --define` compiles with -D flags into a separate directory; the in-tree library is never
    overwritten by a variant."""
    from voronoi_gauss_b200 import build
    cmd = build.compile_command('x.cu', 'x.o', ('VG_BWD_HELPERS=1', 'VG_FWD_PREFETCH=1'))
    assert '-DVG_BWD_HELPERS=1' in cmd and '-DVG_FWD_PREFETCH=1' in cmd
    assert '-gencode' in cmd and 'arch=compute_100a,code=sm_100a' in cmd
    with pytest.raises(ValueError):
        build.build(defines=('VG_BWD_HELPERS=1',))


def test_kernel_timer_without_launches(lib):
    """vg_prof_enable / vg_prof_read with nothing recorded: zero time and launches, no device call; a bad
    kernel id is rejected."""
    from voronoi_gauss_b200 import _lib
    _lib.prof_enable(True)
    assert _lib.prof_read('scatter') == (0.0, 0)
    _lib.prof_enable(False)
    ms, n = ctypes.c_double(), ctypes.c_int64()
    assert lib.vg_prof_read(99, ctypes.byref(ms), ctypes.byref(n)) == 1
