"""vg_foam_forward_noalloc: the forward render for callers that cannot allocate device memory while
rendering. It must give the same outputs as vg_foam_forward (which takes a caller-allocated workspace)
on consecutive calls, since every call reuses the same static scratch; it must not allocate device
memory; and it must refuse scenes larger than that scratch instead of overrunning it. Kept in the last
test file so that a failure here cannot stop the rest of the suite."""

import ctypes

import numpy as np
import pytest
import torch

from conftest import cuda, small_inputs

pytestmark = pytest.mark.gpu

IMG_TOL = 1e-4  # the image tolerance of the other parity tests


def _call(name, pk, x, sh_deg, K, with_workspace):
    from voronoi_gauss_b200 import _lib
    B = x['o'].size(0)
    rgb, T, depth = (torch.empty(B, 3, device='cuda'), torch.empty(B, device='cuda'),
                     torch.empty(B, device='cuda'))
    stats = torch.empty(B, 3, dtype=torch.int32, device='cuda')
    rec = torch.empty(B if K else 0, K, 8, device='cuda')
    common = [pk.ptr, pk.n, pk.m, x['raw'].data_ptr(), x['dA'].data_ptr(), x['cA'].data_ptr(), x['sh'].data_ptr(),
              sh_deg, x['o'].data_ptr(), x['d'].data_ptr(), x['start'].data_ptr(), x['near'].data_ptr(),
              x['far'].data_ptr(), B, 1e-4, 1e-4, K, rgb.data_ptr(), T.data_ptr(), depth.data_ptr(),
              stats.data_ptr(), rec.data_ptr() if K else None]
    stream = torch.cuda.current_stream().cuda_stream
    if with_workspace:
        nbytes = _lib.lib().vg_foam_workspace_bytes(pk.n, sh_deg, B, K, 0)
        ws = torch.empty(nbytes, dtype=torch.uint8, device='cuda')
        _lib.call(name, *common, ws.data_ptr(), nbytes, stream)
    else:
        _lib.call(name, *common, stream)
    torch.cuda.synchronize()
    return rgb, T, depth, stats, rec


def _compare(a, b, K):
    for u, v in zip(a[:3], b[:3]):
        assert float((u - v).abs().max()) <= IMG_TOL
    assert torch.equal(a[3], b[3])
    if K:
        s = a[3][:, 0].clamp(max=K)
        valid = torch.arange(K, device='cuda')[None, :] < s[:, None]
        assert float((a[4][valid] - b[4][valid]).abs().max()) <= IMG_TOL


def test_noalloc_forward_matches_workspace_forward_on_consecutive_calls(foam_small):
    from voronoi_gauss_b200 import ext
    z = foam_small
    pk = ext.GraphPack(cuda(z['points']), cuda(z['offsets']), cuda(z['adj']))
    x = small_inputs(z)
    # first call: SH degree 3 with records
    a = _call('vg_foam_forward_noalloc', pk, x, 3, 64, False)
    b = _call('vg_foam_forward', pk, x, 3, 64, True)
    _compare(a, b, 64)
    # second call on the same scratch: another field, SH degree 1, no records
    x2 = dict(x)
    x2['raw'] = (x['raw'] * 0.7 + 0.2).contiguous()
    x2['sh'] = (x['sh'].flip(0) * 1.3).contiguous()
    a = _call('vg_foam_forward_noalloc', pk, x2, 1, 0, False)
    b = _call('vg_foam_forward', pk, x2, 1, 0, True)
    _compare(a, b, 0)
    assert not torch.equal(a[0], _call('vg_foam_forward', pk, x, 1, 0, True)[0])  # the field did change


def test_noalloc_forward_allocates_no_device_memory(foam_small):
    """The entry point's promise: with the outputs already allocated, repeated calls leave the device's
    free memory unchanged (cudaMemGetInfo sees every allocator, the library's own included)."""
    from voronoi_gauss_b200 import _lib, ext
    z = foam_small
    pk = ext.GraphPack(cuda(z['points']), cuda(z['offsets']), cuda(z['adj']))
    x = small_inputs(z)
    B, K = x['o'].size(0), 64
    outs = [torch.empty(B, 3, device='cuda'), torch.empty(B, device='cuda'), torch.empty(B, device='cuda'),
            torch.empty(B, 3, dtype=torch.int32, device='cuda'), torch.empty(B, K, 8, device='cuda')]
    args = [pk.ptr, pk.n, pk.m, *(x[k].data_ptr() for k in ('raw', 'dA', 'cA', 'sh')), 3,
            *(x[k].data_ptr() for k in ('o', 'd', 'start', 'near', 'far')), B, 1e-4, 1e-4, K,
            *(t.data_ptr() for t in outs), torch.cuda.current_stream().cuda_stream]
    _lib.call('vg_foam_forward_noalloc', *args)  # first call on this device: looks up the scratch address
    torch.cuda.synchronize()
    free_before = torch.cuda.mem_get_info()[0]
    for _ in range(5):
        _lib.call('vg_foam_forward_noalloc', *args)
    torch.cuda.synchronize()
    assert torch.cuda.mem_get_info()[0] == free_before


def test_noalloc_forward_rejects_scenes_beyond_its_scratch():
    from voronoi_gauss_b200 import _lib
    dummy = ctypes.create_string_buffer(16)
    p = ctypes.addressof(dummy)
    rc = _lib.lib().vg_foam_forward_noalloc(p, 131073, 10, p, p, p, p, 3, p, p, p, p, p, 1, 1e-4, 1e-4, 0, p, p, p, p,
                                            None, None)
    assert rc == 2  # VG_ERR_WORKSPACE, before any device work
    assert b'131072' in _lib.lib().vg_last_error()
