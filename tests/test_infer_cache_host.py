"""The per-layout cache of the deferred inference renderer's trace records (ext.trace_records), on the CPU
with the library call replaced by a recorder: records are reused only for the very tensors they were
built from, rebuilt after an in-place change, and never handed to a new layout that happens to reuse the
memory (or the object id) of a freed one."""

import gc

import pytest
import torch


@pytest.fixture()
def recorder(monkeypatch):
    from voronoi_gauss_b200 import ext

    class NoDevice:
        def __init__(self, *a):
            pass

        def __enter__(self):
            return self

        def __exit__(self, *a):
            return False

    calls = []
    monkeypatch.setattr(ext._lib, 'call', lambda name, *a: calls.append(name))
    monkeypatch.setattr(ext.torch.cuda, 'device', NoDevice)
    monkeypatch.setattr(ext, '_stream', lambda dev: 0)
    monkeypatch.setattr(ext, '_TRACE_CACHE', {})
    return ext, calls


def _layout(n_edges=10, n_sites=5):
    return torch.zeros(n_edges, dtype=torch.int32), torch.zeros(n_edges, 4), torch.zeros(n_sites, 20)


def test_records_are_reused_for_the_same_layout(recorder):
    ext, calls = recorder
    nbr, edge, attr = _layout()
    a = ext.trace_records(nbr, edge, attr, 5)
    assert a.shape == (10, 12)
    assert ext.trace_records(nbr, edge, attr, 5) is a and calls == ['vg_infer_trace_records']


def test_in_place_change_rebuilds(recorder):
    ext, calls = recorder
    nbr, edge, attr = _layout()
    a = ext.trace_records(nbr, edge, attr, 5)
    attr[:, 0] += 1.0
    assert ext.trace_records(nbr, edge, attr, 5) is not a and len(calls) == 2


def test_a_new_layout_never_gets_stale_records(recorder):
    ext, calls = recorder
    for _ in range(6):  # freed layouts and their memory are reused by the allocator
        nbr, edge, attr = _layout()
        ext.trace_records(nbr, edge, attr, 5)
        del nbr, edge, attr
        gc.collect()
    assert len(calls) == 6
    assert len(ext._TRACE_CACHE) <= ext._TRACE_CACHE_SIZE
