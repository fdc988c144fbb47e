"""The autograd contracts of ext.foam / march / density / color / conic (ext.py:61-216 of the reference),
checked on the CPU with fake extension objects standing in for libvgb200: which tensors reach the
backward, which outputs are non-differentiable, where the input gradients go, and the no-gradient
shortcuts (no records kept, widened densities without a graph)."""

from types import SimpleNamespace

import pytest
import torch

from voronoi_gauss_b200 import ext


class FakeRender:
    """foam / march extension: records every call, returns tensors derived from the inputs."""

    def __init__(self):
        self.calls = []
        self.kwargs = []

    def _fwd(self, name, args, B, with_rec, cap):
        self.calls.append((name, args, cap))
        raw = args[3]
        rgb = torch.full((B, 3), float(raw.sum()))
        T = torch.full((B,), 0.5)
        depth = torch.ones(B)
        stats = torch.ones(B, 3, dtype=torch.int32)
        out = [rgb, T, depth, stats]
        if with_rec:
            out.append(torch.full((B if cap else 0, cap, 8), 7.0))
        return out

    def foam_forward(self, *args, counts=None):
        self.kwargs.append(('foam_forward', counts))
        return self._fwd('foam_forward', args, len(args[8]), True, args[-1])

    def march_forward(self, *args):
        return self._fwd('march_forward', args, len(args[8]), False, None)

    def _bwd(self, name, args):
        self.calls.append((name, args, None))
        raw, dA, cA, sh = args[3:7]
        return [torch.full_like(raw, 1.0), torch.full_like(dA, 2.0), torch.full_like(cA, 3.0), torch.full_like(sh, 4.0)]

    def foam_backward(self, *args, counts=None):
        self.kwargs.append(('foam_backward', counts))
        return self._bwd('foam_backward', args)

    def march_backward(self, *args):
        return self._bwd('march_backward', args)


class FakeField:
    def __init__(self):
        self.calls = []

    def density_forward(self, P, O, A, raw, ls, quat, x, site, scale_mult):
        self.calls.append(('density_forward', scale_mult))
        return torch.full((len(x),), float(raw.sum()))

    def density_backward(self, P, O, A, raw, ls, quat, x, site, g):
        self.calls.append(('density_backward', x, site, g))
        return [torch.full_like(raw, 1.0), torch.full_like(ls, 2.0), torch.full_like(quat, 3.0)]

    def color_forward(self, P, O, A, ls, quat, sh, sh_deg, x, dirs, site):
        self.calls.append(('color_forward', sh_deg))
        return torch.full((len(x), 3), float(sh.sum()))

    def color_backward(self, P, O, A, ls, quat, sh, sh_deg, x, dirs, site, rgb, g):
        self.calls.append(('color_backward', sh_deg, x, dirs, site, rgb, g))
        return [torch.full_like(ls, 1.0), torch.full_like(quat, 2.0), torch.full_like(sh, 3.0)]

    def conic_forward(self, ls, quat, floor):
        self.calls.append(('conic_forward', floor))
        return torch.zeros(len(ls), 6) + ls.sum()

    def conic_backward(self, ls, quat, floor, gA):
        self.calls.append(('conic_backward', floor, gA))
        return [torch.full_like(ls, 5.0), torch.full_like(quat, 6.0)]


@pytest.fixture()
def fakes(monkeypatch):
    render, field = FakeRender(), FakeField()
    monkeypatch.setattr(ext, '_FOAM', render)
    monkeypatch.setattr(ext, '_MARCH', render)
    monkeypatch.setattr(ext, '_FIELD', field)
    return render, field


def scene(n=5, requires_grad=True):
    graph = SimpleNamespace(points=torch.zeros(n, 3), offsets=torch.zeros(n + 1, dtype=torch.int32),
                            adj=torch.zeros(0, dtype=torch.int32))
    p = [torch.rand(n), torch.rand(n, 6), torch.rand(n, 6), torch.rand(n, 16, 3)]
    for t in p:
        t.requires_grad_(requires_grad)
    return graph, p


def rays(B=4):
    return torch.rand(B, 3), torch.rand(B, 3), torch.zeros(B, dtype=torch.int64), torch.rand(B), torch.rand(B)


def test_foam_saves_records_and_routes_gradients(fakes):
    render, _ = fakes
    graph, (raw, dA, cA, sh) = scene()
    o, d, start, near, far = rays()
    rgb, T, depth, stats = ext.foam(graph, raw, dA, cA, sh, 3, o, d, start, near, far, 1e-4, 1e-4, 16)
    assert rgb.requires_grad and T.requires_grad
    assert not depth.requires_grad and not stats.requires_grad
    name, args, cap = render.calls[-1]
    assert name == 'foam_forward' and cap == 16
    assert args[10].dtype == torch.int32  # start sites converted as the reference does
    (rgb.sum() + 2 * T.sum()).backward()
    name, args, _ = render.calls[-1]
    assert name == 'foam_backward'
    g_rgb, g_T, rec, st = args[-4:]
    assert torch.equal(g_rgb, torch.ones(4, 3)) and torch.equal(g_T, torch.full((4,), 2.0))
    assert rec.shape == (4, 16, 8) and bool((rec == 7).all()) and st.dtype == torch.int32
    assert torch.equal(args[8], o) and torch.equal(args[9], d)  # the same rays reach the backward
    assert bool((raw.grad == 1).all()) and bool((dA.grad == 2).all()) and bool((cA.grad == 3).all())
    assert bool((sh.grad == 4).all())
    # the recording forward keeps the per-cell sample counts of its records and hands them to its backward
    (f_name, f_counts), (b_name, b_counts) = render.kwargs[-2], render.kwargs[-1]
    assert (f_name, b_name) == ('foam_forward', 'foam_backward')
    assert f_counts is not None and f_counts.dtype == torch.int32 and b_counts is f_counts


def test_foam_missing_output_gradient_is_zero(fakes):
    render, _ = fakes
    graph, (raw, dA, cA, sh) = scene()
    rgb, T, _, _ = ext.foam(graph, raw, dA, cA, sh, 3, *rays())
    rgb.sum().backward()  # no gradient reaches T
    g_T = render.calls[-1][1][-3]
    assert torch.equal(g_T, torch.zeros(4))


def test_foam_without_gradients_keeps_no_records(fakes):
    render, _ = fakes
    graph, p = scene(requires_grad=False)
    out = ext.foam(graph, *p, 3, *rays(), record_cap=256)
    assert len(out) == 4 and render.calls[-1][2] == 0
    graph, p = scene()
    with torch.no_grad():
        out = ext.foam(graph, *p, 3, *rays(), record_cap=256)
    assert len(out) == 4 and render.calls[-1][2] == 0 and not out[0].requires_grad


def test_march_contract(fakes):
    render, _ = fakes
    graph, (raw, dA, cA, sh) = scene()
    o, d, start, near, far = rays()
    mid = 0.5 * (near + far)
    rgb, T, depth, stats = ext.march(graph, raw, dA, cA, sh, 3, o, d, start, near, mid, far, 0.01, 8)
    assert not depth.requires_grad and not stats.requires_grad
    args = render.calls[-1][1]
    assert args[14:] == (0.01, 8, 1e-4, 1e-4)  # dt, n_bg, t_thresh, w_thresh after the rays
    T.sum().backward()
    name, args, _ = render.calls[-1]
    assert name == 'march_backward'
    assert torch.equal(args[-2], torch.zeros(4, 3)) and torch.equal(args[-1], torch.ones(4))
    assert bool((sh.grad == 4).all())


def test_density_contract(fakes):
    _, field = fakes
    graph, (raw, _, _, _) = scene()
    ls, quat = torch.rand(5, 3, requires_grad=True), torch.rand(5, 4, requires_grad=True)
    x, site = torch.rand(7, 3), torch.zeros(7, dtype=torch.int64)
    sigma = ext.density(graph, raw, ls, quat, x, site, 2.0)  # widened: never differentiable
    assert not sigma.requires_grad and field.calls[-1] == ('density_forward', 2.0)
    sigma = ext.density(graph, raw, ls, quat, x, site)
    assert sigma.requires_grad and field.calls[-1] == ('density_forward', 1.0)
    (3 * sigma).sum().backward()
    name, xs, ss, g = field.calls[-1]
    assert name == 'density_backward' and ss.dtype == torch.int32 and torch.equal(g, torch.full((7,), 3.0))
    assert bool((raw.grad == 1).all()) and bool((ls.grad == 2).all()) and bool((quat.grad == 3).all())


def test_color_contract(fakes):
    _, field = fakes
    ls, quat = torch.rand(5, 3, requires_grad=True), torch.rand(5, 4, requires_grad=True)
    sh = torch.rand(5, 16, 3, requires_grad=True)
    graph, _ = scene()
    x, dirs, site = torch.rand(6, 3), torch.rand(6, 3), torch.zeros(6, dtype=torch.int64)
    rgb = ext.color(graph, ls, quat, sh, x, dirs, site, 2)
    rgb.sum().backward()
    name, deg, xs, ds, ss, saved_rgb, g = field.calls[-1]
    assert name == 'color_backward' and deg == 2 and torch.equal(saved_rgb, rgb.detach())
    assert torch.equal(g, torch.ones(6, 3)) and bool((sh.grad == 3).all())
    with torch.no_grad():
        assert not ext.color(graph, ls, quat, sh, x, dirs, site).requires_grad


def test_conic_contract(fakes):
    _, field = fakes
    ls, quat = torch.rand(5, 3, requires_grad=True), torch.rand(5, 4, requires_grad=True)
    A = ext.conic(ls, quat, 0.25)
    (2 * A).sum().backward()
    name, floor, gA = field.calls[-1]
    assert name == 'conic_backward' and floor == 0.25 and torch.equal(gA, torch.full((5, 6), 2.0))
    assert bool((ls.grad == 5).all()) and bool((quat.grad == 6).all())


def test_conic_reference_is_a_rotation_sandwich():
    g = torch.Generator().manual_seed(3)
    ls, quat = torch.randn(50, 3, generator=g, dtype=torch.float64), torch.randn(50, 4, generator=g,
                                                                                dtype=torch.float64)
    A = ext.conic_reference(ls, quat, 0.1)
    full = torch.zeros(50, 3, 3, dtype=torch.float64)
    for k, (i, j) in enumerate(((0, 0), (0, 1), (0, 2), (1, 1), (1, 2), (2, 2))):
        full[:, i, j] = full[:, j, i] = A[:, k]
    ev = torch.linalg.eigvalsh(full)
    want = torch.sort(1.0 / (torch.exp(2 * ls) + 0.01), -1)[0]
    assert torch.allclose(ev, want, rtol=1e-10)
