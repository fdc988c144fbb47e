"""Multi-process logic of the data-parallel layer on CPU ranks (gloo, world size 2): tile sharding covers
every pixel once, the coalesced gradient all-reduce sums, and a rank that fails makes the others' next
collective fail on the host (no GPU involved)."""

import datetime
import os
import socket

import numpy as np
import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp


def _port():
    s = socket.socket()
    s.bind(('127.0.0.1', 0))
    p = s.getsockname()[1]
    s.close()
    return p


def _init(rank, world, port, timeout_s=60):
    os.environ['MASTER_ADDR'] = '127.0.0.1'
    os.environ['MASTER_PORT'] = str(port)
    dist.init_process_group('gloo', rank=rank, world_size=world, timeout=datetime.timedelta(seconds=timeout_s))


def _allreduce_worker(rank, world, port, q):
    import sys
    sys.path.insert(0, os.path.dirname(os.path.dirname(os.path.abspath(__file__))))
    from voronoi_gauss_b200 import dist as vdist
    _init(rank, world, port)
    a = torch.nn.Parameter(torch.zeros(5))
    b = torch.nn.Parameter(torch.zeros(2, 3))
    c = torch.nn.Parameter(torch.zeros(4))  # no gradient on any rank
    a.grad = torch.full((5,), float(rank + 1))
    b.grad = torch.arange(6.0).view(2, 3) * (rank + 1)
    vdist.allreduce_grads([a, b, c])
    mx = vdist.allreduce_max([float(rank), 10.0 - rank], 'cpu')
    q.put((rank, a.grad.tolist(), b.grad.tolist(), c.grad.tolist(), mx))
    dist.destroy_process_group()


def test_allreduce_grads_sums_over_ranks():
    world, port = 2, _port()
    ctx = mp.get_context('spawn')
    q = ctx.Queue()
    procs = [ctx.Process(target=_allreduce_worker, args=(r, world, port, q)) for r in range(world)]
    for p in procs:
        p.start()
    res = [q.get(timeout=120) for _ in range(world)]
    for p in procs:
        p.join(60)
        assert p.exitcode == 0
    for rank, a, b, c, mx in res:
        assert a == [3.0] * 5
        assert b == (torch.arange(6.0).view(2, 3) * 3).tolist()
        assert c == [0.0] * 4
        assert mx == [1.0, 10.0]


def _failing_worker(rank, world, port, q):
    _init(rank, world, port, timeout_s=5)
    x = torch.ones(4)
    dist.all_reduce(x)  # both ranks
    if rank == 1:
        q.put((rank, 'left'))
        q.close()
        q.join_thread()  # flush the message before leaving
        os._exit(3)  # leaves between steps, no collective in flight
    try:
        dist.all_reduce(x)  # the peer is gone: must fail, not hang
        q.put((rank, 'no error'))
    except Exception as e:  # noqa: BLE001
        q.put((rank, 'error:' + type(e).__name__))
    q.close()
    q.join_thread()


def test_rank_failure_surfaces_as_error_on_peers():
    world, port = 2, _port()
    ctx = mp.get_context('spawn')
    q = ctx.Queue()
    procs = [ctx.Process(target=_failing_worker, args=(r, world, port, q)) for r in range(world)]
    for p in procs:
        p.start()
    res = dict(q.get(timeout=120) for _ in range(world))
    for p in procs:
        p.join(60)
    assert res[1] == 'left'
    assert res[0].startswith('error:')


def test_tile_pixels_partition_image():
    from voronoi_gauss_b200 import dist as vdist
    H, W = 70, 90  # ragged edge tiles
    for world in (1, 2, 3, 8):
        parts = [vdist.tile_pixels(H, W, world, r) for r in range(world)]
        allp = np.concatenate(parts)
        assert len(allp) == H * W and len(np.unique(allp)) == H * W
        sizes = [len(p) for p in parts]
        assert max(sizes) - min(sizes) <= 2 * 16 * 16  # at most two tiles apart (ragged edge tiles)


def test_pool_tile_pixels_cover_every_view_once():
    from voronoi_gauss_b200 import dist as vdist
    H, W = 70, 90
    views = 8
    per_rank = [vdist.pool_tile_pixels(H, W, r, views) for r in range(views)]
    for v in range(views):
        allp = np.concatenate([per_rank[r][v] for r in range(views)])
        assert len(allp) == H * W and len(np.unique(allp)) == H * W
    sizes = [sum(len(p) for p in vs) for vs in per_rank]
    # every rank renders about one view's worth of rays, from all the views
    assert max(sizes) - min(sizes) <= 2 * views * 16 * 16 and sum(sizes) == views * H * W
    assert all(len(p) > 0 for p in per_rank[0])
    # a rank's share does not depend on the world size
    assert all(np.array_equal(a, b) for a, b in zip(per_rank[1], vdist.pool_tile_pixels(H, W, 1, views)))
    with pytest.raises(ValueError):
        vdist.pool_tile_pixels(H, W, views, views)


def _scene_worker(rank, world, port, q):
    import sys
    sys.path.insert(0, os.path.dirname(os.path.dirname(os.path.abspath(__file__))))
    from voronoi_gauss_b200 import dist as vdist
    _init(rank, world, port)
    # rank 0 holds the scene; the others start from different (wrong) copies
    pts = torch.arange(12.0).view(4, 3) + 100 * rank
    adj = torch.arange(7, dtype=torch.int32) * (rank + 1)
    vdist.broadcast_scene([pts, adj])
    # every rank shades its own tiles with the pixel index; the gathered frame must be arange
    H, W = 37, 53
    pix = torch.from_numpy(vdist.tile_pixels(H, W, world, rank))
    local = torch.stack([pix.float(), -pix.float()], 1)
    img = vdist.gather_image(local, H, W)
    q.put((rank, pts.tolist(), adj.tolist(), img.tolist()))
    dist.destroy_process_group()


def test_broadcast_scene_and_gather_image():
    world, port = 2, _port()
    ctx = mp.get_context('spawn')
    q = ctx.Queue()
    procs = [ctx.Process(target=_scene_worker, args=(r, world, port, q)) for r in range(world)]
    for p in procs:
        p.start()
    res = [q.get(timeout=120) for _ in range(world)]
    for p in procs:
        p.join(60)
        assert p.exitcode == 0
    ref = torch.arange(37 * 53, dtype=torch.float32).view(37, 53)
    for rank, pts, adj, img in res:
        assert pts == (torch.arange(12.0).view(4, 3)).tolist()
        assert adj == torch.arange(7).tolist()
        img = torch.tensor(img)
        assert torch.equal(img[..., 0], ref) and torch.equal(img[..., 1], -ref)


def test_gather_image_single_process():
    from voronoi_gauss_b200 import dist as vdist
    H, W = 20, 33
    pix = torch.from_numpy(vdist.tile_pixels(H, W, 1, 0))
    img = vdist.gather_image(pix.float()[:, None], H, W)
    assert torch.equal(img[..., 0], torch.arange(H * W, dtype=torch.float32).view(H, W))
