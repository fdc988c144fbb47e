"""Data-parallel rendering and training across the GPUs of one node (one process per GPU).

Rays are independent, so rendering shards with no data-path communication: an image is cut into 16x16
pixel tiles dealt round-robin to the ranks (``tile_pixels``), or every rank renders its own share of the
tiles of a pool of views (``pool_tile_pixels``). The
scene (sites, adjacency, parameters) is replicated on every GPU (``broadcast_scene`` at load time), and
``gather_image`` assembles a tile-sharded frame for output. The one exchange step is in training:
the per-site gradients of all ranks are summed before the (replicated) optimizer step, by asynchronous
NCCL all-reduces over NVLink, one per gradient tensor (``allreduce_grads``). The reference is
single-GPU; this layer has no counterpart there.
"""

from __future__ import annotations

import numpy as np
import torch
import torch.distributed as dist

TILE = 16


def tile_pixels(H, W, world, rank, tile=TILE):
    """Pixel indices (row-major into H x W) of the tiles owned by `rank`: tile t (row-major over the tile
    grid) belongs to rank t mod world; inside a rank, tiles keep their order and pixels are listed tile
    by tile in 4 x 8 sub-tiles so that 32 consecutive rays cover a compact patch."""
    ty, tx = (H + tile - 1) // tile, (W + tile - 1) // tile
    tiles = np.arange(ty * tx)
    mine = tiles[tiles % world == rank]
    out = []
    sy, sx = np.meshgrid(np.arange(tile), np.arange(tile), indexing='ij')
    key = ((sy // 4) * (tile // 8) + sx // 8) * 32 + (sy % 4) * 8 + sx % 8
    sub = np.argsort(key.ravel(), kind='stable')
    sy, sx = sy.ravel()[sub], sx.ravel()[sub]
    for t in mine:
        y0, x0 = (t // tx) * tile, (t % tx) * tile
        y, x = y0 + sy, x0 + sx
        keep = (y < H) & (x < W)
        out.append(y[keep] * W + x[keep])
    return np.concatenate(out) if out else np.zeros(0, np.int64)


def pool_tile_pixels(H, W, rank, views=8, tile=TILE):
    """Weak-scaling deal over a fixed pool of `views` camera views: rank r renders, of every view v, the
    16x16 tiles t with t = r + v mod views (``tile_pixels`` with `views` parts), i.e. one view's worth of
    rays drawn evenly from all the views. A rank's share does not depend on how many ranks run (up to
    `views`), so adding ranks adds work without changing any rank's mix. Returns one pixel-index array
    per view."""
    if not 0 <= rank < views:
        raise ValueError(f'rank {rank} outside the pool of {views} views')
    return [tile_pixels(H, W, views, (rank + v) % views, tile) for v in range(views)]


def allreduce_grads(params, group=None):
    """Sums the .grad of `params` over the ranks, in place: one asynchronous all-reduce per gradient
    tensor (the per-site gradients are a few large contiguous tensors, so no flattening copies), then
    waits for all of them. Parameters without a gradient contribute zeros. Every rank must call it with
    the same parameter list."""
    grads = []
    for p in params:
        if p.grad is None:
            p.grad = torch.zeros_like(p)
        grads.append(p.grad)
    if dist.get_world_size(group) == 1:
        return
    works = [dist.all_reduce(g, group=group, async_op=True) for g in grads]
    for w in works:
        w.wait()


def broadcast_scene(tensors, src=0, group=None):
    """Makes every rank's copy of the scene (sites, adjacency, parameters) equal to rank `src`'s: one
    in-place broadcast per tensor, issued asynchronously and then waited for. Every rank passes tensors of
    the same shapes and dtypes in the same order."""
    if not dist.is_initialized() or dist.get_world_size(group) == 1:
        return
    works = [dist.broadcast(t, src, group=group, async_op=True) for t in tensors]
    for w in works:
        w.wait()


def gather_image(local, H, W, group=None, tile=TILE):
    """The full H x W image from every rank's pixels of ``tile_pixels`` (`local` (P_r, C), in that pixel
    order): the ranks' pixel runs, padded to the longest, are all-gathered and scattered back into image
    order. Returns (H, W, C) on every rank (outside the timed step: this is the output path)."""
    world = dist.get_world_size(group) if dist.is_initialized() else 1
    C = local.shape[1]
    out = torch.empty(H * W, C, dtype=local.dtype, device=local.device)
    if world == 1:
        out[torch.from_numpy(tile_pixels(H, W, 1, 0, tile)).to(local.device)] = local
        return out.view(H, W, C)
    sizes = [len(tile_pixels(H, W, world, r, tile)) for r in range(world)]
    pad = torch.zeros(max(sizes), C, dtype=local.dtype, device=local.device)
    pad[:len(local)] = local
    parts = [torch.empty_like(pad) for _ in range(world)]
    dist.all_gather(parts, pad, group=group)
    for r in range(world):
        idx = torch.from_numpy(tile_pixels(H, W, world, r, tile)).to(local.device)
        out[idx] = parts[r][:sizes[r]]
    return out.view(H, W, C)


def allreduce_max(values, device, group=None):
    """Element-wise maximum over the ranks of a list of floats (timings: the slowest rank counts)."""
    t = torch.tensor(values, dtype=torch.float64, device=device)
    if dist.is_initialized() and dist.get_world_size(group) > 1:
        dist.all_reduce(t, op=dist.ReduceOp.MAX, group=group)
    return [float(x) for x in t]
