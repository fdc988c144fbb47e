"""Benchmark of the B200 Voronoi-Gaussian renderer (one JSON line on rank 0).

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl b200|reference] [--config 3]
    torchrun --nproc-per-node N bench.py --gpus N ...

--config 3 (default, the configuration the headline metric is quoted on): a step is one training
iteration of the interaction-point renderer on BASELINE config 3 (3M sites, 70 % near a union of
spheres, SH degree 3, one 1920x1080 view from an orbit camera of radius 3): conics of both Gaussians,
ext.foam forward with records, background composite and L2 loss against a seeded random target,
backward through foam and conics, and a fused Adam step. With N GPUs every rank renders one view's
worth of rays (weak scaling) and the per-site gradients are summed with NCCL all-reduces before Adam.
`value` has the step's inputs resident in HBM; `e2e` repeats the step with the rays and target copied
from pinned host memory and the loss read back every step. The scene (1 GB of site records and
adjacency) is larger than L2, so no L2 flush is needed between steps. config 1 is the same step on the
tiny scene; --strong renders one 3840x2160 frame of the scene tile-sharded over the GPUs (config 4's
layout).

--config 2: inference. A step renders one 800x800 view of the 1M-site mixture scene (views 0, 8, 16,
... of 100 orbit cameras) with the inference renderer in the reference's fast configuration (fused
colours, fp16 SH, eps 1e-4 for density and colour, 4x8 pixel tiles, Morton order), and the same frames
through the reference's own foam_infer kernel.

--config 5: fixed-step ray marching. A step is one training iteration of ext.march (dt 2/256 through
the unit ball, 1920x1080, the 1M-site mixture scene), forward + backward + Adam, beside the reference's
march kernels.

The roofline object describes the step's dominant kernel, timed by itself inside the timed region with
CUDA events on its launch stream (the library's vg_prof_* registry), against its algorithmic bytes per
launch (formulas in algorithmic_bytes_* below).

`--impl reference` times the reference path on the host cores (the CPU restatement in oracle/, all
threads) on a bounded sample of the same workload, as the reference arm.
"""

from __future__ import annotations

import argparse
import json
import math
import os
import statistics
import subprocess
import sys
import time

import numpy as np
import torch

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, ROOT)

LR = {'raw': 2e-2, 'scale': 5e-3, 'quat': 2e-3, 'sh_dc': 5e-3, 'sh_rest': 2.5e-4, 'bg': 1e-2}  # train.py:21
RECORD_CAP = 256       # ext.foam default (ext.py:205)
T_THRESH = W_THRESH = 1e-4
CM_CHUNK = 64          # samples of one cell per warp in the cell-major passes (foam.cu VG_CM_CHUNK)
CM_SLOTS = 1 << 26     # record slots bucketed per pass of the cell-major passes (foam.cu kCmItems)
REF_REPS = 3           # reference-kernel repetitions (bench_vs_radfoam.py:26-36 protocol: 1 warm-up, >= 3 reps)


def parse():
    ap = argparse.ArgumentParser()
    ap.add_argument('--gpus', type=int, default=int(os.environ.get('WORLD_SIZE', 1)))
    ap.add_argument('--steps', type=int, default=5)
    ap.add_argument('--warmup', type=int, default=3)
    ap.add_argument('--impl', default='b200', choices=['b200', 'reference'])
    ap.add_argument('--config', type=int, default=3, choices=[1, 2, 3, 4, 5])
    ap.add_argument('--sites', type=int, default=None, help='override the site count (smaller runs)')
    ap.add_argument('--width', type=int, default=None)
    ap.add_argument('--height', type=int, default=None)
    ap.add_argument('--cpu-sample', type=int, default=None, help='rays of the CPU baseline sample')
    ap.add_argument('--no-baselines', action='store_true', help='skip the CPU and reference-CUDA baselines')
    ap.add_argument('--strong', action='store_true',
                    help='strong scaling: one frame (default 3840x2160) whose 16x16 tiles are dealt over the GPUs')
    ap.add_argument('--field', action='store_true',
                    help='the NeRF-sampler field kernels (walk, density, colour) on the config-2 scene')
    return ap.parse_args()


# ------------------------------------------------------------------------------------------ setup

def scene_config(cfg):
    """Configuration whose graph a workload renders: config 5 marches through config 2's scene."""
    return 2 if cfg == 5 else cfg


def load_scene(cfg, n_sites, rank, poll_s=2.0, wait_s=3600.0):
    """Graph of the configuration, built once by rank 0 and cached on disk; the other ranks wait for the
    cache. If rank 0 fails to build it, it leaves a marker (named for this launch, so that one left by an
    earlier launch is never read) and the waiting ranks raise at their next poll instead of waiting."""
    from voronoi_gauss_b200 import scenes
    cfg = scene_config(cfg)
    n = scenes.CONFIGS[cfg]['n'] if n_sites is None else n_sites
    path = os.path.join(scenes.cache_dir(), f'graph_c{cfg}_n{n}_s0.npz')
    launch = os.environ.get('TORCHELASTIC_RUN_ID') or os.environ.get('MASTER_PORT') or 'single'
    failed = f'{path}.failed.{launch}'
    if rank == 0:
        try:
            return scenes.build_graph(cfg, n=n)
        except BaseException as e:
            with open(failed, 'w') as f:
                f.write(f'{type(e).__name__}: {e}')
            raise
    t0 = time.time()
    while not os.path.exists(path):
        if os.path.exists(failed):
            with open(failed) as f:
                raise RuntimeError(f'rank 0 could not build the scene ({f.read()})')
        if time.time() - t0 > wait_s:
            raise TimeoutError('scene cache was not written by rank 0')
        time.sleep(poll_s)
    return scenes.build_graph(cfg, n=n)


POOL_VIEWS = 8  # orbit views of the training workload's pool (dist.pool_tile_pixels)


def pool_rays(cfg, gr, W, H, rank):
    """The training workload's rays for `rank`: of each of POOL_VIEWS orbit views (radius 3), the 16x16
    tiles t = rank + v mod POOL_VIEWS, i.e. one W x H frame's worth of rays drawn evenly from the pool, the
    same share at every world size. -> o, d (B, 3), start (B) int32 (each view's nearest site to its
    camera), on the host."""
    from voronoi_gauss_b200 import dist as vdist
    from voronoi_gauss_b200 import scenes, sites
    o_l, d_l, s_l = [], [], []
    for v, pix in enumerate(vdist.pool_tile_pixels(H, W, rank, POOL_VIEWS)):
        centre, c2w = scenes.orbit_camera(v, POOL_VIEWS)
        o_v, d_v = scenes.camera_rays(centre, c2w, W, H, scenes.CONFIGS[cfg]['fov'])
        pix = torch.from_numpy(pix)
        o_l.append(o_v[pix]), d_l.append(d_v[pix])
        s_l.append(torch.full((len(pix),), int(sites.nearest_sites(gr['points'], centre[None])[0]),
                              dtype=torch.int32))
    return torch.cat(o_l).contiguous(), torch.cat(d_l).contiguous(), torch.cat(s_l).contiguous()


def camera(cfg, view, W, H, n_views=8):
    """Orbit camera `view` of n_views; rays in 4x8 pixel-tile order on the host."""
    from voronoi_gauss_b200 import scenes
    centre, c2w = scenes.orbit_camera(view, n_views)
    order = scenes.tile_order(H, W)
    o, d = scenes.camera_rays(centre, c2w, W, H, scenes.CONFIGS[cfg]['fov'], order=order)
    return centre, o, d


def clocks_start():
    try:
        return subprocess.Popen(
            ['nvidia-smi', '--query-gpu=index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,'
             'clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,'
             'clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap', '--format=csv,noheader',
             '-lms', '200'], stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
    except OSError:
        return None


def clocks_stop(proc, gpu_index):
    if proc is None:
        return None
    proc.terminate()
    try:
        out, _ = proc.communicate(timeout=10)
    except subprocess.TimeoutExpired:
        proc.kill()
        out, _ = proc.communicate()
    sm, mx, reasons = [], [], set()
    names = ['hw_slowdown', 'hw_thermal_slowdown', 'sw_thermal_slowdown', 'sw_power_cap']
    for line in out.strip().splitlines():
        f = [x.strip() for x in line.split(',')]
        if len(f) < 9 or f[0] != str(gpu_index):
            continue
        try:
            sm.append(float(f[1].split()[0]))
            mx.append(float(f[2].split()[0]))
        except ValueError:
            continue
        for name, v in zip(names, f[5:9]):
            if v.lower() == 'active':
                reasons.add(name)
    if not sm:
        return None
    return {'sm_mhz': statistics.median(sm), 'sm_max_mhz': max(mx), 'reasons': sorted(reasons), 'samples': len(sm)}


def measured_peak():
    path = os.path.join(ROOT, 'MEASURED_PEAKS.json')
    if os.path.exists(path):
        with open(path) as f:
            return float(json.load(f)['hbm_gbs']), 'measured'
    return 6650.0, 'fallback'


def dram_traffic(kernel, units):
    """DRAM bytes (read + write) of one launch of `kernel` processing `units` work units, scaled from a
    small one-kernel ncu capture (profiles/dram_traffic.json: bytes per unit, measured on a case larger
    than L2); None when no capture of that kernel is recorded."""
    path = os.path.join(ROOT, 'profiles', 'dram_traffic.json')
    if not os.path.exists(path):
        return None, None
    with open(path) as f:
        tab = json.load(f)
    k = tab.get(kernel)
    if not k:
        return None, None
    return float(k['dram_bytes_per_unit']) * units, k['source']


class KernelTimer:
    """Device time of the library's kernel classes inside a timed region (vg_prof_* of the C ABI)."""

    def __init__(self, kernels):
        from voronoi_gauss_b200 import _lib
        self._lib, self.kernels = _lib, kernels

    def __enter__(self):
        self._lib.prof_enable(True)
        return self

    def __exit__(self, *exc):
        self._lib.prof_enable(False)

    def read(self):
        return {k: self._lib.prof_read(k) for k in self.kernels}


# ----------------------------------------------------------------------------------- algorithmic bytes

def _pass_chunks(cells, deg, n_sites):
    """Chunks of at most CM_CHUNK samples per cell for the sample cells of one pass, and their summed
    neighbourhood sizes: -> (chunks, sum over chunks of deg(cell) + 1)."""
    if cells.numel() == 0:
        return 0, 0
    cnt = torch.bincount(cells, minlength=n_sites)
    ch = (cnt + CM_CHUNK - 1) // CM_CHUNK
    return int(ch.sum()), int((ch * (deg + 1)).sum())


def training_units(stats, rec, offsets, K):
    """Work units of the training step's kernels, counted from one recorded forward (rec after the colour
    pass: field 7 > 0 marks the samples that carry a colour): per pass of CM_SLOTS record slots, the
    chunks of the colour pass (coloured samples) and of the scatter (every sample of the fully recorded
    rays), with their neighbourhood sizes."""
    B = stats.size(0)
    n_sites = offsets.numel() - 1
    deg = (offsets[1:] - offsets[:-1]).long()
    rays_pass = max(1, min(B, CM_SLOTS // K))
    u = dict(col_chunks=0, col_nbr=0, col_samples=0, sc_chunks=0, sc_nbr=0, sc_samples=0, cell_n=0.0)
    n_sum, s_sum = 0.0, 0
    for r0 in range(0, B, rays_pass):
        st = stats[r0:r0 + rays_pass]
        rc = rec[r0:r0 + rays_pass]
        fits = st[:, 0] <= K
        valid = (torch.arange(K, device=rec.device)[None, :] < st[:, :1]) & fits[:, None]
        cells = rc[..., 1].view(torch.int32)[valid].long()
        a, b = _pass_chunks(cells, deg, n_sites)
        u['sc_chunks'] += a
        u['sc_nbr'] += b
        u['sc_samples'] += cells.numel()
        n_sum += float((deg[cells] + 1).double().sum())
        s_sum += cells.numel()
        col = valid & (rc[..., 7] > 0)
        cells = rc[..., 1].view(torch.int32)[col].long()
        a, b = _pass_chunks(cells, deg, n_sites)
        u['col_chunks'] += a
        u['col_nbr'] += b
        u['col_samples'] += cells.numel()
    u['cell_n'] = n_sum / max(s_sum, 1)
    return u


def algorithmic_bytes_training(stats, units, nb, K):
    """Algorithmic bytes per step of the training kernels, counted on the reference's fp32 layout (a site
    record = index 4 + position 12 + raw 4 + density conic 24 + colour conic 24 + SH 12 nb bytes; its
    gradient = 13 + 3 nb floats):
      traversal  sum_r [44 n S_r + 16 n W_r + 68] + 32 per recorded sample (the record written)
      colour     per (chunk, neighbour site) of the colour pass: index + position + colour conic + SH
                 (40 + 12 nb); per coloured sample: its record read and written (64) and its ray (24)
      replay     per recorded sample: record read (32) + item written (64); per ray 44 (rgb, T, gradients)
      scatter    per (chunk, neighbour site): the site record (68 + 12 nb) and its gradient read and
                 written (2 x 4 (13 + 3 nb)); per sample: its 64-byte item
    with S, W samples and walk steps per ray, n the mean neighbourhood size of the visited cells."""
    st = stats.double()
    S, W = float(st[:, 0].sum()), float(st[:, 2].sum())
    B = stats.size(0)
    recorded = float(st[:, 0].clamp(max=K).sum())
    n = units['cell_n']
    return {
        'traversal': 44 * n * S + 16 * n * W + 68 * B + 32 * recorded,
        'color': (40 + 12 * nb) * units['col_nbr'] + 88 * units['col_samples'],
        'replay': 96 * units['sc_samples'] + 44 * B,
        'scatter': (68 + 12 * nb + 8 * (13 + 3 * nb)) * units['sc_nbr'] + 64 * units['sc_samples'],
    }


def training_unit_counts(units):
    """Work units per kernel class (for scaling a small capture's DRAM bytes to a full launch)."""
    return {'scatter': units['sc_nbr'], 'color': units['col_nbr'], 'replay': units['sc_samples']}


def launches_per_step(n_rays, record_cap):
    """libvgb200 kernels launched by one training step (the CUB scans compiled into the library count
    as two kernels each): 2 conics; forward: field pack, deferred traversal, overflow rays, per pass of
    at most 2^26 record slots (scan, bucket, chunks, colour), composite; backward: field pack, re-traced
    rays, per pass (count, scan, bucketed items, chunks, scatter), gradient unpack; 2 conic backwards."""
    passes = math.ceil(n_rays / max(1, CM_SLOTS // record_cap))
    forward = 3 + passes * (2 + 3) + 1
    backward = 2 + passes * (1 + 2 + 3) + 1
    return 2 + forward + backward + 2


def roofline(times, nbytes, steps, peak, peak_kind, units=None, note=None):
    """Roofline object of the dominant kernel class (largest device time in the timed region)."""
    dom = max(times, key=lambda k: times[k][0])
    ms, launches = times[dom]
    per_launch_ms = ms / max(launches, 1)
    launches_per_step = launches / steps
    per_launch_bytes = nbytes[dom] / max(launches_per_step, 1e-9)
    achieved = per_launch_bytes / (per_launch_ms * 1e-3) / 1e9
    out = {'bound': 'hbm', 'kernel': dom, 'achieved': round(achieved, 1), 'peak': peak, 'unit': 'GB/s',
           'frac': round(achieved / peak, 4), 'traffic': None, 'peak_kind': f'{peak_kind} (HBM copy)',
           'kernel_ms_per_launch': round(per_launch_ms, 4), 'launches_per_step': round(launches_per_step, 2),
           'algorithmic_bytes_per_launch': per_launch_bytes,
           'kernel_ms_per_step': {k: round(v[0] / steps, 3) for k, v in times.items()}}
    if units is not None and dom in units:
        traffic, source = dram_traffic(dom, units[dom] / max(launches_per_step, 1e-9))
        if traffic is not None:
            out['traffic'] = traffic
            out['traffic_source'] = source
            out['dram_gbs'] = round(traffic / (per_launch_ms * 1e-3) / 1e9, 1)
    if note:
        out['note'] = note
    return out


# --------------------------------------------------------------------------------------- training arm

def run_training(args):
    import torch.distributed as dist

    from voronoi_gauss_b200 import dist as vdist
    from voronoi_gauss_b200 import ext, render, scenes, sites
    from voronoi_gauss_b200.model import VoronoiGaussField

    world = int(os.environ.get('WORLD_SIZE', 1))
    rank = int(os.environ.get('RANK', 0))
    local = int(os.environ.get('LOCAL_RANK', 0))
    cfgd = scenes.CONFIGS[args.config]
    W = args.width or (3840 if args.strong else cfgd['W'])
    H = args.height or (2160 if args.strong else cfgd['H'])
    gr = load_scene(args.config, args.sites, rank)
    if world > 1:
        import datetime
        dist.init_process_group('nccl', timeout=datetime.timedelta(seconds=600), device_id=torch.device('cuda', local))
    torch.cuda.set_device(local)
    dev = torch.device('cuda', local)
    prm = scenes.make_params(args.config, gr['points'].astype(np.float64))
    if args.strong:
        # one frame, its 16x16 tiles dealt round-robin over the ranks (dist.tile_pixels)
        centre, c2w = scenes.orbit_camera(0, 8)
        o_v, d_v = scenes.camera_rays(centre, c2w, W, H, cfgd['fov'])
        pix = torch.from_numpy(vdist.tile_pixels(H, W, world, rank))
        o_h, d_h = o_v[pix].contiguous(), d_v[pix].contiguous()
        start_h = torch.full((len(o_h),), int(sites.nearest_sites(gr['points'], centre[None])[0]),
                             dtype=torch.int32)
    else:
        # one frame's worth of rays per GPU from a fixed pool of views: the same share at every world size
        if world > POOL_VIEWS:
            raise SystemExit(f'--gpus {world}: the weak-scaling workload deals a pool of {POOL_VIEWS} views')
        o_h, d_h, start_h = pool_rays(args.config, gr, W, H, rank)
    B = len(o_h)
    gen = torch.Generator().manual_seed(0)
    target_h = torch.rand(B, 3, generator=gen)

    points = torch.from_numpy(gr['points']).to(dev)
    offsets = torch.from_numpy(gr['offsets']).to(dev)
    adj = torch.from_numpy(gr['adj']).to(dev)
    prm_d = {k: (v.to(dev) if torch.is_tensor(v) else v) for k, v in prm.items()}
    model = VoronoiGaussField.from_params(points, offsets, adj, prm_d)
    opt = torch.optim.Adam(model.param_groups(LR), eps=1e-15, fused=True)
    params = [p for p in model.parameters()]
    nb = (model.sh_deg + 1) ** 2

    o, d = o_h.to(dev), d_h.to(dev)
    start = start_h.to(dev)
    target = target_h.to(dev)
    last = {}

    def foam_step(o, d, start, target):
        opt.zero_grad(set_to_none=True)
        near, _, far = render.ray_bounds(o, d, 0.02, 4.0)
        dA = ext.conic(model.d_log_scale, model.d_quat)
        cA = ext.conic(model.c_log_scale, model.c_quat)
        fg, T, _, stats = ext.foam(model.graph, model.raw, dA, cA, model.sh(), model.sh_deg, o, d, start, near, far,
                                   T_THRESH, W_THRESH, RECORD_CAP)
        background = torch.sigmoid(model.bg_logit)  # seen through what the rays leave unabsorbed
        loss = ((fg + T.unsqueeze(1) * background - target) ** 2).mean()
        loss.backward()
        if world > 1:
            vdist.allreduce_grads(params)
        opt.step()
        last['stats'] = stats
        return loss

    torch.cuda.synchronize()
    for _ in range(args.warmup):
        foam_step(o, d, start, target)
    torch.cuda.synchronize()
    if world > 1:
        dist.barrier()

    # ---- device-resident timed region (kernel classes timed by their own events on the launch stream)
    clk = clocks_start() if local == 0 else None
    time.sleep(0.3 if clk else 0)
    t0, t1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    kt = KernelTimer(['traversal', 'color', 'replay', 'scatter'])
    torch.cuda.synchronize()
    if world > 1:
        dist.barrier()
    with kt:
        t0.record()
        for _ in range(args.steps):
            foam_step(o, d, start, target)
        t1.record()
        torch.cuda.synchronize()
    if world > 1:
        dist.barrier()
    clocks = clocks_stop(clk, local) if clk else None
    ms = t0.elapsed_time(t1) / args.steps
    ktimes = kt.read()
    if world > 1:
        tt = torch.tensor([ms], device=dev)
        dist.all_reduce(tt, op=dist.ReduceOp.MAX)
        ms = float(tt)

    # ---- work units and algorithmic bytes of this workload, from one recorded forward
    with torch.no_grad():
        near, _, far = render.ray_bounds(o, d, 0.02, 4.0)
        dA = ext.conic(model.d_log_scale, model.d_quat)
        cA = ext.conic(model.c_log_scale, model.c_quat)
        _, _, _, stats, rec = ext.foam_extension().foam_forward(
            model.graph.points, model.graph.offsets, model.graph.adj, model.raw, dA, cA, model.sh(), model.sh_deg, o, d,
            start, near, far, T_THRESH, W_THRESH, RECORD_CAP)
        units = training_units(stats, rec, model.graph.offsets, RECORD_CAP)
        nbytes = algorithmic_bytes_training(stats, units, nb, RECORD_CAP)
        samples_per_ray = float(stats[:, 0].double().mean())
        del rec

    # ---- end to end: pinned host inputs in, loss out, every step
    o_p, d_p, t_p = o_h.pin_memory(), d_h.pin_memory(), target_h.pin_memory()
    s_p = start_h.pin_memory()
    loss_h = torch.empty((), dtype=torch.float32).pin_memory()
    h2d = o_p.numel() * 4 + d_p.numel() * 4 + t_p.numel() * 4 + s_p.numel() * 4
    torch.cuda.synchronize()
    if world > 1:
        dist.barrier()
    # the inputs of step i + 1 are copied on a side stream while step i computes (two device buffer sets)
    copy_stream = torch.cuda.Stream(dev)
    main_stream = torch.cuda.current_stream(dev)
    bufs = [[torch.empty_like(x, device=dev) for x in (o_p, d_p, s_p, t_p)] for _ in range(2)]
    copied = [torch.cuda.Event() for _ in range(2)]
    consumed = [torch.cuda.Event() for _ in range(2)]

    def upload(i):
        k = i % 2
        with torch.cuda.stream(copy_stream):
            copy_stream.wait_event(consumed[k])
            for dst, src in zip(bufs[k], (o_p, d_p, s_p, t_p)):
                dst.copy_(src, non_blocking=True)
            copied[k].record(copy_stream)

    for ev in consumed:
        ev.record(main_stream)
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record()
    upload(0)
    for i in range(args.steps):
        if i + 1 < args.steps:
            upload(i + 1)
        k = i % 2
        main_stream.wait_event(copied[k])
        oo, dd, ss, tt_ = bufs[k]
        loss = foam_step(oo, dd, ss, tt_)
        consumed[k].record(main_stream)
        loss_h.copy_(loss.detach(), non_blocking=True)
    e1.record()
    torch.cuda.synchronize()
    e2e_ms = e0.elapsed_time(e1) / args.steps
    if world > 1:
        tt = torch.tensor([e2e_ms], device=dev)
        dist.all_reduce(tt, op=dist.ReduceOp.MAX)
        e2e_ms = float(tt)

    rays_total = W * H if args.strong else B * world
    value = rays_total / (ms * 1e-3) / 1e6
    peak, peak_kind = measured_peak()
    step_kernel_ms = sum(v[0] for v in ktimes.values()) / args.steps
    line = {
        'metric': (f'training Mrays/s (fwd+bwd+Adam), one {W}x{H} frame tile-sharded over the GPUs, '
                   f'{len(gr["points"])} sites' if args.strong else
                   f'training Mrays/s (fwd+bwd+Adam) @{W}x{H}, {len(gr["points"])} sites'),
        'value': round(value, 3), 'unit': 'Mrays/s',
        'n_gpus': world, 'steps': args.steps, 'warmup': args.warmup, 'ms_per_step': round(ms, 3),
        'higher_is_better': True, 'scaling': 'strong' if args.strong else 'weak', 'vs_baseline': None, 'dtype': 'f32',
        'data': 'synthetic',
        'config': {'workload': f'config{args.config}: {len(gr["points"])} sites ({cfgd["kind"]}), SH deg '
                               f'{model.sh_deg}, {W}x{H} rays per GPU, training step (fwd+bwd+Adam), record_cap '
                               f'{RECORD_CAP}, t/w_thresh {T_THRESH:g}' + ('' if args.strong else
                               f'; each GPU renders the 16x16 tiles t = rank + v mod {POOL_VIEWS} of orbit views '
                               f'v = 0..{POOL_VIEWS - 1} (one {W}x{H} frame of rays, the same share at every N)'),
                   'rays_per_gpu': B, 'sites': len(gr['points']),
                   'parallelism': f'dp{world} (each GPU its own share of the view pool, NCCL all-reduce of site '
                                  'gradients)' if world > 1 else 'single GPU',
                   'l2': 'inputs larger than L2 (scene records + adjacency ~1 GB read every step)'},
        'fps': round(1000.0 / ms, 3), 'samples_per_ray': round(samples_per_ray, 2),
        'roofline': roofline(ktimes, nbytes, args.steps, peak, peak_kind, training_unit_counts(units),
                             note='dominant kernel class timed by its own CUDA events inside the timed region; '
                                  'algorithmic bytes counted per (chunk, neighbour site) of the cell-major passes '
                                  '(each chunk loads its neighbourhood once), reference fp32 layout'),
        'work_units': units,
        'e2e': {'value': round(rays_total / (e2e_ms * 1e-3) / 1e6, 3), 'unit': 'Mrays/s', 'ms_per_step':
                round(e2e_ms, 3), 'h2d_bytes_per_step': h2d, 'd2h_bytes_per_step': 4,
                'copies': 'rays, start sites and target from pinned host memory every step, the next step\'s on a '
                          'side stream while the current one computes; the loss read back every step'},
        'gpu_launches': launches_per_step(B, RECORD_CAP) * args.steps,
        'clocks': clocks,
    }
    line['roofline']['timed_kernels_ms_per_step'] = round(step_kernel_ms, 3)
    if os.environ.get('VG_LIB_PATH'):  # a variant build of the library: name it and its knobs
        from voronoi_gauss_b200 import _lib
        knobs = os.path.join(os.path.dirname(_lib.LIB_PATH), 'defines.txt')
        line['config']['library'] = {'path': _lib.LIB_PATH, 'defines': open(knobs).read().split()
                                     if os.path.exists(knobs) else []}
    if rank == 0 and world == 1 and not args.no_baselines:
        line['cpu_baseline'] = cpu_baseline(gr, prm, o_h, d_h, start_h, args)
        line['ref_cuda'] = ref_cuda_training(model, o, d, start, args)
    if world > 1:
        dist.destroy_process_group()
    if rank == 0:
        print(json.dumps(line), flush=True)


def time_reps(fn, reps=REF_REPS):
    """bench_vs_radfoam.time_ms protocol (bench_vs_radfoam.py:26-36): one warm-up call, then a CUDA event
    pair around `reps` calls -> ms per call."""
    fn()
    torch.cuda.synchronize()
    a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    a.record()
    for _ in range(reps):
        fn()
    b.record()
    torch.cuda.synchronize()
    return a.elapsed_time(b) / reps


def ref_cuda_training(model, o, d, start, args):
    """The reference's own CUDA kernels (built unchanged from its sources into oracle/_ref) on the same
    workload: foam_forward with records, then foam_backward, each timed over REF_REPS calls."""
    from oracle import ref_build
    if not ref_build.available('vgf_foam'):
        return {'unavailable': 'oracle/_ref/vgf_foam not built'}
    from voronoi_gauss_b200 import ext, render
    rf = ref_build.load_reference('vgf_foam')
    with torch.no_grad():
        near, _, far = render.ray_bounds(o, d, 0.02, 4.0)
        dA = ext.conic(model.d_log_scale, model.d_quat)
        cA = ext.conic(model.c_log_scale, model.c_quat)
        sh = model.sh().contiguous()
        g = model.graph
        B = o.size(0)
        args_ = (g.points, g.offsets, g.adj, model.raw.detach(), dA, cA, sh, model.sh_deg, o, d, start, near, far,
                 T_THRESH, W_THRESH)
        f_ms = time_reps(lambda: rf.foam_forward(*args_, RECORD_CAP))
        out = rf.foam_forward(*args_, RECORD_CAP)
        rgb, T, _, stats, rec = out
        gr, gT = torch.ones_like(rgb), torch.ones_like(T)
        b_ms = time_reps(lambda: rf.foam_backward(*args_, rgb, T, gr, gT, rec, stats))
        del out, rec
        return {'kind': 'reference CUDA kernels (foam.cu, built unchanged for sm_100a)', 'reps': REF_REPS,
                'fwd_ms': round(f_ms, 3), 'bwd_ms': round(b_ms, 3), 'fwd_mrays_s': round(B / (f_ms * 1e-3) / 1e6, 3),
                'fwd_bwd_mrays_s': round(B / ((f_ms + b_ms) * 1e-3) / 1e6, 3)}


def cpu_baseline(gr, prm, o_h, d_h, start_h, args, seconds=10.0, max_chunks=64):
    """The CPU restatement of the path (oracle/, all host threads) on a bounded sample of the workload:
    chunks of rays drawn without replacement from the view (seeded), each timed through the forward with
    records and the backward, until `seconds` of CPU work have been spent (or `max_chunks` chunks); host
    memory stays at one chunk's records. The conics come from the oracle too (host only)."""
    from oracle import oracle
    from voronoi_gauss_b200 import render
    chunk = args.cpu_sample or 16384
    B = o_h.size(0)
    chunk = min(chunk, B)
    order = torch.from_numpy(np.random.default_rng(1).permutation(B))
    dA = oracle.conic_forward(prm['d_log_scale'], prm['d_quat'])
    cA = oracle.conic_forward(prm['c_log_scale'], prm['c_quat'])
    threads = os.cpu_count() or 1
    rays, fwd_s, bwd_s, k = 0, 0.0, 0.0, 0
    while fwd_s + bwd_s < seconds and k < max_chunks and (k + 1) * chunk <= B:
        sel = torch.sort(order[k * chunk:(k + 1) * chunk])[0]
        o, d = o_h[sel].contiguous(), d_h[sel].contiguous()
        near, _, far = render.ray_bounds(o, d, 0.02, 4.0)
        start = start_h[sel].numpy()
        a = (gr['points'], gr['offsets'], gr['adj'], prm['raw'], dA, cA, prm['sh'], prm['sh_deg'], o, d, start, near,
             far, T_THRESH, W_THRESH)
        t0 = time.time()
        rgb, T, depth, stats, rec = oracle.foam_forward(*a, RECORD_CAP, n_threads=threads)
        t1 = time.time()
        oracle.foam_backward(*a, rgb, T, np.ones_like(rgb), np.ones_like(T), rec, stats, n_threads=threads)
        t2 = time.time()
        del rec
        rays, fwd_s, bwd_s, k = rays + chunk, fwd_s + t1 - t0, bwd_s + t2 - t1, k + 1
    return {'value': round(rays / (fwd_s + bwd_s) / 1e6, 6), 'unit': 'Mrays/s', 'cores': threads, 'kind': 'port',
            'sample': f'{k} chunks of {chunk} random rays of the view ({rays} rays), forward (records) + backward, '
                      f'{fwd_s + bwd_s:.1f} s of CPU time',
            'fwd_s': round(fwd_s, 3), 'bwd_s': round(bwd_s, 3)}


# -------------------------------------------------------------------------------------- inference arm

INFER_MODES = {
    # the reference's fast configuration (bench_infer.py:30-31): fused colours, fp16 SH, eps 1e-4, tiles, Morton
    'fused_fp16_eps': dict(pack=dict(sh_half=True, eps_density=1e-4, reorder=True), colors='fused', eps_color=1e-4),
    # exact colours, fp32, no skipping, tiles (bench_infer.py:20-21 with tiles)
    'exact_fp32': dict(pack=dict(), colors='exact', eps_color=0.0),
}


def algorithmic_bytes_infer(stats, nb, half):
    """Algorithmic bytes of one inference frame on the packed layout: per sample its cell's edge run
    (20 bytes per neighbour: the edge record and the site id), per density term evaluated the site's
    density conic and raw (32), per SH evaluation the site's coefficients (6 nb bytes in fp16, 12 nb in
    fp32) and colour conic (32); per walk step an edge run; per ray 68 bytes of ray I/O. Neighbourhood
    sizes are those of the visited cells (n, measured)."""
    st = stats.double()
    S, W, dens, sh = (float(st[:, i].sum()) for i in (0, 2, 3, 4))
    return S, W, dens, sh, (6 if half else 12) * nb


def run_infer(args):
    from oracle import ref_build
    from voronoi_gauss_b200 import render, scenes, sites
    from voronoi_gauss_b200.model import VoronoiGaussField

    torch.cuda.set_device(0)
    dev = torch.device('cuda', 0)
    cfgd = scenes.CONFIGS[2]
    W = args.width or cfgd['W']
    H = args.height or cfgd['H']
    gr = load_scene(2, args.sites, 0)
    prm = scenes.make_params(2, gr['points'].astype(np.float64))
    model = VoronoiGaussField.from_params(*(torch.from_numpy(gr[k]).to(dev) for k in ('points', 'offsets', 'adj')),
                                          {k: (v.to(dev) if torch.is_tensor(v) else v) for k, v in prm.items()})
    n_views = cfgd['n_cams']
    views = [(8 * i) % n_views for i in range(max(args.steps, 1))]
    rays = {}
    for v in sorted(set(views)):
        centre, c2w = scenes.orbit_camera(v, n_views)
        o, d = scenes.camera_rays_device(centre, c2w, W, H, cfgd['fov'], device=dev, tile=(4, 8))
        s = int(sites.nearest_sites(gr['points'], centre[None])[0])
        rays[v] = (o, d, torch.full((W * H,), s, dtype=torch.int32, device=dev))
    B = W * H
    nb = (model.sh_deg + 1) ** 2
    rf = ref_build.load_reference('vgf_foam_infer') if (ref_build.available('vgf_foam_infer')
                                                         and not args.no_baselines) else None
    peak, peak_kind = measured_peak()
    results = {}
    for name, mode in INFER_MODES.items():
        pack = render.pack_foam(model, **mode['pack'])
        kw = dict(colors=mode['colors'], eps_color=mode['eps_color'], t_thresh=T_THRESH, w_thresh=W_THRESH)

        def frame(v, impl='b200'):
            o, d, s = rays[v]
            if impl == 'b200':
                return render.render_rays_foam_infer(model, pack, o, d, s, **kw)
            if impl == 'per_ray':
                return render.render_rays_foam_infer(model, pack, o, d, s, exact_stats=True, **kw)
            return reference_infer(rf, model, pack, o, d, s, **kw)

        for _ in range(args.warmup):
            frame(views[0])
        torch.cuda.synchronize()
        kt = KernelTimer(['infer', 'infer_color'])
        t0, t1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        with kt:
            t0.record()
            for v in views:
                frame(v)
            t1.record()
            torch.cuda.synchronize()
        ms = t0.elapsed_time(t1) / len(views)
        out = frame(views[0])
        entry = {'ms': round(ms, 3), 'fps': round(1000 / ms, 2), 'mrays_s': round(B / (ms * 1e-3) / 1e6, 2),
                 'samples_per_ray': round(float(out['stats'][:, 0].double().mean()), 2)}
        times = kt.read()
        k_ms = times['infer'][0] / len(views)
        S, Wk, dens, sh, shb = algorithmic_bytes_infer(out['stats'], nb, mode['pack'].get('sh_half', False))
        off = pack['offsets']
        n_bar = float(((off[1:] - off[:-1]).double()).mean())
        # the traversal of the deferred pipeline reads edge runs and density rows only (no colours)
        nbytes = 20 * n_bar * (S + Wk) + 32 * dens + 68 * B
        entry['trace_ms'] = round(k_ms, 3)
        entry['colour_ms'] = round(times['infer_color'][0] / len(views), 3)
        entry['trace_achieved_gbs'] = round(nbytes / (k_ms * 1e-3) / 1e9, 1)
        entry['per_ray_ms'] = round(statistics.mean(time_reps(lambda v=v: frame(v, 'per_ray')) for v in views[:2]), 3)
        per_ray = frame(views[0], 'per_ray')
        entry['identical_to_per_ray'] = bool(torch.equal(out['rgb'], per_ray['rgb']))
        if rf is not None:
            ref_ms = statistics.mean(time_reps(lambda v=v: frame(v, 'reference')) for v in views[:2])
            ref_out = frame(views[0], 'reference')
            entry['reference_ms'] = round(ref_ms, 3)
            entry['reference_mrays_s'] = round(B / (ref_ms * 1e-3) / 1e6, 2)
            entry['speedup_vs_reference'] = round(ref_ms / ms, 3)
            entry['max_abs_rgb_vs_reference'] = float((out['rgb'] - ref_out['rgb']).abs().max())
        if name == 'fused_fp16_eps':
            # the reference's stage ablation (bench_infer.py:60-67): every ray's traversal fixed to the full
            # renderer's samples (cap), then exit faces only (stage 0) and exit faces + density (stage 1)
            cap = out['stats'][:, 0].int().contiguous()
            abl = {}
            for stage in (0, 1):
                skw = dict(kw, stage=stage, cap=cap)
                o0, d0, s0 = rays[views[0]]
                abl[f'stage{stage}_ms'] = round(time_reps(lambda: render.render_rays_foam_infer(
                    model, pack, o0, d0, s0, **skw)), 3)
                if rf is not None:
                    abl[f'reference_stage{stage}_ms'] = round(time_reps(lambda: reference_infer(
                        rf, model, pack, o0, d0, s0, **skw)), 3)
            entry['ablation_view0'] = abl
        results[name] = entry
        del pack
    head = results['fused_fp16_eps']
    # end to end: the frame's rays from pinned host memory in, the image back to pinned host memory
    pack = render.pack_foam(model, **INFER_MODES['fused_fp16_eps']['pack'])
    kw = dict(colors='fused', eps_color=1e-4, t_thresh=T_THRESH, w_thresh=W_THRESH)
    host = {v: tuple(x.cpu().pin_memory() for x in rays[v]) for v in set(views)}
    img = torch.empty(B, 3).pin_memory()
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record()
    for v in views:
        o, d, s = (x.to(dev, non_blocking=True) for x in host[v])
        img.copy_(render.render_rays_foam_infer(model, pack, o, d, s, **kw)['rgb'], non_blocking=True)
    e1.record()
    torch.cuda.synchronize()
    e2e_ms = e0.elapsed_time(e1) / len(views)
    line = {'metric': f'inference Mrays/s @{W}x{H}, {len(gr["points"])} sites (fused colours, fp16 SH, eps 1e-4, '
                      'tiles, Morton)', 'value': head['mrays_s'], 'unit': 'Mrays/s', 'n_gpus': 1,
            'steps': len(views), 'warmup': args.warmup, 'ms_per_step': head['ms'], 'higher_is_better': True,
            'scaling': 'weak', 'vs_baseline': None, 'dtype': 'f32 (fp16 SH storage)', 'data': 'synthetic',
            'config': {'workload': f'config2: {len(gr["points"])} sites (mixture), SH deg {model.sh_deg}, {W}x{H} '
                                   f'views {sorted(set(views))} of {n_views} orbit cameras, forward only',
                       'l2': 'scene larger than L2 (1M sites: ~0.5 GB of packed records read per frame)'},
            'fps': head['fps'], 'modes': results,
            'roofline': {'bound': 'hbm', 'kernel': 'trace (deferred inference)', 'achieved': head['trace_achieved_gbs'],
                         'peak': peak, 'unit': 'GB/s', 'frac': round(head['trace_achieved_gbs'] / peak, 4),
                         'traffic': None, 'peak_kind': peak_kind,
                         'note': 'algorithmic bytes per ray on the packed layout (edge runs, density rows); warps '
                                 'of a pixel tile share cells, so gathers are served from L1/L2'},
            'e2e': {'value': round(B / (e2e_ms * 1e-3) / 1e6, 2), 'unit': 'Mrays/s', 'ms_per_step': round(e2e_ms, 3),
                    'h2d_bytes_per_step': B * 28, 'd2h_bytes_per_step': B * 12},
            'gpu_launches': len(views)}
    print(json.dumps(line), flush=True)


def reference_infer(rf, model, pack, o, d, start, colors='exact', eps_color=0.0, t_thresh=1e-4, w_thresh=1e-4,
                    stage=2, cap=None):
    """render.render_rays_foam_infer through the reference's own foam_infer kernel (oracle/_ref)."""
    from voronoi_gauss_b200 import render
    mode = {'exact': 0, 'baked': 1, 'fused': 2}[colors]
    t_near, _, t_far = render.ray_bounds(o, d, 0.02, 4.0)
    if pack['inv'] is not None:
        start = pack['inv'][start.long()].int()
    cut = 2 * math.log(1 / eps_color) if eps_color > 0 else float('inf')
    if cap is None:
        cap = torch.empty(0, dtype=torch.int32, device=o.device)
    fg, T, depth, stats = rf.foam_infer(*(pack[k] for k in ('points', 'offsets', 'nbr', 'edge', 'attr', 'sh')),
                                        model.sh_deg, o, d, start, t_near.contiguous(), t_far.contiguous(),
                                        float(t_thresh), float(w_thresh), cut, mode, int(stage), cap, pack['orig'])
    return {'rgb': fg + T.unsqueeze(1) * torch.sigmoid(model.bg_logit), 'stats': stats}


# ----------------------------------------------------------------------------------------- march arm

MARCH_DT = 2.0 / 256


def run_march(args):
    from oracle import ref_build
    from voronoi_gauss_b200 import ext, scenes, sites
    from voronoi_gauss_b200.model import VoronoiGaussField

    torch.cuda.set_device(0)
    dev = torch.device('cuda', 0)
    cfgd = scenes.CONFIGS[5]
    W = args.width or cfgd['W']
    H = args.height or cfgd['H']
    gr = load_scene(5, args.sites, 0)
    prm = scenes.make_params(5, gr['points'].astype(np.float64))
    model = VoronoiGaussField.from_params(*(torch.from_numpy(gr[k]).to(dev) for k in ('points', 'offsets', 'adj')),
                                          {k: (v.to(dev) if torch.is_tensor(v) else v) for k, v in prm.items()})
    opt = torch.optim.Adam(model.param_groups(LR), eps=1e-15, fused=True)
    centre, o_h, d_h = camera(5, 0, W, H)
    o, d = o_h.to(dev), d_h.to(dev)
    start = torch.full((W * H,), int(sites.nearest_sites(gr['points'], centre[None])[0]), dtype=torch.int32,
                       device=dev)
    near, mid, far = scenes.march_bounds(o, d)
    target = torch.rand(W * H, 3, generator=torch.Generator().manual_seed(0)).to(dev)
    floor = 0.5 * MARCH_DT
    B = W * H

    def step():
        opt.zero_grad(set_to_none=True)
        dA = ext.conic(model.d_log_scale, model.d_quat, floor)
        cA = ext.conic(model.c_log_scale, model.c_quat, floor)
        fg, T, _, stats = ext.march(model.graph, model.raw, dA, cA, model.sh(), model.sh_deg, o, d, start, near, mid,
                                    far, MARCH_DT, 0, T_THRESH, W_THRESH)
        loss = ((fg + T.unsqueeze(1) * torch.sigmoid(model.bg_logit) - target) ** 2).mean()
        loss.backward()
        opt.step()
        return stats

    for _ in range(args.warmup):
        step()
    torch.cuda.synchronize()
    kt = KernelTimer(['march_fwd', 'march_items', 'scatter'])
    t0, t1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    clk = clocks_start()
    time.sleep(0.3 if clk else 0)
    with kt:
        t0.record()
        for _ in range(args.steps):
            stats = step()
        t1.record()
        torch.cuda.synchronize()
    clocks = clocks_stop(clk, 0) if clk else None
    ms = t0.elapsed_time(t1) / args.steps
    times = kt.read()
    st = stats.double()
    S, Wk = float(st[:, 0].sum()), float(st[:, 2].sum())
    off = model.graph.offsets
    n_bar = float(((off[1:] - off[:-1]).double() + 1).mean())
    nb = (model.sh_deg + 1) ** 2
    C = float(st[:, 1].sum())
    fwd_bytes = 44 * n_bar * S + (24 + 12 * nb) * n_bar * C + 16 * n_bar * Wk + 68 * B
    peak, peak_kind = measured_peak()
    f_ms = times['march_fwd'][0] / max(times['march_fwd'][1], 1)
    line = {'metric': f'march training Mrays/s (fwd+bwd+Adam) @{W}x{H}, dt 2/256, {len(gr["points"])} sites',
            'value': round(B / (ms * 1e-3) / 1e6, 3), 'unit': 'Mrays/s', 'n_gpus': 1, 'steps': args.steps,
            'warmup': args.warmup, 'ms_per_step': round(ms, 3), 'higher_is_better': True, 'scaling': 'weak',
            'vs_baseline': None, 'dtype': 'f32', 'data': 'synthetic',
            'config': {'workload': f'config5: {len(gr["points"])} sites (mixture), SH deg {model.sh_deg}, {W}x{H}, '
                                   'near/mid = unit-ball entry/exit, n_bg 0, dt 2/256 (<= 256 samples per ray)',
                       'l2': 'scene larger than L2'},
            'samples_per_ray': round(S / B, 2), 'walk_steps_per_sample': round(Wk / max(S, 1), 3),
            'kernel_ms_per_step': {k: round(v[0] / args.steps, 3) for k, v in times.items()},
            'roofline': {'bound': 'hbm', 'kernel': 'march_fwd', 'achieved': round(fwd_bytes / (f_ms * 1e-3) / 1e9, 1),
                         'peak': peak, 'unit': 'GB/s', 'frac': round(fwd_bytes / (f_ms * 1e-3) / 1e9 / peak, 4),
                         'traffic': None, 'peak_kind': peak_kind,
                         'note': 'forward formula of the reference fp32 layout with a walk per sample; gathers of a '
                                 'pixel tile are served from L1/L2'},
            'clocks': clocks, 'gpu_launches': None}
    if not args.no_baselines and ref_build.available('vgf_march'):
        rm = ref_build.load_reference('vgf_march')
        with torch.no_grad():
            dA = ext.conic(model.d_log_scale, model.d_quat, floor)
            cA = ext.conic(model.c_log_scale, model.c_quat, floor)
            a = (model.graph.points, model.graph.offsets, model.graph.adj, model.raw.detach(), dA, cA,
                 model.sh().contiguous(), model.sh_deg, o, d, start, near, mid, far, MARCH_DT, 0, T_THRESH, W_THRESH)
            rf_ms = time_reps(lambda: rm.march_forward(*a))
            rgb, T, _, _ = rm.march_forward(*a)
            g1, g2 = torch.ones_like(rgb), torch.ones_like(T)
            rb_ms = time_reps(lambda: rm.march_backward(*a, rgb, T, g1, g2))
        line['ref_cuda'] = {'kind': 'reference CUDA kernels (march.cu, built unchanged for sm_100a)', 'reps': REF_REPS,
                            'fwd_ms': round(rf_ms, 3), 'bwd_ms': round(rb_ms, 3),
                            'fwd_bwd_mrays_s': round(B / ((rf_ms + rb_ms) * 1e-3) / 1e6, 3)}
    print(json.dumps(line), flush=True)


# ----------------------------------------------------------------------------------------- field arm

FIELD_SAMPLES = 192  # samples per ray of the field workload (64 coarse + 2 x 64 proposal, render.py:77-106)


def run_field(args):
    """The NeRF-sampler field kernels (vgf.cu:438-533) on the config-2 scene: a 512x512 view of orbit camera 0,
    FIELD_SAMPLES sorted samples per ray (the midpoints of equal steps in the sampler's normalised
    coordinate, render.s_to_t), their nearest sites by walk, then density and colour forward and
    backward over every sample, each timed by itself (REF_REPS calls) beside the reference's kernels."""
    from oracle import ref_build
    from voronoi_gauss_b200 import ext, render, scenes, sites
    from voronoi_gauss_b200.model import VoronoiGaussField
    torch.cuda.set_device(0)
    dev = torch.device('cuda', 0)
    W = args.width or 512
    H = args.height or 512
    gr = load_scene(2, args.sites, 0)
    prm = scenes.make_params(2, gr['points'].astype(np.float64))
    model = VoronoiGaussField.from_params(*(torch.from_numpy(gr[k]).to(dev) for k in ('points', 'offsets', 'adj')),
                                          {k: (v.to(dev) if torch.is_tensor(v) else v) for k, v in prm.items()})
    centre, o_h, d_h = camera(2, 0, W, H)
    o, d = o_h.to(dev), d_h.to(dev)
    B = W * H
    start = torch.full((B,), int(sites.nearest_sites(gr['points'], centre[None])[0]), dtype=torch.int32, device=dev)
    bounds = render.ray_bounds(o, d, 0.02, 4.0)
    s = ((torch.arange(FIELD_SAMPLES, device=dev, dtype=torch.float32) + 0.5) / FIELD_SAMPLES).expand(B, -1)
    z = render.s_to_t(s.contiguous(), *bounds).contiguous()
    g = model.graph
    fx = ext.extension()
    site, _ = fx.walk(g.points, g.offsets, g.adj, o, d, z, start)
    x = (o[:, None, :] + z[..., None] * d[:, None, :]).reshape(-1, 3).contiguous()
    dirs = d[:, None, :].expand(B, FIELD_SAMPLES, 3).reshape(-1, 3).contiguous()
    site = site.reshape(-1).contiguous()
    M = x.size(0)
    gen = torch.Generator().manual_seed(0)
    g_sigma = torch.randn(M, generator=gen).to(dev)
    g_rgb = torch.randn(M, 3, generator=gen).to(dev)
    raw, dls, dq = model.raw.detach(), model.d_log_scale.detach(), model.d_quat.detach()
    cls, cq, sh = model.c_log_scale.detach(), model.c_quat.detach(), model.sh().detach().contiguous()
    rgb = fx.color_forward(g.points, g.offsets, g.adj, cls, cq, sh, model.sh_deg, x, dirs, site)

    def calls(m):
        return {
            'walk': lambda: m.walk(g.points, g.offsets, g.adj, o, d, z, start),
            'density_forward': lambda: m.density_forward(g.points, g.offsets, g.adj, raw, dls, dq, x, site, 1.0),
            'density_backward': lambda: m.density_backward(g.points, g.offsets, g.adj, raw, dls, dq, x, site, g_sigma),
            'color_forward': lambda: m.color_forward(g.points, g.offsets, g.adj, cls, cq, sh, model.sh_deg, x, dirs,
                                                     site),
            'color_backward': lambda: m.color_backward(g.points, g.offsets, g.adj, cls, cq, sh, model.sh_deg, x, dirs,
                                                       site, rgb, g_rgb),
        }
    mine = {k: round(time_reps(f), 3) for k, f in calls(fx).items()}
    total = sum(mine.values())
    line = {'metric': f'NeRF-sampler field kernels Msamples/s (walk + density fwd/bwd + colour fwd/bwd), {B} rays x '
                      f'{FIELD_SAMPLES} samples, {len(gr["points"])} sites', 'value': round(M / (total * 1e-3) / 1e6, 2),
            'unit': 'Msamples/s', 'n_gpus': 1, 'steps': REF_REPS, 'warmup': 1, 'ms_per_step': round(total, 3),
            'higher_is_better': True, 'scaling': 'weak', 'vs_baseline': None, 'dtype': 'f32', 'data': 'synthetic',
            'config': {'workload': f'config2 scene (mixture), {W}x{H} view of orbit camera 0, {FIELD_SAMPLES} sorted '
                                   'samples per ray (render.s_to_t midpoints), cell-major backwards'},
            'ms': mine}
    if not args.no_baselines and ref_build.available('vgf_ext'):
        ref = {k: round(time_reps(f), 3) for k, f in calls(ref_build.load_reference('vgf_ext')).items()}
        line['reference_ms'] = ref
        line['speedup_vs_reference'] = {k: round(ref[k] / mine[k], 2) for k in mine}
    print(json.dumps(line), flush=True)


# ---------------------------------------------------------------------------------- reference arm

def run_reference(args):
    """Reference arm: the reference path's CPU restatement (oracle/) on the host cores, bounded sample per
    step; rank 0 only."""
    rank = int(os.environ.get('RANK', 0))
    if rank != 0:
        return
    from oracle import oracle
    from voronoi_gauss_b200 import render, scenes, sites
    cfgd = scenes.CONFIGS[args.config]
    W = args.width or cfgd['W']
    H = args.height or cfgd['H']
    gr = load_scene(args.config, args.sites, 0)
    prm = scenes.make_params(args.config, gr['points'].astype(np.float64))
    o_h, d_h, start_h = pool_rays(args.config, gr, W, H, 0)
    # the site-parallel part of a step (conics of both Gaussians and their backward) runs once per full
    # view: timed once here and charged to each sample by its share of the view's rays
    t0 = time.time()
    dA = oracle.conic_forward(prm['d_log_scale'], prm['d_quat'])
    cA = oracle.conic_forward(prm['c_log_scale'], prm['c_quat'])
    zero = np.zeros((len(dA), 6), np.float32)
    oracle.conic_backward(prm['d_log_scale'], prm['d_quat'], 0.0, zero)
    oracle.conic_backward(prm['c_log_scale'], prm['c_quat'], 0.0, zero)
    conic_s = time.time() - t0
    n_rays = min(args.cpu_sample or 16384, W * H)
    B = o_h.size(0)
    threads = os.cpu_count() or 1
    rng = np.random.default_rng(0)
    times = []
    for step in range(args.warmup + args.steps):
        sel = torch.from_numpy(np.sort(rng.choice(B, n_rays, replace=False)))
        o, d = o_h[sel].contiguous(), d_h[sel].contiguous()
        near, _, far = render.ray_bounds(o, d, 0.02, 4.0)
        start = start_h[sel].numpy()
        a = (gr['points'], gr['offsets'], gr['adj'], prm['raw'], dA, cA, prm['sh'], prm['sh_deg'], o, d, start, near,
             far, T_THRESH, W_THRESH)
        t0 = time.time()
        rgb, T, depth, stats, rec = oracle.foam_forward(*a, RECORD_CAP, n_threads=threads)
        target = np.asarray(torch.rand(n_rays, 3, generator=torch.Generator().manual_seed(step)))
        g_rgb = (2.0 / (3 * n_rays)) * (rgb - target)
        oracle.foam_backward(*a, rgb, T, g_rgb, np.zeros_like(T), rec, stats, n_threads=threads)
        if step >= args.warmup:
            times.append(time.time() - t0 + conic_s * n_rays / B)
    ms = 1000 * statistics.mean(times)
    value = n_rays / (ms * 1e-3) / 1e6
    line = {'impl': 'reference', 'metric': f'training Mrays/s (fwd+bwd+Adam) @{W}x{H}, {len(gr["points"])} sites',
            'value': round(value, 6), 'unit': 'Mrays/s', 'n_gpus': int(os.environ.get('WORLD_SIZE', 1)),
            'steps': args.steps, 'warmup': args.warmup, 'ms_per_step': round(ms, 3), 'higher_is_better': True,
            'scaling': 'weak', 'vs_baseline': None, 'dtype': 'f32', 'data': 'synthetic',
            'config': {'workload': f'config{args.config}: {len(gr["points"])} sites, {W}x{H} view, training step, '
                                   f'bounded sample of {n_rays} rays per step on the host cores'},
            'cpu_baseline': {'value': round(value, 6), 'unit': 'Mrays/s', 'cores': threads, 'kind': 'port',
                             'sample': f'{n_rays} random rays of the {W}x{H} view per step, forward with records + '
                                       f'backward, plus {n_rays}/{B} of the conics forward + backward '
                                       f'({conic_s:.2f} s per view)'},
            'e2e': {'value': round(value, 6), 'unit': 'Mrays/s', 'h2d_bytes_per_step': 0, 'd2h_bytes_per_step': 0}}
    print(json.dumps(line), flush=True)


if __name__ == '__main__':
    a = parse()
    if a.impl == 'reference':
        run_reference(a)
    elif a.field:
        run_field(a)
    elif a.config == 2:
        run_infer(a)
    elif a.config == 5:
        run_march(a)
    else:
        run_training(a)
