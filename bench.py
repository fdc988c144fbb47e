"""Benchmark of the B200 Voronoi-Gaussian renderer (one JSON line on rank 0).

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl b200|reference] [--config 3]
    torchrun --nproc-per-node N bench.py --gpus N ...

A step is one training iteration of the interaction-point renderer on BASELINE config 3 (3M sites, 70 %
near a union of spheres, SH degree 3, one 1920x1080 view from an orbit camera of radius 3): conics of
both Gaussians, ext.foam forward with records, background composite and L2 loss against a seeded random
target, backward through foam and conics, and a fused Adam step. With N GPUs every rank renders its own
1080p view (weak scaling; camera = rank) and the per-site gradients are summed with one NCCL
all-reduce before Adam. Inputs (scene and the step's rays) are resident in HBM in the timed region of
`value`; `e2e` repeats the step with the rays and target copied from pinned host memory and the loss
read back every step. The scene (1 GB of site records and adjacency) is larger than L2, so no L2 flush
is needed between steps.

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


def parse():
    ap = argparse.ArgumentParser()
    ap.add_argument('--gpus', type=int, default=int(os.environ.get('WORLD_SIZE', 1)))
    ap.add_argument('--steps', type=int, default=5)
    ap.add_argument('--warmup', type=int, default=3)
    ap.add_argument('--impl', default='b200', choices=['b200', 'reference'])
    ap.add_argument('--config', type=int, default=3)
    ap.add_argument('--sites', type=int, default=None, help='override the site count (smaller runs)')
    ap.add_argument('--width', type=int, default=None)
    ap.add_argument('--height', type=int, default=None)
    ap.add_argument('--cpu-sample', type=int, default=None, help='rays of the CPU baseline sample')
    ap.add_argument('--no-baselines', action='store_true', help='skip the CPU and reference-CUDA baselines')
    ap.add_argument('--strong', action='store_true',
                    help='strong scaling: one frame (default 3840x2160) whose 16x16 tiles are dealt over the GPUs')
    return ap.parse_args()


# ------------------------------------------------------------------------------------------ setup

def load_scene(cfg, n_sites, rank, poll_s=2.0, wait_s=3600.0):
    """Graph of the configuration, built once by rank 0 and cached on disk; the other ranks wait for the
    cache. If rank 0 fails to build it, it leaves a marker (named for this launch, so that one left by an
    earlier launch is never read) and the waiting ranks raise at their next poll instead of waiting."""
    from voronoi_gauss_b200 import scenes
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


def camera(cfg, view, W, H, device):
    from voronoi_gauss_b200 import scenes
    centre, c2w = scenes.orbit_camera(view, 8)
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


# ----------------------------------------------------------------------------------- algorithmic bytes

def algorithmic_bytes(stats, rec, offsets, nb):
    """Per-launch algorithmic bytes of the foam forward and backward kernels (reference fp32 layout):
    forward  = sum_r [44 n S_r + (24 + 12 nb) n C_r + 16 n W_r + 68]
    backward = sum_r [(44 + 56) n S_r + (24 + 12 nb + 8 (6 + 3 nb)) n C_r + 16 n W_r + 84]
    with S samples, C coloured samples (coloured segments + 1 where any), W walk steps per ray and n the
    mean neighbourhood size (degree + 1) of the visited cells, measured from the records."""
    st = stats.double()
    S = st[:, 0].sum()
    C = (st[:, 1] + (st[:, 1] > 0).double()).sum()
    W = st[:, 2].sum()
    K = rec.size(1)
    fits = stats[:, 0] <= K
    s = stats[:, 0].clamp(max=K)
    mask = torch.arange(K, device=rec.device)[None, :] < s[:, None]
    cells = rec[..., 1].view(torch.int32)[mask & fits[:, None]].long()
    deg = (offsets[1:] - offsets[:-1]).long()
    n_bar = float((deg[cells] + 1).double().mean()) if cells.numel() else 16.0
    B = stats.size(0)
    fwd = 44 * n_bar * S + (24 + 12 * nb) * n_bar * C + 16 * n_bar * W + 68 * B
    bwd = 100 * n_bar * S + (24 + 12 * nb + 8 * (6 + 3 * nb)) * n_bar * C + 16 * n_bar * W + 84 * B
    return float(fwd), float(bwd), n_bar


def launches_per_step(n_rays, record_cap):
    """libvgb200 kernels launched by one training step (the CUB scans compiled into the library count
    as two kernels each): 2 conics; forward: field pack, deferred traversal, overflow rays, per pass of
    at most 2^26 record slots (scan, bucket, chunks, colour), composite; backward: field pack, re-traced
    rays, per pass (count, scan, bucketed items, chunks, scatter), gradient unpack; 2 conic backwards."""
    passes = math.ceil(n_rays / max(1, (1 << 26) // record_cap))
    forward = 3 + passes * (2 + 3) + 1
    backward = 2 + passes * (1 + 2 + 3) + 1
    return 2 + forward + backward + 2


# --------------------------------------------------------------------------------------- b200 arm

def run_b200(args):
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
        start_site = int(sites.nearest_sites(gr['points'], centre[None])[0])
        start_h = torch.full((len(o_h),), start_site, dtype=torch.int32)
    elif world == 1:
        centre, o_h, d_h = camera(args.config, 0, W, H, dev)
        start_site = int(sites.nearest_sites(gr['points'], centre[None])[0])
        start_h = torch.full((len(o_h),), start_site, dtype=torch.int32)
    else:
        # N views, 16x16 tiles of each dealt round-robin over the ranks (dist.view_tile_pixels): every rank
        # renders one view's worth of rays from the same mix of views
        o_l, d_l, s_l = [], [], []
        for v, pix in enumerate(vdist.view_tile_pixels(H, W, world, rank)):
            centre, c2w = scenes.orbit_camera(v, 8)
            o_v, d_v = scenes.camera_rays(centre, c2w, W, H, cfgd['fov'])
            pix = torch.from_numpy(pix)
            o_l.append(o_v[pix]), d_l.append(d_v[pix])
            s_l.append(torch.full((len(pix),), int(sites.nearest_sites(gr['points'], centre[None])[0]),
                                  dtype=torch.int32))
        o_h, d_h, start_h = torch.cat(o_l).contiguous(), torch.cat(d_l).contiguous(), torch.cat(s_l)
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
    timing = {'fwd': [], 'bwd': []}
    last = {}

    def foam_step(o, d, start, target, record_events=False):
        opt.zero_grad(set_to_none=True)
        near, _, far = render.ray_bounds(o, d, 0.02, 4.0)
        dA = ext.conic(model.d_log_scale, model.d_quat)
        cA = ext.conic(model.c_log_scale, model.c_quat)
        ev = [torch.cuda.Event(enable_timing=True) for _ in range(4)] if record_events else None
        if ev:
            ev[0].record()
        fg, T, _, stats = ext.foam(model.graph, model.raw, dA, cA, model.sh(), model.sh_deg, o, d, start, near, far,
                                   T_THRESH, W_THRESH, RECORD_CAP)
        if ev:
            ev[1].record()
        background = torch.sigmoid(model.bg_logit)  # seen through what the rays leave unabsorbed
        loss = ((fg + T.unsqueeze(1) * background - target) ** 2).mean()
        if ev:
            ext.BACKWARD_EVENTS = (ev[2], ev[3])
        loss.backward()
        ext.BACKWARD_EVENTS = None
        if world > 1:
            vdist.allreduce_grads(params)
        opt.step()
        if ev:
            timing['ev'] = ev
        last['stats'] = stats
        return loss

    torch.cuda.synchronize()
    for _ in range(args.warmup):
        foam_step(o, d, start, target)
    torch.cuda.synchronize()
    if world > 1:
        dist.barrier()

    # ---- device-resident timed region
    clk = clocks_start() if local == 0 else None
    time.sleep(0.3 if clk else 0)
    t0, t1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    evs = []
    torch.cuda.synchronize()
    if world > 1:
        dist.barrier()
    t0.record()
    for _ in range(args.steps):
        foam_step(o, d, start, target, record_events=True)
        evs.append(timing['ev'])
    t1.record()
    torch.cuda.synchronize()
    if world > 1:
        dist.barrier()
    clocks = clocks_stop(clk, local) if clk else None
    ms = t0.elapsed_time(t1) / args.steps
    fwd_ms = statistics.mean(e[0].elapsed_time(e[1]) for e in evs)
    bwd_ms = statistics.mean(e[2].elapsed_time(e[3]) for e in evs)
    if world > 1:
        tt = torch.tensor([ms, fwd_ms, bwd_ms], device=dev)
        dist.all_reduce(tt, op=dist.ReduceOp.MAX)
        ms, fwd_ms, bwd_ms = (float(x) for x in tt)

    # ---- algorithmic bytes of this workload, from one recorded forward
    with torch.no_grad():
        near, _, far = render.ray_bounds(o, d, 0.02, 4.0)
        dA = ext.conic(model.d_log_scale, model.d_quat)
        cA = ext.conic(model.c_log_scale, model.c_quat)
        _, _, _, stats, rec = ext.foam_extension().foam_forward(
            model.graph.points, model.graph.offsets, model.graph.adj, model.raw, dA, cA, model.sh(), model.sh_deg, o, d,
            start, near, far, T_THRESH, W_THRESH, RECORD_CAP)
        fwd_bytes, bwd_bytes, n_bar = algorithmic_bytes(stats, rec, model.graph.offsets, nb)
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
    dom = 'foam_backward' if bwd_ms >= fwd_ms else 'foam_forward'
    dom_ms, dom_bytes = (bwd_ms, bwd_bytes) if bwd_ms >= fwd_ms else (fwd_ms, fwd_bytes)
    achieved = dom_bytes / (dom_ms * 1e-3) / 1e9
    line = {
        'metric': (f'training Mrays/s (fwd+bwd+Adam), one {W}x{H} frame tile-sharded over the GPUs, 3M sites'
                   if args.strong else 'training Mrays/s (fwd+bwd+Adam) @1080p, 3M sites'),
        'value': round(value, 3), 'unit': 'Mrays/s',
        'n_gpus': world, 'steps': args.steps, 'warmup': args.warmup, 'ms_per_step': round(ms, 3),
        'higher_is_better': True, 'scaling': 'strong' if args.strong else 'weak', 'vs_baseline': None, 'dtype': 'f32',
        'data': 'synthetic',
        'config': {'workload': f'config{args.config}: {len(gr["points"])} sites ({cfgd["kind"]}), SH deg '
                               f'{model.sh_deg}, {W}x{H} rays per GPU, training step (fwd+bwd+Adam), record_cap '
                               f'{RECORD_CAP}, t/w_thresh {T_THRESH:g}',
                   'rays_per_gpu': B, 'sites': len(gr['points']),
                   'parallelism': f'dp{world} (16x16 tiles of {world} views dealt over the GPUs, NCCL all-reduce of '
                                  'site gradients)' if world > 1 else 'single GPU',
                   'l2': 'inputs larger than L2 (scene records + adjacency ~1 GB read every step)'},
        'fps': round(1000.0 / ms, 3), 'fwd_ms': round(fwd_ms, 3), 'bwd_ms': round(bwd_ms, 3),
        'fwd_mrays_s': round(B / (fwd_ms * 1e-3) / 1e6, 3), 'samples_per_ray': round(samples_per_ray, 2),
        'roofline': {'bound': 'hbm', 'kernel': f'{dom} (one vg_{dom} call: all its kernels)',
                     'achieved': round(achieved, 1), 'peak': peak, 'unit': 'GB/s',
                     'frac': round(achieved / peak, 4), 'traffic': None, 'peak_kind': peak_kind,
                     'algorithmic_bytes_per_launch': {'forward': fwd_bytes, 'backward': bwd_bytes},
                     'n_bar': round(n_bar, 3),
                     'note': 'algorithmic bytes count every neighbourhood gather as if from DRAM (reference fp32 '
                             'layout); L1/L2 reuse across the rays of a tile lets achieved exceed DRAM traffic'},
        'e2e': {'value': round(rays_total / (e2e_ms * 1e-3) / 1e6, 3), 'unit': 'Mrays/s', 'ms_per_step':
                round(e2e_ms, 3), 'h2d_bytes_per_step': h2d, 'd2h_bytes_per_step': 4,
                'copies': 'rays, start sites and target from pinned host memory every step, the next step\'s on a '
                          'side stream while the current one computes; the loss read back every step'},
        'gpu_launches': launches_per_step(B, RECORD_CAP) * args.steps,
        'clocks': clocks,
    }
    traffic = os.path.join(ROOT, 'profiles', 'traffic.json')
    if os.environ.get('VG_LIB_PATH'):  # a variant build of the library: name it and its knobs
        from voronoi_gauss_b200 import _lib
        knobs = os.path.join(os.path.dirname(_lib.LIB_PATH), 'defines.txt')
        line['config']['library'] = {'path': _lib.LIB_PATH, 'defines': open(knobs).read().split()
                                     if os.path.exists(knobs) else []}
    if os.path.exists(traffic) and W * H == 1920 * 1080 and args.config == 3 and args.sites is None:
        with open(traffic) as f:
            tr = json.load(f)
        if dom in tr:
            t_bytes = float(tr[dom]['dram_bytes_per_call'])
            line['roofline']['traffic'] = t_bytes
            line['roofline']['dram_gbs'] = round(t_bytes / (dom_ms * 1e-3) / 1e9, 1)
            line['roofline']['dram_frac'] = round(t_bytes / (dom_ms * 1e-3) / 1e9 / peak, 4)
            line['roofline']['traffic_source'] = tr['source']
    if rank == 0 and world == 1 and not args.no_baselines:
        line['cpu_baseline'] = cpu_baseline(gr, prm, o_h, d_h, start_site, args)
        line['ref_cuda'] = ref_cuda_baseline(model, o, d, start, target, args)
    if world > 1:
        dist.destroy_process_group()
    if rank == 0:
        print(json.dumps(line), flush=True)


def ref_cuda_baseline(model, o, d, start, target, args):
    """The reference's own CUDA kernels (built unchanged from its sources into oracle/_ref) on the same
    workload: foam_forward with records + foam_backward, timed with CUDA events."""
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

        def fwd():
            return rf.foam_forward(g.points, g.offsets, g.adj, model.raw.detach(), dA, cA, sh, model.sh_deg, o, d,
                                   start, near, far, T_THRESH, W_THRESH, RECORD_CAP)

        def bwd(out):
            rgb, T, _, stats, rec = out
            return rf.foam_backward(g.points, g.offsets, g.adj, model.raw.detach(), dA, cA, sh, model.sh_deg, o, d,
                                    start, near, far, T_THRESH, W_THRESH, rgb, T, torch.ones_like(rgb),
                                    torch.ones_like(T), rec, stats)
        out = fwd()
        bwd(out)
        torch.cuda.synchronize()
        reps = 2
        a, b, c = (torch.cuda.Event(enable_timing=True) for _ in range(3))
        f_ms = b_ms = 0.0
        for _ in range(reps):
            a.record()
            out = fwd()
            b.record()
            bwd(out)
            c.record()
            torch.cuda.synchronize()
            f_ms += a.elapsed_time(b) / reps
            b_ms += b.elapsed_time(c) / reps
            del out
        return {'kind': 'reference CUDA kernels (foam.cu, built unchanged for sm_100a)', 'fwd_ms': round(f_ms, 3),
                'bwd_ms': round(b_ms, 3), 'fwd_mrays_s': round(B / (f_ms * 1e-3) / 1e6, 3),
                'fwd_bwd_mrays_s': round(B / ((f_ms + b_ms) * 1e-3) / 1e6, 3)}


def cpu_baseline(gr, prm, o_h, d_h, start_site, args, seconds=10.0, max_chunks=64):
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
        start = np.full(chunk, start_site, np.int32)
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


# ---------------------------------------------------------------------------------- reference arm

def run_reference(args):
    """Reference arm: the reference path's CPU restatement (oracle/) on the host cores, bounded sample per
    step; rank 0 only."""
    rank = int(os.environ.get('RANK', 0))
    if rank != 0:
        return
    from oracle import oracle
    from voronoi_gauss_b200 import ext, render, scenes, sites
    cfgd = scenes.CONFIGS[args.config]
    W = args.width or cfgd['W']
    H = args.height or cfgd['H']
    gr = load_scene(args.config, args.sites, 0)
    prm = scenes.make_params(args.config, gr['points'].astype(np.float64))
    centre, o_h, d_h = camera(args.config, 0, W, H, 'cpu')
    start_site = int(sites.nearest_sites(gr['points'], centre[None])[0])
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
        start = np.full(n_rays, start_site, np.int32)
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
    line = {'impl': 'reference', 'metric': 'training Mrays/s (fwd+bwd+Adam) @1080p, 3M sites', 'value':
            round(value, 6), 'unit': 'Mrays/s', 'n_gpus': int(os.environ.get('WORLD_SIZE', 1)), 'steps': args.steps,
            'warmup': args.warmup, 'ms_per_step': round(ms, 3), 'higher_is_better': True, 'scaling': 'weak',
            'vs_baseline': None, 'dtype': 'f32', 'data': 'synthetic',
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
    else:
        run_b200(a)
