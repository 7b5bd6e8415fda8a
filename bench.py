#!/usr/bin/env python
"""Benchmark of the scene-packed attention hot path on B200 (BASELINE.json metric: scene-packed attention TFLOP/s per
GPU). One step = one scene-attention layer of BASELINE cfg2 (HunyuanVideo-1.5 shape: 4 scenes of [8, 6, 10, 7] latent
frames, 1590 tokens per frame, 128 text tokens per scene, frame memory {0, 8, 14, 24}, 16 heads x 128, bf16):
the gather/pack launch (K and V of every segment) plus the attention launches (video queries, text queries), inputs
resident in HBM. Useful FLOPs per step = sum over segments of 4 * lq * lk * H * D (experiments/kernel_breakdown.py:101
of the reference) = 7.187 TFLOP.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]

--impl reference times the reference's CPU path (oracle/cpu_path.py: the reference processor with per-segment fp32
SDPA in place of FlashAttention) on the host cores, rank 0 only. Prints one JSON line (rank 0).
"""
from __future__ import annotations

import argparse
import json
import os
import subprocess
import sys
import time
from pathlib import Path

import numpy as np
import torch

ROOT = Path(__file__).resolve().parent
sys.path.insert(0, str(ROOT))

CFG2 = dict(lengths=[8, 6, 10, 7], T=1590, text=128, heads=16, dim=128, memory=[0, 8, 14, 24])
# a reduced cfg2 (first two scenes) for profiler captures: inputs still larger than L2, a few hundred MB on the device
SMALL = dict(lengths=[8, 6], T=1590, text=128, heads=16, dim=128, memory=[0, 8])
# BASELINE cfg3: Wan2.2-TI2V-5B-shaped layer through the joint [video | text] scene path, sharded (strong scaling)
CFG3 = dict(lengths=[3, 12, 5, 9, 4, 8], T=880, text=256, heads=24, dim=128, memory=[0, 3, 15, 20])
# BASELINE cfg4: full denoising step of the HunyuanVideo-1.5-architecture stand-in (4 scenes x 31 frames, 480p)
# BASELINE cfg5: Wan2.2-shaped long-video stress layer, S scenes x 31 latent frames at 880 tokens per frame, 24 x 128
# heads, frame memory 4 (the first frame of the first four scenes), no joint text (Wan self-attention)
CFG5 = dict(scene_frames=31, T=880, text=0, heads=24, dim=128)
CFG4 = dict(lengths=[31, 31, 31, 31], T=1590, text=128, heads=16, dim=128, memory=[0, 31, 62, 93], hidden=2048,
            blocks=54, frame_hw=(30, 53))
METRIC = 'scene-packed attn TFLOP/s/GPU; DiT step latency @1/2/4/8 B200'
# DRAM bytes / algorithmic bytes of the attention kernel, from the small-case ncu capture summarised in profiles/
TRAFFIC_PER_ALG_BYTE = 373.86 / 392.9


def cfg_layout(cfg):
    """frame memory = the first latent frame of the first scenes (BASELINE cfg1's rule), read by every other scene"""
    from onereel_b200.layout import SceneLayout
    lay = SceneLayout(cfg['lengths'], halo=0)
    lay.extra = {j: [f for f in cfg['memory'] if not lo <= f < hi] for j, (lo, hi) in enumerate(lay.ranges)}
    return lay


def peaks():
    p = ROOT / 'MEASURED_PEAKS.json'
    if p.exists():
        d = json.loads(p.read_text())
        return d['bf16_tflops'], d.get('bf16_tflops_sustained'), d['hbm_gbs'], 'measured'
    return 1590.0, 1400.0, 6650.0, 'fallback'


class Clocks:
    """nvidia-smi sampling of SM clocks and throttle reasons during the timed region"""
    Q = ('index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,clocks_event_reasons.hw_slowdown,'
         'clocks_event_reasons.hw_thermal_slowdown,clocks_event_reasons.sw_thermal_slowdown,'
         'clocks_event_reasons.sw_power_cap')

    def __init__(self, index):
        self.index, self.proc, self.path = index, None, Path(f'/tmp/orl_clocks_{os.getpid()}.csv')

    def __enter__(self):
        try:
            self.proc = subprocess.Popen(['nvidia-smi', f'--id={self.index}', f'--query-gpu={self.Q}',
                                          '--format=csv,noheader,nounits', '-lms', '200'],
                                         stdout=open(self.path, 'w'), stderr=subprocess.DEVNULL)
        except (FileNotFoundError, OSError):
            self.proc = None
        time.sleep(0.3)
        return self

    def __exit__(self, *a):
        if self.proc is not None:
            self.proc.terminate()
            self.proc.wait(timeout=10)

    def summary(self):
        if self.proc is None or not self.path.exists():
            return None
        rows = [r.split(', ') for r in self.path.read_text().strip().splitlines() if r.count(',') >= 8]
        if not rows:
            return None
        sm = [float(r[1]) for r in rows if r[1].replace('.', '').isdigit()]
        mx = max(float(r[2]) for r in rows)
        names = ['hw_slowdown', 'hw_thermal_slowdown', 'sw_thermal_slowdown', 'sw_power_cap']
        reasons = sorted({n for r in rows for n, v in zip(names, r[5:9]) if v.strip() == 'Active'})
        load = [s for s in sm if s > 0.5 * mx] or sm
        self.path.unlink(missing_ok=True)
        return dict(sm_mhz=float(np.median(load)), sm_max_mhz=mx, reasons=reasons, samples=len(rows))


def dist_env():
    return int(os.environ.get('RANK', 0)), int(os.environ.get('WORLD_SIZE', 1)), int(os.environ.get('LOCAL_RANK', 0))


def cpu_baseline(steps=1, warmup=0, target_s=3.0):
    """the reference CPU path on a bounded sample of cfg2 (every `sample`-th query row of every segment, all keys)"""
    from oracle import cpu_path, layout_oracle as LO
    lay = LO.Layout(CFG2['lengths'], halo=0, extra={j: [f for f in CFG2['memory'] if not lo <= f < hi]
                                                   for j, (lo, hi) in enumerate(LO.Layout(CFG2['lengths']).ranges())})
    counts = [CFG2['text']] * len(CFG2['lengths'])
    H, Dh = CFG2['heads'], CFG2['dim']
    probe_t, probe_f, _ = cpu_path.time_cpu(lay, CFG2['T'], counts, H, Dh, sample=512, repeats=1)
    full = 7.187e12
    sample = max(1, int(round(full / (probe_f / probe_t) / target_s)))
    ts, fl = [], 0.0
    for i in range(warmup + steps):
        t, fl, threads = cpu_path.time_cpu(lay, CFG2['T'], counts, H, Dh, sample=sample, repeats=1, seed=i)
        if i >= warmup:
            ts.append(t)
    t = float(np.median(ts))
    return dict(value=fl / t / 1e12, unit='TFLOP/s', cores=threads, kind='port',
                sample=f'cfg2 layer, every {sample}th query row of every segment with all its keys '
                       f'({fl / 1e12:.3f} TFLOP of the 7.187), fp32 torch SDPA per segment, median of {len(ts)}'), t


def run_reference(args):
    rank, world, _ = dist_env()
    if rank != 0:
        return
    cb, t = cpu_baseline(steps=args.steps, warmup=args.warmup)
    line = dict(impl='reference', metric=METRIC, value=cb['value'], unit='TFLOP/s', n_gpus=args.gpus,
                steps=args.steps, warmup=args.warmup, ms_per_step=t * 1e3, higher_is_better=True, scaling='weak',
                vs_baseline=None, dtype='f32', data='synthetic',
                config=dict(workload='cfg2 scene-attention layer (reference CPU path, bounded sample)',
                            layout=CFG2), cpu_baseline=cb,
                e2e=dict(value=cb['value'], unit='TFLOP/s', h2d_bytes_per_step=0, d2h_bytes_per_step=0))
    print(json.dumps(line), flush=True)


def make_inputs(lay, T, counts, H, Dh, dev, rows=None, seed=0):
    """Q/K RMS-normed over D from N(0, 1) (unit weight), V ~ N(0, 1) (BASELINE cfg2), drawn on the device from a
    generator seeded by (seed, first row) so every rank draws only its own rows = the rank's video range (a, b)"""
    g = torch.Generator(device=dev).manual_seed(seed * 1000003 + (rows[0] if rows else 0))
    L, Nt = lay.n_frames * T, sum(counts)
    a, b = rows or (0, L)

    def qk(n):
        x = torch.randn(n, H, Dh, generator=g, device=dev)
        return (x * torch.rsqrt(x.pow(2).mean(-1, keepdim=True) + 1e-6)).to(torch.bfloat16)
    q, k = qk(b - a), qk(b - a)
    v = torch.randn(b - a, H, Dh, generator=g, device=dev).to(torch.bfloat16)
    eq, ek = qk(Nt), qk(Nt)
    ev = torch.randn(Nt, H, Dh, generator=g, device=dev).to(torch.bfloat16)
    return [x.contiguous() for x in (q, k, v, eq, ek, ev)]


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument('--gpus', type=int, default=1)
    ap.add_argument('--steps', type=int, default=100)
    ap.add_argument('--warmup', type=int, default=5)
    ap.add_argument('--impl', default='ours', choices=['ours', 'reference'])
    ap.add_argument('--mode', default='auto',
                    help='parallel path for N > 1: auto (the Eq. 2 chooser), scene or ulysses; a comma list runs '
                         'each in turn and prints one line per mode')
    ap.add_argument('--overlap', default='auto', choices=['auto', 'none', 'lse'],
                    help="K/V gathering: 'lse' attends far scenes to their local keys while the exchange is in flight "
                         "and merges by log-sum-exp (Context.overlap of the reference); 'auto' takes 'lse' from 4 "
                         "GPUs up (measured on 8 B200: +8 %% on the weak cfg2 layer; on 2 the two are even)")
    ap.add_argument('--no-cpu-baseline', action='store_true')
    ap.add_argument('--no-e2e', action='store_true', help='skip the host-buffer end-to-end leg (auto for cfg5)')
    ap.add_argument('--scenes', default='16', help='cfg5: scene counts to sweep (comma list)')
    ap.add_argument('--workload', default='cfg2', choices=['cfg2', 'small', 'cfg3', 'cfg4', 'cfg5'],
                    help='cfg2 (default bench line; weak scaling over N); small: the first two scenes of cfg2, for '
                         'profiler captures; cfg3: BASELINE cfg3 layer sharded over N (strong scaling); cfg4: one '
                         'full DiT denoising step of the stand-in (strong scaling); cfg5: Wan-shaped stress layer '
                         'with --scenes S (strong scaling)')
    args = ap.parse_args()
    if args.impl == 'reference':
        return run_reference(args)
    if args.workload == 'cfg4':
        return run_dit_step(args)
    runs = [(m, sc) for sc in (args.scenes.split(',') if args.workload == 'cfg5' else [None])
            for m in args.mode.split(',')]
    for i, (mode, sc) in enumerate(runs):
        args.mode, args.n_scenes = mode, (int(sc) if sc else None)
        run_layer(args, last=i == len(runs) - 1)


def run_layer(args, last=True):
    """one scene-attention layer per step through the public processor API (the default bench line)"""
    from onereel_b200 import attention as A
    from onereel_b200 import dist as D
    from onereel_b200 import hunyuan15 as HY
    from onereel_b200 import scene as S
    from onereel_b200.csrc.build import build
    from onereel_b200.pack import RunTable
    rank, world, local = dist_env()
    if rank == 0:
        build()
    D.init('nccl')
    if world > 1:
        D.barrier()
        build()                      # other ranks load the library rank 0 built
    dev = torch.device('cuda', local)

    if args.workload == 'cfg5':
        S_ = args.n_scenes
        cfg = dict(CFG5, lengths=[CFG5['scene_frames']] * S_,
                   memory=[j * CFG5['scene_frames'] for j in range(min(4, S_))])
    else:
        cfg = dict({'cfg2': CFG2, 'small': SMALL, 'cfg3': CFG3}[args.workload])
    if args.workload not in ('cfg3', 'cfg5'):
        # weak scaling: N GPUs run cfg2's scene set repeated N times (per-GPU work fixed); every scene reads the frame
        # memory of the first copy, so ranks exchange those rows (the path's real K/V gathering step)
        cfg['lengths'] = cfg['lengths'] * world
    lay = cfg_layout(cfg)
    T, H, Dh = cfg['T'], cfg['heads'], cfg['dim']
    counts = [cfg['text']] * lay.n_scenes
    wan = args.workload == 'cfg5'
    if args.overlap == 'auto':                   # the LSE split pays once most pieces wait for remote keys
        args.overlap = 'lse' if world >= 4 and not wan else 'none'
    if wan:
        from onereel_b200 import comm, wan as WN
        ctx = WN.Context(lay, mode=args.mode, T=T)
        WN.plan_parallel(ctx, H)
        wproc = WN.Processor(ctx, 'self', None, 0)

        class _WanCall:
            """Wan self-attention of the local rows (wan.py:97-107 dispatch) in the processor-call shape"""
            def scene(self, q, k, v, *text):
                if ctx.run_mode == 'ulysses' or world == 1:
                    o = comm.a2a_tokens(wproc.ranges(comm.a2a_heads(q), comm.a2a_heads(k), comm.a2a_heads(v)))
                else:
                    o = wproc.scene(q, k, v)
                return o, text[0]
            ulysses = scene
        proc = _WanCall()
    else:
        ctx = HY.Context(lay, mode=args.mode, T=T, counts={True: counts, False: counts}, fwd=1, overlap=args.overlap)
        HY.plan_parallel(ctx, H)
        proc = HY.Processor(ctx, 0)
    own = ctx.own[rank]
    q, k, v, eq, ek, ev = make_inputs(lay, T, counts, H, Dh, dev, own, seed=0)
    stream = torch.cuda.current_stream(dev)

    def step():
        if ctx.run_mode == 'ulysses':
            return proc.ulysses(q, k, v, eq, ek, ev)
        return proc.scene(q, k, v, eq, ek, ev)

    for _ in range(args.warmup):
        step()
    torch.cuda.synchronize()
    A.check()
    # useful FLOPs of this rank's segments (one timed pass of the instrumented launches)
    S.TIMING = []
    step()
    torch.cuda.synchronize()
    rank_flops = sum(f for _, _, f in S.TIMING)
    S.TIMING = None
    # algorithmic bytes of the attention launches: every query row read and its output written once, every segment's
    # keys and values read once per head (H * D * 2 bytes per row)
    attn_bytes = 0
    if ctx.run_mode == 'scene' and not wan:
        p_ = proc._plan(H, Dh, dev, ctx.overlap == 'lse')
        for pl in (p_.near, p_.far, p_.far_local, p_.far_remote):
            if pl is not None:
                attn_bytes += sum(2 * a + 2 * b for a, b in zip(pl.lq, pl.lk)) * H * Dh * 2

    with Clocks(local) as clk:
        D.barrier()
        torch.cuda.synchronize()
        S.TIMING = []
        packs0 = RunTable.launches
        t0, t1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        t0.record(stream)
        for _ in range(args.steps):
            step()
        t1.record(stream)
        torch.cuda.synchronize()
        D.barrier()
    timing, S.TIMING = S.TIMING, None
    n_launches = len(timing) + RunTable.launches - packs0
    A.check()
    ms = t0.elapsed_time(t1) / args.steps
    attn_ms = sum(a.elapsed_time(b) for a, b, _ in timing) / args.steps

    e2e_ms, h2d, d2h = None, 0, 0
    if not (args.no_e2e or args.workload == 'cfg5'):
        # end to end through the public API with host buffers: every step copies its layer's local q/k/v and the text
        # q/k/v host->device from pinned memory, calls the processor, and copies its outputs device->host. Steps are
        # pipelined the way a caller streaming layers would run them: two device input buffers, H2D on one copy stream,
        # D2H on another, so step i+1's inputs travel while step i computes and step i-1's outputs return.
        host_in = [x.cpu().pin_memory() for x in (q, k, v, eq, ek, ev)]
        dev_in = [[torch.empty_like(x) for x in (q, k, v, eq, ek, ev)] for _ in range(2)]
        host_out = [[torch.empty(q.shape, dtype=q.dtype, pin_memory=True),
                     torch.empty(eq.shape, dtype=eq.dtype, pin_memory=True)] for _ in range(2)]
        s_in, s_out = torch.cuda.Stream(dev), torch.cuda.Stream(dev)
        ready = [torch.cuda.Event() for _ in range(2)]
        done = [torch.cuda.Event() for _ in range(2)]
        done[0].record(stream)
        done[1].record(stream)

        def e2e_step(i):
            b = i % 2
            with torch.cuda.stream(s_in):
                s_in.wait_event(done[b])                      # step i - 2 has finished reading this buffer
                for d_, h_ in zip(dev_in[b], host_in):
                    d_.copy_(h_, non_blocking=True)
                ready[b].record(s_in)
            stream.wait_event(ready[b])
            ov, ot = (proc.ulysses if ctx.run_mode == 'ulysses' else proc.scene)(*dev_in[b])
            done[b].record(stream)
            with torch.cuda.stream(s_out):
                s_out.wait_event(done[b])
                ov.record_stream(s_out)
                ot.record_stream(s_out)
                host_out[b][0].copy_(ov, non_blocking=True)
                host_out[b][1].copy_(ot, non_blocking=True)
        for i in range(2):
            e2e_step(i)
        torch.cuda.synchronize()
        e_steps = max(4, args.steps // 4)
        D.barrier()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record(s_in)
        for i in range(e_steps):
            e2e_step(i)
        e1.record(s_out)
        torch.cuda.synchronize()
        D.barrier()
        A.check()
        e2e_ms = e0.elapsed_time(e1) / e_steps
        h2d = sum(x.numel() * x.element_size() for x in host_in)
        d2h = sum(x.numel() * x.element_size() for x in host_out[0])

    total_flops = rank_flops
    if world > 1:
        import torch.distributed as dist
        t = torch.tensor([ms, attn_ms, e2e_ms or 0.0], device=dev)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        ms, attn_ms_max, e2e_ms = t.tolist()
        e2e_ms = e2e_ms or None
        f = torch.tensor([rank_flops], dtype=torch.float64, device=dev)
        dist.all_reduce(f)
        total_flops = f.item()
    if rank != 0:
        if last:
            D.shutdown()
        return
    peak_burst, peak_sus, hbm, peak_kind = peaks()
    achieved = rank_flops / (attn_ms * 1e-3) / 1e12
    cb = None
    if not args.no_cpu_baseline and args.workload == 'cfg2' and world == 1:
        cb, _ = cpu_baseline()
    line = dict(metric=METRIC, value=total_flops / (ms * 1e-3) / 1e12, unit='TFLOP/s', n_gpus=world,
                steps=args.steps, warmup=args.warmup, ms_per_step=ms, higher_is_better=True,
                scaling='strong' if args.workload in ('cfg3', 'cfg5') else 'weak',
                vs_baseline=None, dtype='bf16', data='synthetic (seeded; Q/K RMS-normed N(0,1), V N(0,1))',
                config=dict(workload=(f'{args.workload}: one ' + ('Wan2.2-shaped self-attention layer through '
                                      'wan.Processor' if wan else 'HunyuanVideo-1.5-shaped scene-attention layer through '
                                      'hunyuan15.Processor.scene') + ' (pack K/V + attention' +
                                      (', K/V exchange over NCCL' if world > 1 else '') + ')'),
                            layout=dict(cfg, scenes=lay.n_scenes), run_mode=ctx.run_mode, path=ctx.path,
                            overlap=args.overlap,
                            own=ctx.own, useful_tflop_per_step=total_flops / 1e12,
                            parallelism=(f'{ctx.run_mode} x{world} ' + ('(strong: layout fixed)'
                                         if args.workload in ('cfg3', 'cfg5')
                                         else '(weak: cfg2 scene set repeated per GPU)') if world > 1 else 'single'),
                            l2='inputs larger than L2 (q/k/v 203 MB each per GPU, packed K/V ~486 MB each)'),
                e2e=None if e2e_ms is None else dict(value=total_flops / (e2e_ms * 1e-3) / 1e12, unit='TFLOP/s',
                         ms_per_step=e2e_ms,
                         h2d_bytes_per_step=h2d, d2h_bytes_per_step=d2h,
                         note='processor call with pinned H2D inputs / D2H outputs every step; consecutive steps '
                              'pipelined on separate copy streams (double-buffered inputs)'),
                roofline=dict(bound='tensor', achieved=achieved, peak=peak_burst, unit='TFLOP/s',
                              frac=achieved / peak_burst,
                              traffic=(attn_bytes * TRAFFIC_PER_ALG_BYTE if args.workload == 'cfg2' and world == 1
                                       else None),
                              traffic_note='bytes per step of the attention launches: their algorithmic bytes (Q + O '
                                           '+ K/V once per segment) x the DRAM/algorithmic ratio of the small-case '
                                           'ncu capture (summarised in profiles/)',
                              frac_of_sustained=achieved / peak_sus if peak_sus else None,
                              kernel='attn_fwd_kernel<128> (all attention launches of a step, rank 0)',
                              peak_source=f'{peak_kind} bf16 burst'),
                gpu_launches=n_launches, clocks=clk.summary(), cpu_baseline=cb)
    print(json.dumps(line), flush=True)
    if last:
        D.shutdown()


def run_dit_step(args):
    """BASELINE cfg4: one denoising step (conditional + unconditional forward of 54 blocks) of the random-init
    HunyuanVideo-1.5-architecture stand-in (onereel_b200/standin.py) on this rank's video rows, scene-parallel
    attention through the B200 processors; latency = device time of the step, max over ranks (strong scaling)."""
    from onereel_b200 import attention as A, dist as D, hunyuan15 as HY, standin
    from onereel_b200.csrc.build import build
    rank, world, local = dist_env()
    if rank == 0:
        build()
    D.init('nccl')
    if world > 1:
        D.barrier()
        build()
    dev = torch.device('cuda', local)
    cfg = CFG4
    lay = cfg_layout(cfg)
    T, H, Dh, C = cfg['T'], cfg['heads'], cfg['dim'], cfg['hidden']
    counts = [cfg['text']] * lay.n_scenes
    if args.overlap == 'auto':                   # measured on 4 B200: the LSE split does not pay for the DiT step
        args.overlap = 'none'
    ctx = HY.Context(lay, mode=args.mode, T=T, counts={True: counts, False: counts}, overlap=args.overlap)
    HY.plan_parallel(ctx, H)
    a, b = ctx.own[rank]
    model = standin.build(ctx, dev, C, H, cfg['blocks'])
    g = torch.Generator().manual_seed(1)
    L, Nt = lay.n_frames * T, sum(counts)
    hs = torch.randn(1, b - a, C, generator=g).to(dev, torch.bfloat16)
    ehs_c, ehs_u = (torch.randn(1, Nt, C, generator=g).to(dev, torch.bfloat16) for _ in range(2))
    temb = torch.randn(1, C, generator=g).to(dev, torch.bfloat16)
    cos, sin = standin.rope_3d(lay.n_frames, *cfg['frame_hw'], Dh)
    rot = (cos.to(dev), sin.to(dev))
    stream = torch.cuda.current_stream(dev)
    for _ in range(args.warmup):
        standin.dit_step(model, ctx, hs, ehs_c, ehs_u, temb, rot)
    torch.cuda.synchronize()
    A.check()
    with Clocks(local) as clk:
        D.barrier()
        t0, t1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        t0.record(stream)
        for _ in range(args.steps):
            standin.dit_step(model, ctx, hs, ehs_c, ehs_u, temb, rot)
        t1.record(stream)
        torch.cuda.synchronize()
        D.barrier()
    A.check()
    ms = t0.elapsed_time(t1) / args.steps
    if world > 1:
        import torch.distributed as dist
        t = torch.tensor([ms], device=dev)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        ms = t.item()
    if rank == 0:
        tokens = L + Nt
        gemm = 2 * cfg['blocks'] * 24 * C * C * tokens
        segs = [(s_.lq, s_.lk) for s_ in HY.S.scene_segments(lay, T, counts, [(j, (lo * T, hi * T)) for j, (lo, hi)
                                                            in enumerate(lay.ranges)], set(range(lay.n_scenes)), (0, L))]
        attn = 2 * cfg['blocks'] * sum(4.0 * x * y * H * Dh for x, y in segs)
        print(json.dumps(dict(metric='DiT step latency (cfg4)', value=ms, unit='ms', n_gpus=world, steps=args.steps,
                              warmup=args.warmup, ms_per_step=ms, higher_is_better=False, scaling='strong',
                              dtype='bf16', data='synthetic (random-init stand-in, seeded)',
                              config=dict(workload='cfg4: one denoising step (2 CFG forwards x 54 blocks) of the '
                                                   'HunyuanVideo-1.5-architecture stand-in', layout=cfg,
                                          run_mode=ctx.run_mode, path=ctx.path, own=ctx.own, overlap=ctx.overlap,
                                          flop_per_step=dict(gemm=gemm, attention=attn)),
                              achieved_tflops=(gemm + attn) / (ms * 1e-3) / 1e12, clocks=clk.summary())), flush=True)
    D.shutdown()


if __name__ == '__main__':
    main()
