#!/usr/bin/env python
"""Benchmark of the scene-packed attention hot path on B200 (BASELINE.json metric: "scene-packed attn TFLOP/s/GPU;
DiT step latency @1/2/4/8 B200").

Headline step = one scene-attention layer of BASELINE cfg2 (HunyuanVideo-1.5 shape: 4 scenes of [8, 6, 10, 7] latent
frames, 1590 tokens per frame, 128 text tokens per scene, frame memory {0, 8, 14, 24}, 16 heads x 128, bf16) through
hunyuan15.Processor.scene: the gather/pack launch (K and V of every segment) plus the attention launches, inputs
resident in HBM. Useful FLOPs per step = sum over segments of 4 * lq * lk * H * D (experiments/kernel_breakdown.py:101
of the reference) = 7.187 TFLOP. At N GPUs the headline runs cfg2's scene set repeated N times (weak scaling: about one
cfg2 per GPU, every scene reading the same four frame-memory frames, pulled from their owner over NVLink peer memory;
--exchange nccl moves them by NCCL send/recv instead, as the reference does).

Beside the headline, the same JSON line carries, at every N (all timed on the device, max over ranks):
  parity       the rank's outputs of the timed path against a one-GPU recompute of the same rows on the same rank
               (bit-exact expected for K/V gathering without the LSE split and for Ulysses) and against fp32 attention
               on sampled rows of every segment (max-abs 2e-2, mean-abs 2e-3);
  phases_ms    per-phase device time of the headline step (near attention, exposed exchange wait, far attention,
               text-row sync; Ulysses: all-to-all in, attention, text all-reduce, all-to-all out);
  comm         the K/V exchange timed alone with its bytes, the text-row bytes, and the measured NCCL peaks
               (pairwise send/recv per direction, all-to-all) — roofline_nvlink divides the exchange's bytes per GPU
               by its time and by the pairwise peak;
  cfg3         BASELINE cfg3 (Wan2.2-TI2V-5B shape, joint [video | text] scene path) strong-scaled over N: TFLOP/s of
               K/V gathering, Ulysses and the Eq. 2 choice ('auto'), with V_G / V_U and each mode's parity;
  dit_step     BASELINE cfg4: latency of one full denoising step (2 CFG forwards x 54 blocks) of the random-init
               HunyuanVideo-1.5-architecture stand-in, strong-scaled over N, with its clocks.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference] [--legs LIST]

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
CFG4 = dict(lengths=[31, 31, 31, 31], T=1590, text=128, heads=16, dim=128, memory=[0, 31, 62, 93], hidden=2048,
            blocks=54, frame_hw=(30, 53))
# BASELINE cfg5: Wan2.2-shaped long-video stress layer, S scenes x 31 latent frames at 880 tokens per frame, 24 x 128
# heads, frame memory 4 (the first frame of the first four scenes), no joint text (Wan self-attention)
CFG5 = dict(scene_frames=31, T=880, text=0, heads=24, dim=128)
METRIC = 'scene-packed attn TFLOP/s/GPU; DiT step latency @1/2/4/8 B200'
# DRAM bytes / algorithmic bytes of the attention kernel, from the small-case ncu capture summarised in profiles/
TRAFFIC_PER_ALG_BYTE = 373.86 / 392.9
MAX_ABS, MEAN_ABS = 2e-2, 2e-3          # north_star's tolerance on bf16 inputs
# NVLink 5 peer copy per direction per GPU, as measured on this pool's B200 nodes (nominal 900 GB/s)
NVLINK_PEER_GBS = 770.0
LEGS = ('parity', 'phases', 'comm', 'kernels', 'cfg3', 'dit', 'fa2')


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


def cpu_model() -> str:
    try:
        for line in Path('/proc/cpuinfo').read_text().splitlines():
            if line.startswith('model name'):
                return line.split(':', 1)[1].strip()
    except OSError:
        pass
    return 'unknown'


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
                                          '--format=csv,noheader,nounits', '-lms', '50'],
                                         stdout=open(self.path, 'w'), stderr=subprocess.DEVNULL)
        except (FileNotFoundError, OSError):
            self.proc = None
        # the timed region starts once the sampler is running (its first line written; NVML start-up can take
        # a second on a busy 8-GPU host), so a short region still gets samples
        t0 = time.time()
        while self.proc is not None and time.time() - t0 < 10.0:
            if self.path.exists() and self.path.stat().st_size > 0:
                break
            time.sleep(0.05)
        self.start_lines = self._lines()
        return self

    def _lines(self):
        try:
            return len(self.path.read_text().strip().splitlines())
        except OSError:
            return 0

    def __exit__(self, *a):
        if self.proc is not None:
            self.proc.terminate()
            self.proc.wait(timeout=10)

    def summary(self):
        if self.proc is None or not self.path.exists():
            return None
        lines = self.path.read_text().strip().splitlines()
        # the samples taken while the timed region ran (the lines written before it started are dropped, but the
        # last of those is kept when the region was shorter than one sampling interval)
        lines = lines[max(0, getattr(self, 'start_lines', 0) - 1):]
        rows = [r.split(', ') for r in lines if r.count(',') >= 8]
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


# ------------------------------------------------------------------------------------------------ CPU reference arm

def cpu_baseline(steps=3, warmup=1, target_s=3.0):
    """the reference CPU path on a bounded sample of cfg2 (every `sample`-th query row of every segment, all keys):
    `warmup` untimed runs, then the median of `steps` timed runs"""
    from oracle import cpu_path, layout_oracle as LO
    lay = LO.Layout(CFG2['lengths'], halo=0, extra={j: [f for f in CFG2['memory'] if not lo <= f < hi]
                                                   for j, (lo, hi) in enumerate(LO.Layout(CFG2['lengths']).ranges())})
    counts = [CFG2['text']] * len(CFG2['lengths'])
    H, Dh = CFG2['heads'], CFG2['dim']
    probe_t, probe_f, _ = cpu_path.time_cpu(lay, CFG2['T'], counts, H, Dh, sample=512, repeats=1)
    full = 7.187e12
    sample = max(1, int(round(full / (probe_f / probe_t) / target_s)))
    ts, fl, threads = [], 0.0, 1
    for i in range(warmup + steps):
        t, fl, threads = cpu_path.time_cpu(lay, CFG2['T'], counts, H, Dh, sample=sample, repeats=1, seed=i)
        if i >= warmup:
            ts.append(t)
    t = float(np.median(ts))
    return dict(value=fl / t / 1e12, unit='TFLOP/s', cores=threads, kind='port', cpu=cpu_model(),
                sample=f'cfg2 layer, every {sample}th query row of every segment with all its keys '
                       f'({fl / 1e12:.3f} TFLOP of the 7.187), fp32 torch SDPA per segment, median of {len(ts)} '
                       f'after {warmup} warm-up'), t


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


# ------------------------------------------------------------------------------------------------ inputs

def full_inputs(lay, T, counts, H, Dh, dev, seed=0):
    """the whole layer's q / k / v (video rows) and eq / ek / ev (text rows), drawn on the device from one seeded
    generator, identical on every rank (so any rank can recompute any rows): Q/K RMS-normed over D from N(0, 1) with
    unit weight, V ~ N(0, 1) (BASELINE cfg2)"""
    g = torch.Generator(device=dev).manual_seed(seed)
    L, Nt = lay.n_frames * T, sum(counts)

    def qk(n):
        x = torch.randn(n, H, Dh, generator=g, device=dev)
        return (x * torch.rsqrt(x.pow(2).mean(-1, keepdim=True) + 1e-6)).to(torch.bfloat16)
    q, k = qk(L), qk(L)
    v = torch.randn(L, H, Dh, generator=g, device=dev).to(torch.bfloat16)
    eq, ek = qk(Nt), qk(Nt)
    ev = torch.randn(Nt, H, Dh, generator=g, device=dev).to(torch.bfloat16)
    return q, k, v, eq, ek, ev


def reduce(vals, op='max', dtype=torch.float64):
    """element-wise max / sum / min of a list of numbers over the ranks"""
    from onereel_b200 import dist as D
    if D.world() == 1:
        return list(vals)
    import torch.distributed as dist
    t = torch.tensor(vals, dtype=dtype, device=torch.device('cuda', torch.cuda.current_device()))
    dist.all_reduce(t, op={'max': dist.ReduceOp.MAX, 'sum': dist.ReduceOp.SUM, 'min': dist.ReduceOp.MIN}[op],
                    group=D.group())
    return t.tolist()


# ------------------------------------------------------------------------------------------------ one layer

class LayerBench:
    """one scene-attention layer on this rank through hunyuan15.Processor (scene or Ulysses by the plan)"""

    def __init__(self, cfg, mode, overlap, dev, exchange='peer'):
        from onereel_b200 import dist as D, hunyuan15 as HY
        self.cfg, self.dev = cfg, dev
        self.rank, self.world = D.rank(), D.world()
        self.lay = lay = cfg_layout(cfg)
        self.T, self.H, self.Dh = cfg['T'], cfg['heads'], cfg['dim']
        self.counts = [cfg['text']] * lay.n_scenes
        self.ctx = HY.Context(lay, mode=mode, T=self.T, counts={True: self.counts, False: self.counts}, fwd=1,
                              overlap=overlap, exchange=exchange)
        HY.plan_parallel(self.ctx, self.H)
        self.proc = HY.Processor(self.ctx, 0)
        self.own = tuple(self.ctx.own[self.rank])
        self.full = full_inputs(lay, self.T, self.counts, self.H, self.Dh, dev)
        a, b = self.own
        q, k, v, eq, ek, ev = self.full
        self.inputs = [q[a:b].contiguous(), k[a:b].contiguous(), v[a:b].contiguous(), eq, ek, ev]
        self.stream = torch.cuda.current_stream(dev)
        self._peer_kv = None

    def step(self, inputs=None):
        x = self.inputs if inputs is None else inputs
        if self.ctx.run_mode == 'ulysses':
            return self.proc.ulysses(*x)
        if inputs is None and self.world > 1 and self.ctx.exchange == 'peer':
            # the layer's K / V as a producer that writes them into the exchange buffer of the generation the
            # exchange uses next (both generations hold the same resident inputs, written once)
            from onereel_b200 import comm, peer
            if comm.PEER_UNAVAILABLE is None:
                if self._peer_kv is None:
                    # before this rank's first barrier on this buffer, so no peer reads it yet
                    sp = peer.space_for(max(b - a for a, b in self.ctx.own), self.H * self.Dh, x[1].dtype, self.dev)
                    nr = x[1].shape[0]
                    for buf, _, _ in sp.gens:
                        buf[0, :nr].copy_(x[1].reshape(nr, -1))
                        buf[1, :nr].copy_(x[2].reshape(nr, -1))
                    self._peer_kv = True
                kk, vv = peer.kv_inputs(self.ctx.own, self.H, self.Dh, x[1].dtype, self.dev)
                x = [x[0], kk, vv] + list(x[3:])
        return self.proc.scene(*x)

    def release_full(self):
        self.full = None

    def time(self, warmup, steps, clocks=True):
        """W untimed steps, one instrumented step (useful FLOPs of this rank's launches), then K steps timed with CUDA
        events on the launching stream between barriers; returns per-rank figures"""
        from onereel_b200 import attention as A, dist as D, scene as S
        from onereel_b200.pack import RunTable
        for _ in range(warmup):
            self.step()
        torch.cuda.synchronize()
        A.check()
        S.TIMING = []
        self.step()
        torch.cuda.synchronize()
        rank_flops = sum(f for _, _, f in S.TIMING)
        S.TIMING = None
        clk = Clocks(torch.cuda.current_device()) if clocks else None
        if clk:
            clk.__enter__()
        try:
            D.barrier()
            torch.cuda.synchronize()
            S.TIMING = []
            packs0, attn0 = RunTable.launches, A.LAUNCHES
            t0, t1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            t0.record(self.stream)
            for _ in range(steps):
                self.step()
            t1.record(self.stream)
            torch.cuda.synchronize()
            D.barrier()
        finally:
            if clk:
                clk.__exit__()
        timing, S.TIMING = S.TIMING, None
        A.check()
        return dict(ms=t0.elapsed_time(t1) / steps, attn_ms=sum(a.elapsed_time(b) for a, b, _ in timing) / steps,
                    rank_flops=rank_flops, launches=A.LAUNCHES - attn0 + RunTable.launches - packs0,
                    clocks=clk.summary() if clk else None)

    def attn_alg_bytes(self):
        """algorithmic bytes of the attention launches of one step on this rank: every query row read and its output
        written once, every segment's keys and values read once per head"""
        if self.ctx.run_mode != 'scene':
            return 0
        p = self.proc._plan(self.H, self.Dh, self.dev, self.ctx.overlap == 'lse')
        tot = 0
        for pl in (p.near, p.far, p.far_local, p.far_remote):
            if pl is not None:
                tot += sum(2 * a + 2 * b for a, b in zip(pl.lq, pl.lk)) * self.H * self.Dh * 2
        return tot

    def parity(self, fp32_rows=16):
        """the timed path's outputs on this rank against (1) the same rows computed as one GPU computes them, on this
        rank from the full inputs (the rank's scene pieces with every key local; the text segments of every scene it
        touches) and (2) fp32 attention on `fp32_rows` evenly spaced query rows of every segment. Reduced over ranks."""
        from onereel_b200 import scene as S
        lay, T, H, Dh = self.lay, self.T, self.H, self.Dh
        from onereel_b200 import attention as A
        a, b = self.own
        splits0 = A.SPLITS
        ov, ot = self.step()
        torch.cuda.synchronize()
        split = A.SPLITS > splits0              # a coarse Ulysses launch took the key split (LSE merge)
        q, k, v, eq, ek, ev = self.full
        L = lay.n_frames * T
        mine, _ = S.pieces(lay, T, self.own)
        touch = {j for j, _ in mine}
        plan = S.ScenePlan(S.scene_segments(lay, T, self.counts, mine, touch, (0, L)), H * Dh * 2, H, self.dev)
        kp, vp = plan.pack_kv(k, v, ek, ev)
        ref_v, ref_t = torch.zeros_like(q), torch.zeros_like(eq)
        S.attend_segments(plan, q, eq, kp, vp, ref_v, ref_t)
        tr = S.text_ranges(self.counts)
        trows = torch.cat([torch.arange(*tr[j]) for j in sorted(touch)] or [torch.zeros(0, dtype=torch.long)])
        trows = trows.to(self.dev)
        got = torch.cat([ov.flatten(), ot[trows].flatten()])
        want = torch.cat([ref_v[a:b].flatten(), ref_t[trows].flatten()])
        bit = bool(torch.equal(got, want))
        d = (got.float() - want.float()).abs()
        mx, sm, n = d.max().item() if d.numel() else 0.0, d.sum().item(), d.numel()
        # fp32 on sampled rows of every segment
        fmx, fsm, fn, frows = 0.0, 0.0, 0, 0
        scale = Dh ** -0.5
        for i, sg in enumerate(plan.segs):
            pick = torch.linspace(0, sg.lq - 1, min(sg.lq, fp32_rows)).round().long().unique().to(self.dev)
            q0 = sg.q[1]
            qq = (q if sg.kind == 'v' else eq)[q0 + pick].float()
            k0, kl = plan.cu_k[i], plan.lk[i]
            if kl == 0:
                ref = torch.zeros_like(qq)
            else:
                s = torch.einsum('qhd,khd->hqk', qq, kp[k0:k0 + kl].float()) * scale
                ref = torch.einsum('hqk,khd->qhd', torch.softmax(s, -1), vp[k0:k0 + kl].float())
            o = (ov[q0 - a + pick] if sg.kind == 'v' else ot[q0 + pick]).float()
            e = (o - ref).abs()
            fmx, fsm, fn, frows = max(fmx, e.max().item()), fsm + e.sum().item(), fn + e.numel(), frows + len(pick)
        del kp, vp, ref_v, ref_t
        mx, fmx = reduce([mx, fmx], 'max')
        sm, n, fsm, fn, frows, rows = reduce([sm, n, fsm, fn, frows, (b - a) + len(trows)], 'sum')
        bit = bool(reduce([1.0 if bit else 0.0], 'min')[0])
        split = bool(reduce([1.0 if split else 0.0], 'max')[0])
        expect_bit = ((self.ctx.run_mode == 'ulysses' and not split) or
                      (self.ctx.run_mode != 'ulysses' and not (self.ctx.overlap == 'lse' and self.world > 1)))
        fp32 = dict(max_abs=fmx, mean_abs=fsm / max(fn, 1), rows=int(frows), tolerance=[MAX_ABS, MEAN_ABS])
        ok_fp32 = fmx <= MAX_ABS and fp32['mean_abs'] <= MEAN_ABS
        ok_1gpu = bit if expect_bit else (mx <= MAX_ABS and sm / max(n, 1) <= MEAN_ABS)
        return dict(path=self.ctx.run_mode, overlap=self.ctx.overlap, key_split=split, ok=bool(ok_fp32 and ok_1gpu),
                    one_gpu=dict(bit_exact=bit, expected_bit_exact=expect_bit, max_abs=mx, mean_abs=sm / max(n, 1),
                                 rows=int(rows), what='the rank\'s video rows and the text rows of every scene it '
                                                      'touches, recomputed as one GPU computes them'),
                    fp32=fp32)

    def phases(self, steps):
        """device time per phase of the step on every rank (events on the compute stream; 'exchange_wait' = the time
        the compute stream stood waiting for the K/V exchange), mean over steps: a list indexed by rank"""
        from onereel_b200 import hunyuan15 as HY
        names = ['exchange', 'near', 'far_local', 'exchange_wait', 'far', 'far_remote', 'text_sync', 'a2a_in',
                 'attention', 'a2a_out']
        HY.PHASES = []
        for _ in range(steps):
            self.step()
        torch.cuda.synchronize()
        marks, HY.PHASES = HY.PHASES, None
        acc = dict.fromkeys(names, 0.0)
        total = 0.0
        start = None
        prev = None
        for name, e in marks:
            if name == 'start':
                if start is not None:
                    total += start.elapsed_time(prev)
                start = prev = e
                continue
            acc[name] += prev.elapsed_time(e)
            prev = e
        total += start.elapsed_time(prev)
        mine = {n: round(acc[n] / steps, 4) for n in names if acc[n] > 0}
        mine['step'] = round(total / steps, 4)
        from onereel_b200 import dist as D
        return D.all_gather_object(mine)

    def comm(self, steps=10):
        """the K/V exchange of one layer timed alone (posted and waited on the compute stream), its bytes per GPU, and
        the text-row sync bytes; gathering path only"""
        from onereel_b200 import comm, dist as D
        if self.world == 1 or self.ctx.run_mode != 'scene':
            return None
        lay, T, own_all, r = self.lay, self.T, self.ctx.own, self.rank
        k, v = self.inputs[1], self.inputs[2]
        kind = self.ctx.exchange
        for _ in range(3):
            comm.kv_exchange(kind, lay, own_all, T, k, v).wait()
        torch.cuda.synchronize()
        D.barrier()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record(self.stream)
        for _ in range(steps):
            comm.kv_exchange(kind, lay, own_all, T, k, v).wait()
        e1.record(self.stream)
        torch.cuda.synchronize()
        D.barrier()
        ms = e0.elapsed_time(e1) / steps
        need, common, p2p = comm.exchange_plan(lay, own_all, T)
        n = len(own_all)
        rows_in = sum(hi - lo for p in range(n) if p != r for lo, hi in comm.clip(need[r], *own_all[p]))
        rows_out = (sum(hi - lo for q in range(n) if q != r for lo, hi in p2p[(r, q)]) +
                    sum(hi - lo for lo, hi in common[r]))
        bcast = sum(hi - lo for p in range(n) for lo, hi in common[p])
        rb = 2 * self.H * self.Dh * 2                      # K and V rows
        # text rows of send_text_rows: scene j's text outputs from the owner of its first frame to the others
        t_in = t_out = 0
        touches = lambda p, lo, hi: lo * T < own_all[p][1] and hi * T > own_all[p][0]
        from onereel_b200 import scene as S
        for (lo, hi), (t0, t1) in zip(lay.ranges, S.text_ranges(self.counts)):
            src = next(p for p in range(n) if own_all[p][0] <= lo * T < own_all[p][1])
            peers = [p for p in range(n) if p != src and touches(p, lo, hi)]
            if src == r:
                t_out += len(peers) * (t1 - t0)
            elif r in peers:
                t_in += t1 - t0
        ms_max, = reduce([ms], 'max')
        b_in, b_out, tb_in, tb_out = reduce([rows_in * rb, rows_out * rb, t_in * rb // 2, t_out * rb // 2], 'max')
        if kind == 'peer' and comm.PEER_UNAVAILABLE is None:
            # rows this rank serves: every pull whose source is this rank, in either stage of every rank's plan
            from onereel_b200 import peer
            # (tables built on the host with 16-byte rows, the smallest row the pack accepts; served counts rows)
            plans = [peer._Plan(lay, own_all, T, (), q, 'cpu', 16) for q in range(n)]
            served = sum(nb // 16 for pl in plans for tab in (pl.stage1, pl.stage2) if tab is not None
                         for src, nb in zip(tab.src_slot, tab.nbytes_list) if src == r)
            b_in, b_out = reduce([rows_in * rb, served * rb], 'max')
            note = ('K and V of this rank copied into its symmetric buffer, device barrier, every interval pulled '
                    'over NVLink (TMA bulk copies); rows every rank reads in two stages (a stripe from the owner, '
                    'the rest from the other readers); bytes per GPU and direction, max over ranks')
        else:
            kind = 'nccl'
            note = ('grouped NCCL send/recv of K and V plus the broadcast of rows every rank reads; bytes per GPU '
                    'and direction, max over ranks (a broadcast counted once at its root)')
        return dict(exchange=dict(kind=kind, ms_alone=ms_max, bytes_in_max=b_in, bytes_out_max=b_out,
                                  broadcast_rows=bcast, note=note),
                    text_rows=dict(bytes_in_max=tb_in, bytes_out_max=tb_out))


def nccl_peaks(dev, mib=256, iters=8):
    """measured NCCL bandwidth between this node's GPUs: pairwise send/recv (rank r <-> r ^ 1, every pair at once; GB/s
    per direction per GPU) and all-to-all (GB/s of data each GPU sends to the others), max time over ranks"""
    import torch.distributed as dist
    from onereel_b200 import dist as D
    r, n = D.rank(), D.world()
    if n < 2:
        return None
    nbytes = mib << 20
    s = torch.empty(nbytes, dtype=torch.uint8, device=dev)
    rcv = torch.empty_like(s)
    g = D.group()
    partner = r ^ 1

    def pair():
        if partner < n:
            for w in dist.batch_isend_irecv([dist.P2POp(dist.isend, s, partner, group=g),
                                             dist.P2POp(dist.irecv, rcv, partner, group=g)]):
                w.wait()

    def a2a():
        dist.all_to_all_single(rcv, s, group=g)

    out = {}
    stream = torch.cuda.current_stream(dev)
    for name, fn, moved in (('p2p_gbs', pair, nbytes), ('a2a_gbs', a2a, nbytes * (n - 1) / n)):
        for _ in range(2):
            fn()
        torch.cuda.synchronize()
        D.barrier()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record(stream)
        for _ in range(iters):
            fn()
        e1.record(stream)
        torch.cuda.synchronize()
        ms, = reduce([e0.elapsed_time(e1) / iters], 'max')
        out[name] = moved / (ms * 1e-3) / 1e9
    out['size_mib'] = mib
    return out


# ------------------------------------------------------------------------------------------------ e2e leg

def e2e_leg(lb, steps):
    """end to end through the public processor API with host buffers: every step copies its layer's local q/k/v and
    the text q/k/v host->device from pinned memory, calls the processor, and copies its outputs device->host. Steps
    are pipelined the way a caller streaming layers would run them: two device input buffers, H2D on one copy stream,
    D2H on another, so step i+1's inputs travel while step i computes and step i-1's outputs return."""
    from onereel_b200 import attention as A, dist as D
    dev, stream = lb.dev, lb.stream
    src = lb.inputs
    host_in = [x.cpu().pin_memory() for x in src]
    dev_in = [[torch.empty_like(x) for x in src] for _ in range(2)]
    host_out = [[torch.empty(src[0].shape, dtype=src[0].dtype, pin_memory=True),
                 torch.empty(src[3].shape, dtype=src[3].dtype, pin_memory=True)] for _ in range(2)]
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
        ov, ot = lb.step(dev_in[b])
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
    D.barrier()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record(s_in)
    for i in range(steps):
        e2e_step(i)
    e1.record(s_out)
    torch.cuda.synchronize()
    D.barrier()
    A.check()
    ms, = reduce([e0.elapsed_time(e1) / steps], 'max')
    h2d = sum(x.numel() * x.element_size() for x in host_in)
    d2h = sum(x.numel() * x.element_size() for x in host_out[0])
    return ms, h2d, d2h


# ------------------------------------------------------------------------------------------------ legs

def kernels_leg(lb, dev, warmup=3, steps=10):
    """the HBM-bound kernels of the path on the cfg2 layer, each timed alone with CUDA events on its stream (inputs
    larger than L2), against the measured copy bandwidth: the K/V pack, the fused q/k RMSNorm + RoPE, the two LSE
    merges, the frame-memory pooling. bytes = algorithmic bytes per launch (every byte the kernel must read and
    write once)."""
    from onereel_b200 import attention as A, frame_memory as FM, rope
    from onereel_b200.layout import SceneLayout
    _, _, hbm, kind = peaks()
    stream = torch.cuda.current_stream(dev)
    q, k, v, eq, ek, ev = lb.inputs
    H, Dh = lb.H, lb.Dh
    plan = lb.proc._plan(H, Dh, dev, False).near
    res = {}

    def timed(name, fn, nbytes, what):
        for _ in range(warmup):
            fn()
        torch.cuda.synchronize()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record(stream)
        for _ in range(steps):
            fn()
        e1.record(stream)
        torch.cuda.synchronize()
        ms = e0.elapsed_time(e1) / steps
        gbs = nbytes / (ms * 1e-3) / 1e9
        res[name] = dict(ms=ms, bytes=nbytes, achieved_gbs=gbs, peak_gbs=hbm, frac=gbs / hbm, what=what)

    kp, vp = plan.pack_kv(k, v, ek, ev)
    timed('pack', lambda: plan.pack_kv(k, v, ek, ev, out=(kp, vp)), 2 * 2 * kp.numel() * 2,
          'orl_pack: K and V of every cfg2 segment gathered into the packed layout (read + write of every key row)')
    del kp, vp
    rows = q.shape[0]
    x = q.reshape(rows, H * Dh)
    w = torch.ones(Dh, dtype=torch.bfloat16, device=dev)
    cos = torch.rand(rows, Dh, device=dev)
    sin = torch.rand(rows, Dh, device=dev)
    y = torch.empty_like(q)
    timed('qk_norm_rope', lambda: rope.qk_norm_rope(x, w, cos, sin, H, 1e-6, True, 0, out=y),
          rows * H * Dh * 2 * 2 + rows * Dh * 4 * 2,
          "orl_qk_norm_rope on the layer's video rows (Hunyuan per-head RMSNorm + RoPE): read x, cos, sin; write y")
    del y, cos, sin
    n = rows
    o1, o2 = q.clone(), k.clone()
    l1 = torch.randn(H, n, device=dev)
    l2 = torch.randn(H, n, device=dev)
    timed('lse_merge', lambda: A.lse_merge(o1, l1, o2, l2), 3 * n * H * Dh * 2 + 3 * n * H * 4,
          "orl_lse_merge of two bf16 partial outputs of the layer's video rows (read o1, o2, both lse; write o1, lse)")
    acc = o1.float()
    del o1
    timed('lse_merge_acc', lambda: A.lse_merge_acc(acc, l1, o2, l2),
          2 * n * H * Dh * 4 + n * H * Dh * 2 + 3 * n * H * 4,
          'orl_lse_merge_acc into an fp32 accumulator (Scene-Ring step): read + write acc, read the bf16 part')
    del acc, o2
    C = 2048
    hs = torch.randn(n, C, device=dev).to(torch.bfloat16)
    frame = (torch.arange(n, device=dev) // lb.T).to(torch.int64)
    fm = FM.FrameMemory(budget=4)
    fm.reset(SceneLayout(list(lb.lay.lengths), halo=0), n_layers=1)
    timed('frame_pool', lambda: fm.collect(frame, hs, layer=0), n * C * 2,
          "orl_frame_pool: per-frame sums of one layer's hidden states [rows, 2048] bf16 (read once)")
    return dict(kernels=res, peak_source=f'{kind} HBM copy bandwidth ({hbm:.0f} GB/s)')


def fa2_leg(dev, warmup=3, steps=10):
    """the reference's own GPU kernel on the same packed cfg2 segments, for a GPU-to-GPU comparison: FlashAttention-2
    2.8.3 varlen (src/onereel/attention.py:39-43 with BACKEND 'fa2'), against this kernel on the same packed q / k / v;
    also the max / mean abs difference of the two outputs. Returns None when flash_attn is not importable or fails."""
    try:
        import flash_attn
        from flash_attn import flash_attn_varlen_func
    except Exception as e:                                  # not installed, or no kernel image for this GPU
        return dict(unavailable=f'{type(e).__name__}: {e}'[:200])
    from onereel_b200 import attention as A, scene as S
    cfg = CFG2
    lay = cfg_layout(cfg)
    T, H, Dh = cfg['T'], cfg['heads'], cfg['dim']
    counts = [cfg['text']] * lay.n_scenes
    q, k, v, eq, ek, ev = full_inputs(lay, T, counts, H, Dh, dev)
    L = lay.n_frames * T
    mine = [(j, (lo * T, hi * T)) for j, (lo, hi) in enumerate(lay.ranges)]
    plan = S.ScenePlan(S.scene_segments(lay, T, counts, mine, set(range(lay.n_scenes)), (0, L)), H * Dh * 2, H, dev)
    kp, vp = plan.pack_kv(k, v, ek, ev)
    qp = torch.cat([(q if s_.kind == 'v' else eq)[s_.q[1]:s_.q[2]] for s_ in plan.segs])
    del q, k, v
    cu_q = torch.tensor(plan.cu_q, dtype=torch.int32, device=dev)
    cu_k = torch.tensor(plan.cu_k, dtype=torch.int32, device=dev)
    flops = sum(4.0 * a * b * H * Dh for a, b in zip(plan.lq, plan.lk))
    runs = dict(fa2=lambda: flash_attn_varlen_func(qp, kp, vp, cu_q, cu_k, max(plan.lq), max(plan.lk)),
                b200=lambda: A.attend(qp, kp, vp, plan.cu_q[:-1], plan.lq, plan.cu_k[:-1], plan.lk)[0])
    res = dict(kernel=f'flash_attn {flash_attn.__version__} flash_attn_varlen_func (the reference\'s fa2 backend)',
               workload='cfg2 packed segments (q packed, K/V packed), one call')
    stream = torch.cuda.current_stream(dev)
    try:
        for name, fn in runs.items():
            for _ in range(warmup):
                fn()
            torch.cuda.synchronize()
            e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            e0.record(stream)
            for _ in range(steps):
                fn()
            e1.record(stream)
            torch.cuda.synchronize()
            ms = e0.elapsed_time(e1) / steps
            res[name] = dict(ms=ms, tflops=flops / (ms * 1e-3) / 1e12)
        d = (runs['fa2']().float() - runs['b200']().float()).abs()
        res['b200_vs_fa2'] = dict(max_abs=d.max().item(), mean_abs=d.mean().item(), tolerance=[MAX_ABS, MEAN_ABS])
        res['speedup'] = res['fa2']['ms'] / res['b200']['ms']
    except Exception as e:
        res['unavailable'] = f'{type(e).__name__}: {e}'[:200]
    A.check()
    return res


def cfg3_leg(dev, world, warmup=3, steps=50):
    """BASELINE cfg3 over the N GPUs (strong scaling): each parallel mode timed, with its parity"""
    from onereel_b200 import attention as A
    modes = ['scene'] if world == 1 else ['scene', 'ulysses', 'auto']
    res = {}
    for mode in modes:
        lb = LayerBench(CFG3, mode, 'none', dev)
        t = lb.time(warmup, steps, clocks=False)
        ms, attn_ms = reduce([t['ms'], t['attn_ms']], 'max')
        flops, = reduce([t['rank_flops']], 'sum')
        par = lb.parity()
        ph = lb.phases(5)
        res[mode] = dict(run_mode=lb.ctx.run_mode, tflops=flops / (ms * 1e-3) / 1e12, ms_per_step=ms,
                         attention_ms_max=attn_ms, useful_tflop=flops / 1e12, phases_ms=ph, parity=par)
        if mode == 'auto' or world == 1:
            res['eq2'] = dict(lb.ctx.path) if lb.ctx.path else None
        del lb
        torch.cuda.empty_cache()
        A.check()
    res['workload'] = ('cfg3: one Wan2.2-TI2V-5B-shaped layer (6 scenes [3,12,5,9,4,8] x 880 tokens per frame, 256 '
                       'text tokens per scene, frame memory {0,3,15,20}, 24 x 128 heads, bf16) through the joint '
                       '[video | text] scene path of hunyuan15.Processor, sharded over N (strong scaling)')
    return res


def dit_leg(dev, world, rank, warmup=3, steps=3):
    """BASELINE cfg4: one denoising step (conditional + unconditional forward of 54 blocks) of the random-init
    HunyuanVideo-1.5-architecture stand-in (onereel_b200/standin.py) on this rank's video rows, scene-parallel
    attention through the B200 processors; latency = device time of the step, max over ranks (strong scaling)"""
    from onereel_b200 import attention as A, dist as D, hunyuan15 as HY, standin
    cfg = CFG4
    lay = cfg_layout(cfg)
    T, H, Dh, C = cfg['T'], cfg['heads'], cfg['dim'], cfg['hidden']
    counts = [cfg['text']] * lay.n_scenes
    ctx = HY.Context(lay, mode='auto', T=T, counts={True: counts, False: counts}, overlap='none')
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
    for _ in range(warmup):
        standin.dit_step(model, ctx, hs, ehs_c, ehs_u, temb, rot)
    torch.cuda.synchronize()
    A.check()
    with Clocks(torch.cuda.current_device()) as clk:
        D.barrier()
        t0, t1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        t0.record(stream)
        for _ in range(steps):
            standin.dit_step(model, ctx, hs, ehs_c, ehs_u, temb, rot)
        t1.record(stream)
        torch.cuda.synchronize()
        D.barrier()
    A.check()
    ms, = reduce([t0.elapsed_time(t1) / steps], 'max')
    tokens = L + Nt
    gemm = 2 * cfg['blocks'] * 24 * C * C * tokens
    segs = [(s_.lq, s_.lk) for s_ in HY.S.scene_segments(lay, T, counts, [(j, (lo * T, hi * T)) for j, (lo, hi)
                                                        in enumerate(lay.ranges)], set(range(lay.n_scenes)), (0, L))]
    attn = 2 * cfg['blocks'] * sum(4.0 * x * y * H * Dh for x, y in segs)
    del model
    torch.cuda.empty_cache()
    return dict(ms=ms, steps=steps, warmup=warmup, scaling='strong', run_mode=ctx.run_mode, path=ctx.path,
                workload='cfg4: one denoising step (2 CFG forwards x 54 blocks) of the random-init '
                         'HunyuanVideo-1.5-architecture stand-in (hidden 2048, 16 x 128 heads), 4 scenes x 31 '
                         'latent frames x 1590 tokens, 128 text tokens per scene, frame memory 4, bf16',
                flop_per_step=dict(gemm=gemm, attention=attn), achieved_tflops=(gemm + attn) / (ms * 1e-3) / 1e12,
                clocks=clk.summary())


# ------------------------------------------------------------------------------------------------ main

def setup():
    from onereel_b200 import dist as D
    from onereel_b200.csrc.build import build
    rank, world, local = dist_env()
    if rank == 0:
        build()
    D.init('nccl', timeout_s=180.0)
    if world > 1:
        D.barrier()
        build()                      # other ranks load the library rank 0 built
    return rank, world, local, torch.device('cuda', local)


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument('--gpus', type=int, default=1)
    ap.add_argument('--steps', type=int, default=20)
    ap.add_argument('--warmup', type=int, default=5)
    ap.add_argument('--impl', default='ours', choices=['ours', 'reference'])
    ap.add_argument('--mode', default='auto',
                    help='parallel path of the headline for N > 1: auto (the Eq. 2 chooser), scene or ulysses')
    ap.add_argument('--overlap', default='auto', choices=['auto', 'none', 'lse'],
                    help="K/V gathering: 'lse' attends far scenes to their local keys while the exchange is in flight "
                         "and merges by log-sum-exp (Context.overlap of the reference); 'auto' takes 'lse' from 4 "
                         "GPUs up (measured on 8 B200: +8 %% on the weak cfg2 layer; on 2 the two are even)")
    ap.add_argument('--exchange', default='peer', choices=['peer', 'nccl'],
                    help='K/V exchange of the gathering path: over peer memory (symmetric buffers, device barrier, '
                         'one pull launch) or NCCL send/recv (the reference scheme)')
    ap.add_argument('--legs', default=','.join(LEGS),
                    help=f'extra measurements in the line (comma list of {", ".join(LEGS)}; "none" for none)')
    ap.add_argument('--no-cpu-baseline', action='store_true')
    ap.add_argument('--no-e2e', action='store_true', help='skip the host-buffer end-to-end leg')
    ap.add_argument('--dit-steps', type=int, default=3)
    ap.add_argument('--scenes', default='16', help='cfg5: scene counts to sweep (comma list)')
    ap.add_argument('--workload', default='cfg2', choices=['cfg2', 'small', 'cfg3', 'cfg4', 'cfg5'],
                    help='cfg2 (default: the full line); small: the first two scenes of cfg2, one line, for profiler '
                         'captures; cfg3 / cfg4: that leg alone; cfg5: Wan-shaped stress layer with --scenes S')
    args = ap.parse_args()
    if args.impl == 'reference':
        return run_reference(args)
    rank, world, local, dev = setup()
    from onereel_b200 import dist as D
    try:
        if args.workload == 'cfg5':
            for sc in args.scenes.split(','):
                run_wan_stress(args, int(sc), dev, rank, world)
        elif args.workload == 'cfg4':
            r = dit_leg(dev, world, rank, warmup=args.warmup, steps=args.steps)
            if rank == 0:
                print(json.dumps(dict(metric='DiT step latency (cfg4)', value=r['ms'], unit='ms', n_gpus=world,
                                      higher_is_better=False, **r)), flush=True)
        elif args.workload == 'cfg3':
            r = cfg3_leg(dev, world, args.warmup, args.steps)
            if rank == 0:
                print(json.dumps(dict(metric='cfg3 scene attention TFLOP/s', n_gpus=world, cfg3=r)), flush=True)
        else:
            run_headline(args, dev, rank, world, local)
    finally:
        D.shutdown()


def run_headline(args, dev, rank, world, local):
    from onereel_b200 import attention as A
    legs = set() if args.legs == 'none' else set(args.legs.split(','))
    cfg = dict({'cfg2': CFG2, 'small': SMALL}[args.workload])
    # weak scaling: N GPUs run cfg2's scene set repeated N times (per-GPU work about fixed); every scene reads the
    # frame memory of the first copy, so ranks exchange those rows (the path's real K/V gathering step)
    cfg['lengths'] = cfg['lengths'] * world
    # the LSE split hides an NCCL exchange from 4 GPUs up; the peer-memory pull is short and runs before attention
    overlap = args.overlap if args.overlap != 'auto' else ('lse' if world >= 4 and args.exchange == 'nccl' else 'none')
    lb = LayerBench(cfg, args.mode, overlap, dev, args.exchange)
    t = lb.time(args.warmup, args.steps)
    ms, attn_ms_max = reduce([t['ms'], t['attn_ms']], 'max')
    total_flops, = reduce([t['rank_flops']], 'sum')
    attn_bytes = lb.attn_alg_bytes()
    extra = {}
    if 'parity' in legs:
        extra['parity'] = lb.parity()
    if 'phases' in legs:
        extra['phases_ms'] = lb.phases(max(3, args.steps // 4))
    comm = lb.comm() if 'comm' in legs and world > 1 else None
    e2e = None
    if not args.no_e2e:
        e2e_ms, h2d, d2h = e2e_leg(lb, max(4, args.steps // 4))
        e2e = dict(value=total_flops / (e2e_ms * 1e-3) / 1e12, unit='TFLOP/s', ms_per_step=e2e_ms,
                   h2d_bytes_per_step=h2d, d2h_bytes_per_step=d2h,
                   note='processor call with pinned H2D inputs / D2H outputs every step; consecutive steps '
                        'pipelined on separate copy streams (double-buffered inputs)')
    if 'kernels' in legs and world == 1:
        extra['hbm_kernels'] = kernels_leg(lb, dev)
    run_mode, path, own = lb.ctx.run_mode, lb.ctx.path, lb.ctx.own
    from onereel_b200 import comm as _comm
    exch = ('peer memory (symmetric buffers, device barrier, TMA bulk pull)'
            if args.exchange == 'peer' and _comm.PEER_UNAVAILABLE is None else 'NCCL send/recv')
    layout = dict(cfg, scenes=lb.lay.n_scenes)
    del lb
    torch.cuda.empty_cache()
    peaks_nccl = nccl_peaks(dev) if 'comm' in legs and world > 1 else None
    if comm is not None:
        comm['nccl_peaks'] = peaks_nccl
    if 'cfg3' in legs:
        extra['cfg3'] = cfg3_leg(dev, world)
    if 'dit' in legs:
        extra['dit_step'] = dit_leg(dev, world, rank, steps=args.dit_steps)
    if 'fa2' in legs and rank == 0 and world == 1:
        extra['reference_gpu_kernel'] = fa2_leg(dev)
    A.check()
    if rank != 0:
        return
    peak_burst, peak_sus, hbm, peak_kind = peaks()
    achieved = t['rank_flops'] / (t['attn_ms'] * 1e-3) / 1e12
    cb = None
    if not args.no_cpu_baseline and args.workload == 'cfg2' and world == 1:
        cb, _ = cpu_baseline()
    roof_nv = None
    if comm is not None:
        ex = comm['exchange']
        b = max(ex['bytes_in_max'], ex['bytes_out_max'])
        ach = b / (ex['ms_alone'] * 1e-3) / 1e9
        waits = [ph.get('exchange_wait', 0.0) for ph in extra.get('phases_ms', [])]
        roof_nv = dict(bound='nvlink', achieved=ach, peak=NVLINK_PEER_GBS, unit='GB/s', frac=ach / NVLINK_PEER_GBS,
                       bytes=b, frac_of_nccl_p2p=(ach / peaks_nccl['p2p_gbs']) if peaks_nccl else None,
                       what='K/V exchange of the headline layer timed alone: the busiest GPU\'s bytes in one direction '
                            '/ exchange time; peak = the pool\'s measured NVLink peer copy per direction (nominal 900)',
                       exposed_wait_ms_max=max(waits) if waits else None)
    line = dict(metric=METRIC, value=total_flops / (ms * 1e-3) / 1e12, unit='TFLOP/s', n_gpus=world,
                steps=args.steps, warmup=args.warmup, ms_per_step=ms, higher_is_better=True, scaling='weak',
                vs_baseline=None, dtype='bf16', data='synthetic (seeded; Q/K RMS-normed N(0,1), V N(0,1))',
                value_per_gpu=total_flops / (ms * 1e-3) / 1e12 / world,
                config=dict(workload=(f'{args.workload}: one HunyuanVideo-1.5-shaped scene-attention layer through '
                                      'hunyuan15.Processor (pack K/V + attention' +
                                      (f', K/V exchange over {exch}' if world > 1 else '') + ')'),
                            layout=layout, run_mode=run_mode, path=path, overlap=overlap, own=own,
                            useful_tflop_per_step=total_flops / 1e12,
                            useful_tflop_per_gpu=total_flops / 1e12 / world,
                            parallelism=(f'{run_mode} x{world} (weak: cfg2 scene set repeated per GPU)'
                                         if world > 1 else 'single'),
                            value_note='value = whole-job TFLOP/s over the N GPUs; value_per_gpu = value / N',
                            l2='inputs larger than L2 (q/k/v 203 MB each per GPU, packed K/V ~486 MB each)'),
                e2e=e2e,
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
                roofline_nvlink=roof_nv, comm=comm,
                gpu_launches=t['launches'], clocks=t['clocks'], cpu_baseline=cb, **extra)
    print(json.dumps(line), flush=True)


def run_wan_stress(args, n_scenes, dev, rank, world):
    """BASELINE cfg5: one Wan-shaped self-attention layer (no joint text) of S scenes x 31 frames, strong-scaled"""
    from onereel_b200 import attention as A, comm, dist as D, scene as S, wan as WN
    cfg = dict(CFG5, lengths=[CFG5['scene_frames']] * n_scenes,
               memory=[j * CFG5['scene_frames'] for j in range(min(4, n_scenes))])
    lay = cfg_layout(cfg)
    T, H, Dh = cfg['T'], cfg['heads'], cfg['dim']
    ctx = WN.Context(lay, mode=args.mode, T=T)
    WN.plan_parallel(ctx, H)
    wproc = WN.Processor(ctx, 'self', None, 0)
    a, b = ctx.own[rank]
    q, k, v, _, _, _ = full_inputs(lay, T, [0] * lay.n_scenes, H, Dh, dev)
    q, k, v = q[a:b].contiguous(), k[a:b].contiguous(), v[a:b].contiguous()

    def step():
        if ctx.run_mode == 'ulysses' or world == 1:
            return comm.a2a_tokens(wproc.ranges(comm.a2a_heads(q), comm.a2a_heads(k), comm.a2a_heads(v)))
        return wproc.scene(q, k, v)
    for _ in range(args.warmup):
        step()
    torch.cuda.synchronize()
    S.TIMING = []
    step()
    torch.cuda.synchronize()
    flops = sum(f for _, _, f in S.TIMING)
    S.TIMING = None
    D.barrier()
    stream = torch.cuda.current_stream(dev)
    t0, t1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    t0.record(stream)
    for _ in range(args.steps):
        step()
    t1.record(stream)
    torch.cuda.synchronize()
    D.barrier()
    A.check()
    ms, = reduce([t0.elapsed_time(t1) / args.steps], 'max')
    total, = reduce([flops], 'sum')
    if rank == 0:
        print(json.dumps(dict(metric='cfg5 Wan-shaped stress layer TFLOP/s', value=total / (ms * 1e-3) / 1e12,
                              unit='TFLOP/s', n_gpus=world, ms_per_step=ms, scenes=n_scenes, run_mode=ctx.run_mode,
                              path=ctx.path, scaling='strong')), flush=True)


if __name__ == '__main__':
    main()
