"""The reference's CPU path of the scene-packed attention layer — TEST / BASELINE INFRASTRUCTURE ONLY.

The CPU baseline is the reference's own scene processor (src/onereel/models/hunyuan15.py:212-251 with
`_segments` 153-170 and attention.packed 65-71) with the FlashAttention varlen call replaced by per-segment fp32
`torch.nn.functional.scaled_dot_product_attention` on the host cores. This module restates that path on the CPU:
gather each segment's rows (the reference's torch.cat), one fp32 SDPA per segment, scatter the outputs. It is what
`bench.py --impl reference` and the `cpu_baseline` leg time; it never runs inside the product.
"""
from __future__ import annotations

import os
import time

import torch

from oracle import layout_oracle as LO


def segment_index(lay, T, counts, own=None):
    """per packed segment: (kind, query row index tensor, key row index tensor) over [video | text] rows"""
    L = lay.n_frames * T
    own = own or (0, L)
    mine, text_for = LO.scene_pieces(lay, T, own)
    segs = LO.hunyuan_segments(lay, T, counts, mine, text_for)
    idx = lambda rows: torch.tensor([L + r[1] if isinstance(r, tuple) else r for r in rows], dtype=torch.long)
    return [(kind, idx(qr), idx(kr)) for kind, j, qr, kr in segs]


def scene_layer(segs, q, k, v, sample=1):
    """one layer of the reference CPU path on [video | text] rows q / k / v (fp32 [rows, H, D]). sample > 1 keeps
    every sample-th query row of each segment (a bounded sample of the same work). Returns (out, useful FLOPs)."""
    out = torch.zeros_like(q)
    flops = 0.0
    H, Dh = q.shape[1:]
    for kind, qi, ki in segs:
        qi = qi[::sample]
        qq = q.index_select(0, qi).transpose(0, 1)[None]
        kk = k.index_select(0, ki).transpose(0, 1)[None]
        vv = v.index_select(0, ki).transpose(0, 1)[None]
        o = torch.nn.functional.scaled_dot_product_attention(qq, kk, vv)[0].transpose(0, 1)
        out.index_copy_(0, qi, o)
        flops += 4.0 * len(qi) * len(ki) * H * Dh
    return out, flops


def time_cpu(lay, T, counts, H, Dh, sample, repeats=3, seed=0):
    """median seconds of one sampled layer and its useful FLOPs, on all host threads"""
    torch.set_num_threads(os.cpu_count())
    segs = segment_index(lay, T, counts)
    n = lay.n_frames * T + sum(counts)
    g = torch.Generator().manual_seed(seed)
    q, k, v = (torch.randn(n, H, Dh, generator=g) for _ in range(3))
    scene_layer(segs, q, k, v, sample=max(sample, 64))          # warm-up on a smaller sample
    times = []
    for _ in range(repeats):
        t0 = time.perf_counter()
        _, flops = scene_layer(segs, q, k, v, sample)
        times.append(time.perf_counter() - t0)
    return sorted(times)[len(times) // 2], flops, torch.get_num_threads()
