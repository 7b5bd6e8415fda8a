"""CPU restatement of the reference's packed varlen attention and scene processors.

TEST INFRASTRUCTURE ONLY (see oracle/__init__.py).

The reference computes attention through flash-attn 2.8.3.post1 (`flash_attn_varlen_func`, third-party, not vendored in
the reference: .gitignore:48-51) called from src/onereel/attention.py:39-62. Its published algorithm is exact
non-causal softmax attention per packed segment, out = softmax(q k^T * D^-0.5) v, with the natural-log log-sum-exp
lse = log(sum_k exp(q.k * D^-0.5)) laid out [H, Nq] (attention.py:46-53). This module restates that directly in
float64 numpy (the exact value the bf16 kernel approximates), plus:
  - the scene processor outputs of src/onereel/models/hunyuan15.py:212-251 (`Processor.scene`) and wan.py:110-152,
    built from oracle.layout_oracle's segment order;
  - the log-sum-exp merge of two partial results (hunyuan15.py:274-276, parallel/ring.py:63-70).
"""
from __future__ import annotations

import numpy as np

from oracle import layout_oracle as LO


def attend(q, k, v, scale=None):
    """q [lq, H, D], k / v [lk, H, D] (any float dtype) -> (out [lq, H, D] float64, lse [H, lq] float64)"""
    q, k, v = (np.asarray(x, dtype=np.float64) for x in (q, k, v))
    D = q.shape[-1]
    scale = D ** -0.5 if scale is None else scale
    s = np.einsum('qhd,khd->hqk', q, k) * scale
    m = s.max(-1, keepdims=True)
    p = np.exp(s - m)
    den = p.sum(-1, keepdims=True)
    out = np.einsum('hqk,khd->qhd', p / den, v)
    lse = (m + np.log(den))[..., 0]
    return out, lse


def varlen(q, k, v, cu_q, cu_k, scale=None):
    """flash_attn_varlen_func semantics on packed q [Nq, H, D], k / v [Nk, H, D]: (out [Nq, H, D], lse [H, Nq])"""
    Nq, H, D = q.shape
    out = np.zeros((Nq, H, D))
    lse = np.full((H, Nq), -np.inf)
    for i in range(len(cu_q) - 1):
        a, b, c, d = int(cu_q[i]), int(cu_q[i + 1]), int(cu_k[i]), int(cu_k[i + 1])
        if b > a and d > c:
            out[a:b], lse[:, a:b] = attend(q[a:b], k[c:d], v[c:d], scale)
    return out, lse


def lse_merge(o1, l1, o2, l2):
    """two partial results over disjoint key sets -> the result over their union (hunyuan15.py:274-276)"""
    m = np.maximum(l1, l2)
    m = np.where(np.isinf(m), 0.0, m)
    w1, w2 = np.exp(l1 - m), np.exp(l2 - m)
    den = w1 + w2
    o = (o1 * (w1 / den).T[..., None] + o2 * (w2 / den).T[..., None])
    return o, m + np.log(den)


def _gather(rows, video, text):
    """rows from oracle.layout_oracle (token index or ('t', i)) -> stacked float64 rows"""
    return np.stack([text[r[1]] if isinstance(r, tuple) else video[r] for r in rows]).astype(np.float64)


def hunyuan_scene(lay, T, counts, q, k, v, eq, ek, ev, own=None):
    """hunyuan15.Processor.scene on one rank whose video rows are own = (a, b) of the full token range, with the
    full tensors given (q/k/v [L, H, D], eq/ek/ev [text rows, H, D]). Returns (ov [b - a, H, D], ot [text, H, D],
    text_rows_valid [text] bool): ov for the rank's rows, ot for the sentences whose text queries the rank runs or
    receives (send_text_rows, comm.py:204-223); rows of untouched sentences are not defined and marked invalid."""
    L = lay.n_frames * T
    a, b = own if own is not None else (0, L)
    mine, text_for = LO.scene_pieces(lay, T, (a, b))
    ov = np.zeros((b - a,) + q.shape[1:])
    ot = np.zeros(eq.shape)
    valid = np.zeros(eq.shape[0], dtype=bool)
    tr = LO.text_ranges(counts)
    touched = {j for j, _ in mine}
    segs = LO.hunyuan_segments(lay, T, counts, mine, set(range(lay.n_scenes)) & touched)
    for kind, j, qr, kr in segs:
        o, _ = attend(_gather(qr, q, eq), _gather(kr, k, ek), _gather(kr, v, ev))
        if kind == 'v':
            ov[qr[0] - a:qr[-1] + 1 - a] = o
        else:
            t0, t1 = tr[j]
            ot[t0:t1] = o
            valid[t0:t1] = True
    return ov, ot, valid


def wan_scene(lay, T, q, k, v, own=None):
    """wan.Processor.ranges / scene (wan.py:110-152): video queries of scene j read key_frames(j); no joint text"""
    L = lay.n_frames * T
    a, b = own if own is not None else (0, L)
    mine, _ = LO.scene_pieces(lay, T, (a, b))
    ov = np.zeros((b - a,) + q.shape[1:])
    for j, (lo, hi) in mine:
        kr = LO.token_rows(lay.key_frames(j), T)
        o, _ = attend(q[lo:hi], k[kr], v[kr])
        ov[lo - a:hi - a] = o
    return ov


def masked_dense(lay, T, counts, q, k, v, eq, ek, ev):
    """the BASELINE cfg1 check: one dense softmax over [video | text] with a scene block mask (the mask construction of
    experiments/kernel_breakdown.py:76-90, generalised to halo/extra frames): video token of scene j reads its key
    frames and sentence j; text of sentence j reads scene j's frames and sentence j. Returns (ov, ot) float64."""
    L = lay.n_frames * T
    tr = LO.text_ranges(counts)
    Nt = eq.shape[0]
    allow = np.zeros((L + Nt, L + Nt), dtype=bool)
    for j in range(lay.n_scenes):
        lo, hi = lay.ranges()[j]
        t0, t1 = tr[j]
        kv = np.array(LO.token_rows(lay.key_frames(j), T))
        own_rows = np.arange(lo * T, hi * T)
        txt = L + np.arange(t0, t1)
        allow[np.ix_(own_rows, kv)] = True
        allow[np.ix_(own_rows, txt)] = True
        allow[np.ix_(txt, own_rows)] = True
        allow[np.ix_(txt, txt)] = True
    Q = np.concatenate([q, eq]).astype(np.float64)
    K = np.concatenate([k, ek]).astype(np.float64)
    V = np.concatenate([v, ev]).astype(np.float64)
    D = Q.shape[-1]
    s = np.einsum('qhd,khd->hqk', Q, K) * D ** -0.5
    s = np.where(allow[None], s, -np.inf)
    s = s - s.max(-1, keepdims=True)
    p = np.exp(s)
    p /= p.sum(-1, keepdims=True)
    o = np.einsum('hqk,khd->qhd', p, V)
    return o[:L], o[L:]
