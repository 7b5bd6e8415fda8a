"""Varlen attention on the B200 kernel (onereel_b200/csrc/attn_fwd.cu) — the drop-in for src/onereel/attention.py.

Same functions, arguments and return values as the reference module (attention.py:13-84): `cu_seqlens`, `dense`,
`varlen`, `varlen_lse`, `packed`, `packed_lse`, `overlapping_ranges`, and the module global `BACKEND`. The reference
selects FlashAttention-2/-3 by BACKEND; here every value runs the sm_100a kernel ('b200'; the reference's 'fa2', 'fa3'
and 'auto' are accepted so existing callers keep working). There is no CPU or library fallback: inputs must be bf16
CUDA tensors with head_dim 64 or 128.

Kernel failures: the kernel never hangs; a bounded wait that gives up sets a per-device error word. `check()`
synchronises and raises if it is set (tests and benchmarks call it; it costs a device sync).
"""
from __future__ import annotations

from collections import OrderedDict

import numpy as np
import torch

from onereel_b200 import _lib as L
from onereel_b200.pack import pack_rows

BACKEND = 'b200'         # 'b200' (also accepted: the reference's 'fa2' | 'fa3' | 'auto', all served by this kernel)
_BACKENDS = ('b200', 'fa2', 'fa3', 'auto')


def backend() -> str:
    if BACKEND not in _BACKENDS:
        raise ImportError(f'unknown attention backend {BACKEND!r}')
    return 'b200'


def cu_seqlens(lengths, device='cuda') -> torch.Tensor:
    """attention.py:28-29: int32 [0, cumsum(lengths)]"""
    return torch.tensor([0] + np.cumsum(lengths).tolist(), dtype=torch.int32, device=device)


# ------------------------------------------------------------------------------------------------ plans and errors

_PLANS: OrderedDict = OrderedDict()
_ERR: dict = {}


def _err_word(device: torch.device) -> torch.Tensor:
    key = device.index if device.index is not None else torch.cuda.current_device()
    if key not in _ERR:
        _ERR[key] = torch.zeros(1, dtype=torch.int32, device=device)
    return _ERR[key]


def check(device=None) -> None:
    """synchronise and raise if a kernel on `device` (default: every device used) set a bit in its error word (a
    bounded wait that ran out, or cu_seqlens the device planner rejected)"""
    for key, w in list(_ERR.items()):
        if device is not None and torch.device(device).index not in (None, key):
            continue
        bits = int(w.item())
        if bits:
            w.zero_()
            raise L.OrlError(f'kernel on cuda:{key} reported: {L.describe_error_bits(bits)}')


def plan(q_start, q_len, k_start, k_len, heads: int, device) -> tuple[torch.Tensor, int]:
    """device work list for segments given as (start, length) rows (cached: layouts repeat every layer and step)"""
    key = (tuple(q_start), tuple(q_len), tuple(k_start), tuple(k_len), heads, str(device))
    hit = _PLANS.get(key)
    if hit is not None:
        _PLANS.move_to_end(key)
        return hit
    arrs = [np.ascontiguousarray(x, dtype=np.int32) for x in (q_start, q_len, k_start, k_len)]
    n_seg = len(arrs[0])
    need = L.lib().orl_attn_plan_ranges(*(L.i32p(a) for a in arrs), n_seg, heads, None, 0)
    if need >= 0:                                   # nothing to do
        need_n = 0
    else:
        L.check(need if need > -1000 else 0, 'orl_attn_plan_ranges')
        need_n = -need - 1000
    work = np.zeros(max(need_n, 1), dtype=L.WORK_DTYPE)
    n = L.check(L.lib().orl_attn_plan_ranges(*(L.i32p(a) for a in arrs), n_seg, heads, work.ctypes.data, len(work)),
                'orl_attn_plan_ranges')
    dev = torch.from_numpy(work.view(np.uint8)).to(device)
    _PLANS[key] = (dev, n)
    if len(_PLANS) > 512:
        _PLANS.popitem(last=False)
    return dev, n


def _host_list(x) -> list[int]:
    return x.tolist() if isinstance(x, torch.Tensor) else [int(v) for v in x]


def _check_inputs(q, k, v):
    for name, x in (('q', q), ('k', k), ('v', v)):
        if not (isinstance(x, torch.Tensor) and x.is_cuda and x.dtype == torch.bfloat16):
            raise TypeError(f'{name} must be a bf16 CUDA tensor (the B200 path has no fallback), got '
                            f'{getattr(x, "dtype", type(x))} on {getattr(x, "device", "?")}')
        if x.dim() != 3 or x.stride(-1) != 1 or x.stride(1) != x.shape[2] or x.stride(0) != x.shape[1] * x.shape[2]:
            raise ValueError(f'{name} must be a contiguous [rows, heads, head_dim] tensor, got {tuple(x.shape)} '
                             f'strides {x.stride()}')
    if q.shape[1:] != k.shape[1:] or k.shape != v.shape:
        raise ValueError(f'shape mismatch q {tuple(q.shape)} k {tuple(k.shape)} v {tuple(v.shape)}')
    if q.shape[2] not in (64, 128):
        raise ValueError(f'head_dim {q.shape[2]} not supported (64 or 128)')


# Key split of coarse launches (split_keys=True): a launch of fewer than SPLIT_WAVES waves of work items whose longest
# segment has at least SPLIT_MIN_KEYS keys runs as two launches over the two halves of every segment's keys, on two
# streams so the second fills the first's tail, merged by log-sum-exp. Exact attention, but another rounding than
# one pass: callers that promise bit-exact results across partitions (K/V gathering) never ask for it.
SPLIT_WAVES = 4
SPLIT_MIN_KEYS = 2048
LAUNCHES = 0          # attention launches issued by this process (benchmark launch accounting)
SPLITS = 0            # launches that took the key split
_SIDE = {}
_SMS = {}


def _sm_count(dev) -> int:
    key = dev.index if dev.index is not None else torch.cuda.current_device()
    if key not in _SMS:
        _SMS[key] = torch.cuda.get_device_properties(key).multi_processor_count
    return _SMS[key]


def _attend_split(q, k, v, q_start, q_len, k_start, k_len, out, lse, scale):
    """the two key halves (at a 128-key boundary) on the current and a side stream, then orl_lse_merge"""
    global SPLITS
    SPLITS += 1
    dev = q.device
    H, Nq = q.shape[1], q.shape[0]
    half = [128 * ((x + 255) // 256) if x >= 256 else x for x in k_len]
    cur = torch.cuda.current_stream(dev)
    key = dev.index if dev.index is not None else torch.cuda.current_device()
    side = _SIDE.get(key)
    if side is None:
        side = _SIDE[key] = torch.cuda.Stream(dev)
    out = torch.empty_like(q) if out is None else out
    lse_a = torch.empty(H, Nq, dtype=torch.float32, device=dev) if not isinstance(lse, torch.Tensor) else lse
    out_b = torch.empty_like(q)
    lse_b = torch.empty(H, Nq, dtype=torch.float32, device=dev)
    side.wait_stream(cur)
    attend(q, k, v, q_start, q_len, k_start, half, out=out, lse=lse_a, scale=scale)
    with torch.cuda.stream(side):
        attend(q, k, v, q_start, q_len, [a + h for a, h in zip(k_start, half)], [x - h for x, h in zip(k_len, half)],
               out=out_b, lse=lse_b, scale=scale, stream=side.cuda_stream)
    out_b.record_stream(side)
    lse_b.record_stream(side)
    cur.wait_stream(side)
    lse_merge(out, lse_a, out_b, lse_b)
    return out, (lse_a if lse is not None else None)


def attend(q, k, v, q_start, q_len, k_start, k_len, out=None, lse=None, scale=None, stream=None, split_keys=False):
    """the kernel call: segment i = q rows q_start[i] + [0, q_len[i]) attending to k / v rows k_start[i] + [0, k_len[i]).
    out [Nq, H, D] bf16 (allocated if None); lse None, True (allocate [H, Nq] fp32) or a tensor. split_keys: allow the
    key split of coarse launches (see SPLIT_WAVES)."""
    _check_inputs(q, k, v)
    Nq, H, Dh = q.shape
    dev = q.device
    work, n = plan(q_start, q_len, k_start, k_len, H, dev)
    if (split_keys and stream is None and n and n < SPLIT_WAVES * _sm_count(dev) and
            max(k_len) >= SPLIT_MIN_KEYS):
        if lse is True:
            lse = torch.empty(H, Nq, dtype=torch.float32, device=dev)
        return _attend_split(q, k, v, q_start, q_len, k_start, k_len, out, lse, scale)
    if out is None:
        out = torch.empty_like(q)
    if lse is True:
        lse = torch.empty(H, Nq, dtype=torch.float32, device=dev)
    scale = Dh ** -0.5 if scale is None else float(scale)
    s = stream if stream is not None else torch.cuda.current_stream(dev).cuda_stream
    global LAUNCHES
    LAUNCHES += 1
    L.check(L.lib().orl_attn_fwd(q.data_ptr(), k.data_ptr(), v.data_ptr(), out.data_ptr(),
                                 None if lse is None else lse.data_ptr(), Nq, k.shape[0], H, Dh, scale,
                                 work.data_ptr(), n, _err_word(dev).data_ptr(), s), 'orl_attn_fwd')
    return out, lse


def attend_work(q, k, v, work, n_items: int, out, lse=None, scale=None, stream=None):
    """the kernel call with a caller-held device work list (orl_attn_plan_ranges items, possibly edited on the
    device since: the bounded memory sets each item's key count per head from its selection)"""
    _check_inputs(q, k, v)
    Nq, H, Dh = q.shape
    dev = q.device
    scale = Dh ** -0.5 if scale is None else float(scale)
    s = stream if stream is not None else torch.cuda.current_stream(dev).cuda_stream
    L.check(L.lib().orl_attn_fwd(q.data_ptr(), k.data_ptr(), v.data_ptr(), out.data_ptr(),
                                 None if lse is None else lse.data_ptr(), Nq, k.shape[0], H, Dh, scale,
                                 work.data_ptr(), n_items, _err_word(dev).data_ptr(), s), 'orl_attn_fwd')
    return out


def _cu_to_ranges(cu_q, cu_k):
    cq, ck = _host_list(cu_q), _host_list(cu_k)
    if len(cq) != len(ck):
        raise ValueError('cu_seqlens_q and cu_seqlens_k differ in length')
    qs, ks = cq[:-1], ck[:-1]
    ql = [b - a for a, b in zip(cq[:-1], cq[1:])]
    kl = [b - a for a, b in zip(ck[:-1], ck[1:])]
    if any(x < 0 for x in ql + kl):
        raise ValueError('cu_seqlens must be non-decreasing')
    return qs, ql, ks, kl


_CU_WORK = {}    # (device, stream) -> work-list scratch of orl_attn_fwd_cu (uint8), grown as needed


def _attend_cu(q, k, v, cu_q, cu_k, lse):
    """cu_seqlens on the device: orl_attn_fwd_cu plans the work list on the GPU, no host synchronisation. The
    scratch is per (device, stream), so calls on one stream reuse it in order."""
    _check_inputs(q, k, v)
    for name, c in (('cu_seqlens_q', cu_q), ('cu_seqlens_k', cu_k)):
        if c.dtype != torch.int32 or c.dim() != 1 or c.device != q.device or not c.is_contiguous():
            raise TypeError(f'{name} must be a contiguous int32 tensor on {q.device}')
    if cu_q.numel() != cu_k.numel() or cu_q.numel() < 1:
        raise ValueError('cu_seqlens_q and cu_seqlens_k differ in length')
    Nq, H, Dh = q.shape
    dev = q.device
    n_seg = cu_q.numel() - 1
    need = L.check(L.lib().orl_attn_fwd_cu_capacity(Nq, n_seg, H), 'orl_attn_fwd_cu_capacity')
    stream = torch.cuda.current_stream(dev)
    key = (dev.index, stream.cuda_stream)
    work = _CU_WORK.get(key)
    if work is None or work.numel() < need * L.WORK_DTYPE.itemsize:
        work = _CU_WORK[key] = torch.empty(need * L.WORK_DTYPE.itemsize, dtype=torch.uint8, device=dev)
    out = torch.empty_like(q)
    lse_t = torch.empty(H, Nq, dtype=torch.float32, device=dev) if lse else None
    L.check(L.lib().orl_attn_fwd_cu(q.data_ptr(), k.data_ptr(), v.data_ptr(), out.data_ptr(),
                                    None if lse_t is None else lse_t.data_ptr(), Nq, k.shape[0], H, Dh, Dh ** -0.5,
                                    cu_q.data_ptr(), cu_k.data_ptr(), n_seg, work.data_ptr(),
                                    work.numel() // L.WORK_DTYPE.itemsize, _err_word(dev).data_ptr(),
                                    stream.cuda_stream), 'orl_attn_fwd_cu')
    return out, lse_t


def varlen(q, k, v, cu_q, cu_k, max_q, max_k):
    """attention.py:39-43: packed q [Nq, H, D], k / v [Nk, H, D] -> out [Nq, H, D]. cu_seqlens as device int32
    tensors (as the reference passes them) are planned on the GPU without a host sync; host lists are planned on
    the host."""
    if isinstance(cu_q, torch.Tensor) and cu_q.is_cuda:
        return _attend_cu(q, k, v, cu_q, cu_k, lse=False)[0]
    return attend(q, k, v, *_cu_to_ranges(cu_q, cu_k))[0]


def varlen_lse(q, k, v, cu_q, cu_k, max_q, max_k):
    """attention.py:46-53: (out [Nq, H, D], lse [H, Nq] fp32, natural log)"""
    if isinstance(cu_q, torch.Tensor) and cu_q.is_cuda:
        return _attend_cu(q, k, v, cu_q, cu_k, lse=True)
    return attend(q, k, v, *_cu_to_ranges(cu_q, cu_k), lse=True)


def _pack_segments(segments):
    lq = [s[0].shape[0] for s in segments]
    lk = [s[1].shape[0] for s in segments]
    q0 = segments[0][0]
    H, Dh = q0.shape[1:]
    qp = q0.new_empty(sum(lq), H, Dh)
    kp = q0.new_empty(sum(lk), H, Dh)
    vp = q0.new_empty(sum(lk), H, Dh)
    c = lambda x: x if x.is_contiguous() else x.contiguous()
    pack_rows([c(s[0]) for s in segments], qp)
    pack_rows([c(s[1]) for s in segments], kp)
    pack_rows([c(s[2]) for s in segments], vp)
    cq, ck = np.cumsum([0] + lq), np.cumsum([0] + lk)
    return qp, kp, vp, lq, list(cq[:-1]), lk, list(ck[:-1])


def packed_lse(segments):
    """attention.py:56-62: list of (out, lse [H, n]) per segment, one kernel call"""
    qp, kp, vp, lq, qs, lk, ks = _pack_segments(segments)
    o, lse = attend(qp, kp, vp, qs, lq, ks, lk, lse=True)
    return list(zip(o.split(lq), lse.split(lq, dim=1)))


def packed(segments):
    """attention.py:65-71: segments = list of (q, k, v) -> list of outputs, one gather/pack launch per tensor and one
    attention launch"""
    qp, kp, vp, lq, qs, lk, ks = _pack_segments(segments)
    return attend(qp, kp, vp, qs, lq, ks, lk)[0].split(lq)


def overlapping_ranges(q, k, v, q_ranges, k_ranges):
    """attention.py:74-84: q rows q_ranges[j] attend to k / v rows k_ranges[j], read in place (no copy); q_ranges
    tile q in order"""
    qs = [a for a, _ in q_ranges]
    ql = [b - a for a, b in q_ranges]
    if qs and (qs[0] != 0 or any(qs[i] + ql[i] != qs[i + 1] for i in range(len(qs) - 1)) or qs[-1] + ql[-1] != q.shape[0]):
        raise ValueError('q_ranges must tile q in order')
    return attend(q, k, v, qs, ql, [a for a, _ in k_ranges], [b - a for a, b in k_ranges])[0]


def dense(q, k, v):
    """attention.py:32-36: q, k, v [B, S, H, D] -> [B, S, H, D], full attention per batch entry"""
    B, S, H, Dh = q.shape
    Sk = k.shape[1]
    c = lambda x: x.reshape(B * x.shape[1], H, Dh).contiguous()
    o = attend(c(q), c(k), c(v), [b * S for b in range(B)], [S] * B, [b * Sk for b in range(B)], [Sk] * B)[0]
    return o.view(B, S, H, Dh)


def lse_merge(o1, lse1, o2, lse2):
    """in place: (o1, lse1) <- the merge of two partial results over disjoint keys (hunyuan15.py:274-276,
    ring.py:63-70). o [n, H, D] bf16 contiguous, lse [H, >= n] fp32 (row stride = its second dimension)."""
    n, H, Dh = o1.shape
    s = torch.cuda.current_stream(o1.device).cuda_stream
    L.check(L.lib().orl_lse_merge(o1.data_ptr(), lse1.data_ptr(), o2.data_ptr(), lse2.data_ptr(), n, lse1.stride(0),
                                  lse2.stride(0), H, Dh, s), 'orl_lse_merge')
    return o1, lse1


def lse_merge_acc(acc, lse_acc, part, lse_part):
    """in place: fp32 (acc, lse_acc) <- merged with a bf16 partial result (part, lse_part) over disjoint keys
    (ring.py:63-70). acc [n, H, D] fp32 / part [n, H, D] bf16 contiguous rows, lse [H, >= n] fp32."""
    n, H, Dh = acc.shape
    s = torch.cuda.current_stream(acc.device).cuda_stream
    L.check(L.lib().orl_lse_merge_acc(acc.data_ptr(), lse_acc.data_ptr(), part.data_ptr(), lse_part.data_ptr(), n,
                                      lse_acc.stride(0), lse_part.stride(0), H, Dh, s), 'orl_lse_merge_acc')
    return acc, lse_acc
