"""q/k RMSNorm + rotary embedding on the fused CUDA kernel (orl_qk_norm_rope) — the q/k preparation of the
reference processors (src/onereel/models/hunyuan15.py:187-190: per-head RMSNorm then diffusers' apply_rotary_emb;
src/onereel/models/wan.py:64-74 `_qk`: hidden-dimension RMSNorm then Wan's interleaved RoPE, compiled by the reference
into a Triton kernel)."""
from __future__ import annotations

import torch

from onereel_b200 import _lib as L


def qk_norm_rope(x: torch.Tensor, weight: torch.Tensor, cos: torch.Tensor, sin: torch.Tensor, heads: int,
                 eps: float, per_head: bool, sin_shift: int, out: torch.Tensor | None = None,
                 row_map: torch.Tensor | None = None) -> torch.Tensor:
    """x [rows, heads * D] (or [1, rows, heads * D]) bf16 -> [rows, heads, D] bf16, normalised and rotated; cos / sin
    [rows, D] (any float dtype; converted to fp32 contiguous). out / row_map: write row i to out[row_map[i]]."""
    if x.dim() == 3:
        x = x[0]
    if not (x.is_cuda and x.dtype == torch.bfloat16):
        raise TypeError('qk_norm_rope: x must be a bf16 CUDA tensor (no fallback)')
    x = x.contiguous()
    rows, hidden = x.shape
    Dh = hidden // heads
    w = weight.to(device=x.device, dtype=torch.bfloat16).contiguous()
    c = cos.to(device=x.device, dtype=torch.float32).reshape(rows, -1).contiguous()
    s = sin.to(device=x.device, dtype=torch.float32).reshape(rows, -1).contiguous()
    if out is None:
        out = torch.empty(rows, heads, Dh, dtype=torch.bfloat16, device=x.device)
    rm = None if row_map is None else row_map.to(device=x.device, dtype=torch.int32).contiguous()
    L.check(L.lib().orl_qk_norm_rope(x.data_ptr(), out.data_ptr(), w.data_ptr(), c.data_ptr(), s.data_ptr(), rows,
                                     heads, Dh, int(per_head), float(eps), int(sin_shift), c.shape[1],
                                     None if rm is None else rm.data_ptr(),
                                     torch.cuda.current_stream(x.device).cuda_stream), 'orl_qk_norm_rope')
    return out


def rotate_rows(x: torch.Tensor, rows: torch.Tensor, cos: torch.Tensor, sin: torch.Tensor, sin_shift: int = 0):
    """in place: rows `rows` (int32 CUDA tensor) of x [N, H, D] bf16 rotated by the table rows cos / sin
    [len(rows), D] fp32 (orl_rope_rows)"""
    Nr = rows.numel()
    if Nr == 0:
        return x
    H, Dh = x.shape[1:]
    L.check(L.lib().orl_rope_rows(x.data_ptr(), rows.data_ptr(), Nr, H, Dh, cos.data_ptr(), sin.data_ptr(),
                                  cos.shape[1], int(sin_shift), torch.cuda.current_stream(x.device).cuda_stream),
            'orl_rope_rows')
    return x
