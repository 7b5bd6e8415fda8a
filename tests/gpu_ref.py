"""fp32 torch reference of packed varlen attention on the GPU (the floating-point kernel's numerics reference), and
shared tolerances. Not a product path: tests only."""
import torch

# the tolerance north_star states against the reference's FlashAttention varlen output on bf16 inputs
MAX_ABS, MEAN_ABS = 2e-2, 2e-3


def ref_attention(q, k, v, q_start, q_len, k_start, k_len, rows=None, chunk=2048):
    """fp32 softmax(q k^T / sqrt(D)) v per segment; rows (optional, per segment a LongTensor of row offsets within
    the segment) restricts the query rows computed. Returns dict seg -> (row offsets, out [n, H, D] fp32,
    lse [H, n] fp32)."""
    res = {}
    Dh = q.shape[-1]
    for i, (qs, ql, ks, kl) in enumerate(zip(q_start, q_len, k_start, k_len)):
        if ql == 0:
            continue
        r = torch.arange(ql, device=q.device) if rows is None else rows[i].to(q.device)
        kk = k[ks:ks + kl].float()
        vv = v[ks:ks + kl].float()
        outs, lses = [], []
        for c in range(0, len(r), chunk):
            qq = q[qs + r[c:c + chunk]].float()
            s = torch.einsum('qhd,khd->hqk', qq, kk) * Dh ** -0.5
            lse = torch.logsumexp(s, -1)
            p = torch.softmax(s, -1)
            outs.append(torch.einsum('hqk,khd->qhd', p, vv))
            lses.append(lse)
        res[i] = (r, torch.cat(outs), torch.cat(lses, 1))
    return res


def compare(out, lse, ref, q_start):
    """max / mean abs error of out (bf16 [Nq, H, D]) and max abs LSE error against ref_attention's result"""
    errs, lerrs, n = [], [], 0
    for i, (r, o, l) in ref.items():
        rows = q_start[i] + r
        d = (out[rows].float() - o).abs()
        errs.append(d.flatten())
        if lse is not None:
            lerrs.append((lse[:, rows] - l).abs().max())
    e = torch.cat(errs)
    return e.max().item(), e.mean().item(), (max(x.item() for x in lerrs) if lerrs else 0.0)
