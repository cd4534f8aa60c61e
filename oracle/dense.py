"""Restatement of the dense full-attention window (test oracle only).

Follows `CoreAttention.full_attention`,
`NeutronGT/models/gt_dist_node_level_single_window.py:56-109` (identical math in
`NeutronGT/models/graphormer_dist_node_level.py:42-65`), for one window (batch 1):

    S     = (q * sqrt(D)) k^T                         (:75-76; the reference multiplies)
    X     = S + attn_bias + pruning_mask              (:78-87, each optional, broadcast)
    X     = masked_fill(X, mask, -1e9)                (:89-99, mask [s, s] bool, all heads)
    P     = softmax(X, dim=-1), dropout(P)            (:101-102)
    out   = P v                                       (:103)
    node_scores[j] = sum_i mean_h |S[h, i, j]|        (:108, raw S: before bias and mask)

`full_attention` is plain torch (any device, any float dtype) and differentiable, so the
backward comes from autograd.  `full_attention_chunked` computes the same forward and the
explicit backward (no bias or mask) in blocks of query rows, for windows whose [H, s, s]
score tensor does not fit (s = 32,768 at the GPH_Large shape):

    dP = dO v^T,  delta_i = <dO_i, out_i>,  dX = P (dP - delta)
    dq = scale dX k,  dk = scale dX^T q,  dv = P^T dO

Both are pinned against the reference's own outputs (tests/golden/dense_attention.pt).
"""
from __future__ import annotations

import math

import torch


def full_attention(k, q, v, attn_bias=None, mask=None, pruning_mask=None, scale=None, keep=None, dropout_p=0.0):
    """q, k, v: [1, s, H, D] (or [s, H, D]); returns (out with q's shape, node_scores [s]).
    `keep` ([H, s, s] bool) applies a dropout keep mask scaled by 1 / (1 - dropout_p)."""
    shape = q.shape
    heads, dim = shape[-2], shape[-1]
    qh, kh, vh = (t.reshape(-1, heads, dim).transpose(0, 1) for t in (q, k, v))     # [H, s, D]
    scale = math.sqrt(dim) if scale is None else scale
    score = torch.matmul(qh * scale, kh.transpose(1, 2))                           # [H, s, s]
    x = score
    for add in (attn_bias, pruning_mask):      # [1, H or 1, s, s] or anything broadcastable to [H, s, s]
        if add is not None:
            x = x + (add[0] if add.dim() == 4 else add)
    if mask is not None:
        x = x.masked_fill(mask.to(x.device).unsqueeze(0), -1e9)
    p = torch.softmax(x, dim=-1)
    if keep is not None:
        p = p * keep.to(p.device, p.dtype) / (1.0 - dropout_p)
    out = torch.matmul(p, vh).transpose(0, 1).reshape(shape)
    ns = score.detach().abs().mean(dim=0).sum(dim=0)
    return out, ns


@torch.no_grad()
def full_attention_chunked(q, k, v, dout, scale=None, rows=4096):
    """q, k, v, dout: [s, H, D] (any float dtype; computed in fp32 unless given fp64).
    Returns (out, node_scores, dq, dk, dv) without building the full [H, s, s] tensors."""
    dt = torch.float64 if q.dtype == torch.float64 else torch.float32
    s, heads, dim = q.shape
    scale = math.sqrt(dim) if scale is None else scale
    qh, kh, vh, gh = (t.to(dt).transpose(0, 1).contiguous() for t in (q, k, v, dout))   # [H, s, D]
    out = torch.empty_like(qh)
    dq = torch.empty_like(qh)
    dk = torch.zeros_like(kh)
    dv = torch.zeros_like(vh)
    ns = torch.zeros(s, dtype=dt, device=q.device)
    for h in range(heads):
        kt, vt = kh[h].t(), vh[h].t()
        for r0 in range(0, s, rows):
            r1 = min(s, r0 + rows)
            sc = torch.matmul(qh[h, r0:r1] * scale, kt)                  # [r, s]
            ns += sc.abs().sum(dim=0) / heads
            p = torch.softmax(sc, dim=-1)
            del sc
            o = torch.matmul(p, vh[h])
            out[h, r0:r1] = o
            g = gh[h, r0:r1]
            delta = (g * o).sum(-1, keepdim=True)
            dp = torch.matmul(g, vt)
            ds = p * (dp - delta)
            del dp
            dq[h, r0:r1] = torch.matmul(ds, kh[h]) * scale
            dk[h] += torch.matmul(ds.t(), qh[h, r0:r1]) * scale
            dv[h] += torch.matmul(p.t(), g)
            del p, ds
    tr = lambda t: t.transpose(0, 1).contiguous()  # noqa: E731
    return tr(out), ns, tr(dq), tr(dk), tr(dv)
