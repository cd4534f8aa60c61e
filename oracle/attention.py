"""CPU restatement of the graph-sparse window attention (test oracle only).

Follows `CoreAttention.sparse_attention_bias`,
`NeutronGT/models/gt_dist_node_level_single_window.py:112-179` (identical math in
`NeutronGT/models/graphormer_dist_node_level.py:67-98`).  Per edge e = (src -> dst)
and head h, with D the head size:

    s_e   = clamp(sum_i k[src,h,i] * q[dst,h,i] / sqrt(D), -5, 5)      (:130-139)
    s_e  += attn_bias[0, h, src, dst]          (only when a bias is given, :142-152)
    p_e   = exp(s_e)                                                     (:156)
    Z_d   = sum_{e into d} p_e                                           (:172-173)
    x_d   = (sum_{e into d} p_e v[src]) / (Z_d + 1e-6)                   (:161-175)
    node_scores[d] = sum_{e into d} mean_h p_e, length max(dst)+1        (:177-178)

The backward is the chain rule of that forward written out explicitly (the
reference gets it from torch autograd):

    a_e  = p_e / (Z_d + 1e-6)
    dv  += a_e dO_d
    dp_e = (<dO_d, v_src> - <dO_d, x_d>) / (Z_d + 1e-6)
    ds_e = dp_e p_e 1[-5 <= s_raw <= 5]          (clamp passes grads on the closed range)
    dq_d += ds_e k_src / sqrt(D);  dk_src += ds_e q_d / sqrt(D)
    dbias[0, h, src, dst] += dp_e p_e

Everything is torch on the CPU; sums over edges use `index_add_`, which on the
CPU adds in edge order, the same order the reference's CPU scatter uses.
"""
from __future__ import annotations

import math

import torch

EPS = 1e-6
CLAMP = 5.0


def _as_shd(t: torch.Tensor, heads: int) -> torch.Tensor:
    return t.reshape(-1, heads, t.shape[-1])


def _edge_bias(attn_bias, src, dst):
    # attn_bias: [1, H, s, s]; the reference permutes to [s, s, H] and gathers [src, dst, :]
    return attn_bias[0][:, src, dst].transpose(0, 1)


def sparse_attention_forward(q, k, v, edge_index, attn_bias=None):
    """Returns (x [s, H, D], node_scores [max(dst)+1], Z [s, H], raw scores [E, H])."""
    heads, dim = q.shape[-2], q.shape[-1]
    q = _as_shd(q, heads)
    k = _as_shd(k, heads)
    v = _as_shd(v, heads)
    src = edge_index[0].to(torch.long)
    dst = edge_index[1].to(torch.long)
    scale = math.sqrt(dim)
    raw = (k[src] * q[dst] / scale).sum(-1)                       # [E, H]
    score = raw.clamp(-CLAMP, CLAMP)
    if attn_bias is not None:
        score = score + _edge_bias(attn_bias, src, dst)
    p = torch.exp(score)
    wv = torch.zeros_like(v).index_add_(0, dst, v[src] * p.unsqueeze(-1))
    z = p.new_zeros(v.shape[0], heads).index_add_(0, dst, p)
    x = wv / (z.unsqueeze(-1) + EPS)
    ns_len = int(dst.max()) + 1 if dst.numel() else 0
    node_scores = p.new_zeros(ns_len).index_add_(0, dst, p.mean(dim=1))
    return x, node_scores, z, raw


def sparse_attention_backward(q, k, v, edge_index, dout, attn_bias=None):
    """Returns (dq, dk, dv, dattn_bias) with dq/dk/dv shaped [s, H, D]."""
    heads, dim = q.shape[-2], q.shape[-1]
    q = _as_shd(q, heads)
    k = _as_shd(k, heads)
    v = _as_shd(v, heads)
    dout = _as_shd(dout, heads)
    src = edge_index[0].to(torch.long)
    dst = edge_index[1].to(torch.long)
    scale = math.sqrt(dim)
    x, _, z, raw = sparse_attention_forward(q, k, v, edge_index, attn_bias)
    score = raw.clamp(-CLAMP, CLAMP)
    if attn_bias is not None:
        score = score + _edge_bias(attn_bias, src, dst)
    p = torch.exp(score)
    inv = 1.0 / (z + EPS)                                          # [s, H]
    delta = (dout * x).sum(-1)                                     # [s, H]
    a = p * inv[dst]
    dv = torch.zeros_like(v).index_add_(0, src, a.unsqueeze(-1) * dout[dst])
    dp = ((dout[dst] * v[src]).sum(-1) - delta[dst]) * inv[dst]
    dpre = dp * p                                                  # grad wrt clamped score (+bias)
    mask = (raw >= -CLAMP) & (raw <= CLAMP)
    ds = dpre * mask.to(dpre.dtype)
    dq = torch.zeros_like(q).index_add_(0, dst, ds.unsqueeze(-1) * k[src] / scale)
    dk = torch.zeros_like(k).index_add_(0, src, ds.unsqueeze(-1) * q[dst] / scale)
    dbias = None
    if attn_bias is not None:
        dbias = torch.zeros_like(attn_bias)
        flat = dbias[0].reshape(heads, -1)
        n = attn_bias.shape[-1]
        flat.index_add_(1, src * n + dst, dpre.transpose(0, 1))
    return dq, dk, dv, dbias
