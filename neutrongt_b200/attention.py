"""Graph-sparse window attention behind the reference's `CoreAttention` interface.

`sparse_attention_bias(q, k, v, edge_index, attn_bias)` has the contract of
`CoreAttention.sparse_attention_bias` (`NeutronGT/models/gt_dist_node_level_single_window.py:112-179`,
identical in `NeutronGT/models/graphormer_dist_node_level.py:67-98`):

* q, k, v: [b, s, H, D] (b == 1, as in NeutronGT) or [s, H, D]; float32 or bfloat16
* edge_index: [2, E] integer tensor, row 0 = source (K/V row), row 1 = destination
* attn_bias: None or [1, H, s, s]; the bias of edge (src, dst) in head h is
  attn_bias[0, h, src, dst]
* returns x [s, H, D] (same dtype as q) and node_scores [max(dst) + 1] float32,
  node_scores[d] = sum over in-edges of d of the head-mean of exp(score)

Forward and backward are the CUDA kernels of `csrc/spattn.cu`; q, k, v and attn_bias
receive gradients, node_scores is returned without one (the models detach it,
`…single_window.py:627`).
"""
from __future__ import annotations

import math

import torch
import torch.nn as nn

from . import _lib
from .edge_csr import EdgeCSR, edge_csr_for


class _SparseWindowAttention(torch.autograd.Function):
    @staticmethod
    def forward(ctx, q, k, v, edge_bias, csr: EdgeCSR):
        s, heads, dim = q.shape
        out = torch.empty_like(q)
        z = torch.empty(s, heads, dtype=torch.float32, device=q.device)
        ns = torch.empty(csr.node_scores_len, dtype=torch.float32, device=q.device)
        L = _lib.lib()
        first, rows, nseg = csr.seg_tables(0)
        part = _seg_part(0, heads, dim, nseg, 0, q.device)
        _lib.check(L.ngt_spattn_forward_seg(_lib.dtype_code(q.dtype), s, csr.e, heads, dim, _lib.ptr(q),
                                            _lib.ptr(k), _lib.ptr(v), _lib.ptr(csr.dst_rowptr),
                                            _lib.ptr(csr.dst_src), _lib.ptr(edge_bias), _lib.ptr(out),
                                            _lib.ptr(z), _lib.ptr(ns), ns.numel(), csr.seg_edges, _lib.ptr(first),
                                            _lib.ptr(rows), nseg, _lib.ptr(part), _lib.stream_of(q)),
                   "ngt_spattn_forward_seg")
        ctx.save_for_backward(q, k, v, out, z, edge_bias)
        ctx.csr = csr
        ctx.mark_non_differentiable(ns)
        return out, ns

    @staticmethod
    def backward(ctx, dout, _dns):
        q, k, v, out, z, edge_bias = ctx.saved_tensors
        csr: EdgeCSR = ctx.csr
        if dout is None:
            return None, None, None, None, None
        dout = dout.to(q.dtype).contiguous()
        s, heads, dim = q.shape
        delta = torch.empty(s, heads, dtype=torch.float32, device=q.device)
        dq = torch.empty_like(q)
        dk = torch.empty_like(k)
        dv = torch.empty_like(v)
        dbias = None
        if edge_bias is not None and ctx.needs_input_grad[3]:
            dbias = torch.empty_like(edge_bias)
        L = _lib.lib()
        fd, rd, nd = csr.seg_tables(0)
        fs, rs, ns_ = csr.seg_tables(1)
        part = _seg_part(1, heads, dim, nd, ns_, q.device)
        _lib.check(L.ngt_spattn_backward_seg(_lib.dtype_code(q.dtype), s, csr.e, heads, dim, _lib.ptr(q),
                                             _lib.ptr(k), _lib.ptr(v), _lib.ptr(out), _lib.ptr(dout),
                                             _lib.ptr(z), _lib.ptr(csr.dst_rowptr), _lib.ptr(csr.dst_src),
                                             _lib.ptr(csr.src_rowptr), _lib.ptr(csr.src_dst),
                                             _lib.ptr(csr.src_to_dst_slot), _lib.ptr(edge_bias),
                                             _lib.ptr(delta), _lib.ptr(dq), _lib.ptr(dk), _lib.ptr(dv),
                                             _lib.ptr(dbias), csr.seg_edges, _lib.ptr(fd), _lib.ptr(rd), nd,
                                             _lib.ptr(fs), _lib.ptr(rs), ns_, _lib.ptr(part), _lib.stream_of(q)),
                   "ngt_spattn_backward_seg")
        return dq, dk, dv, dbias, None


def _seg_part(pass_: int, heads: int, dim: int, nseg_dst: int, nseg_src: int, device):
    """fp32 scratch for the heavy-row segment partial sums (None when there are no segments)."""
    if nseg_dst == 0 and nseg_src == 0:
        return None
    nbytes = _lib.size_query(_lib.lib().ngt_spattn_seg_part_size, pass_, heads, dim, nseg_dst, nseg_src)
    return _lib.workspace(nbytes, device)


class WindowAttentionBuffers:
    """Preallocated outputs for repeated forward/backward launches on one window.

    Launches the same kernels as `sparse_attention_bias` without autograd bookkeeping
    or allocation, so the launches can be timed one by one or captured in a CUDA graph.
    """

    def __init__(self, q, k, v, csr: EdgeCSR):
        self.q, self.k, self.v, self.csr = q, k, v, csr
        s, heads, dim = q.shape
        self.shape = (s, heads, dim)
        dev = q.device
        self.out = torch.empty_like(q)
        self.z = torch.empty(s, heads, dtype=torch.float32, device=dev)
        self.ns = torch.empty(max(csr.node_scores_len, 0), dtype=torch.float32, device=dev)
        self.delta = torch.empty(s, heads, dtype=torch.float32, device=dev)
        self.dq = torch.empty_like(q)
        self.dk = torch.empty_like(k)
        self.dv = torch.empty_like(v)
        self.code = _lib.dtype_code(q.dtype)
        self.segs = (csr.seg_tables(0), csr.seg_tables(1))
        nd, ns_ = self.segs[0][2], self.segs[1][2]
        self.part_f = _seg_part(0, heads, dim, nd, 0, dev)
        self.part_b = _seg_part(1, heads, dim, nd, ns_, dev)

    def forward(self):
        s, heads, dim = self.shape
        c = self.csr
        (fd, rd, nd), _ = self.segs
        _lib.check(_lib.lib().ngt_spattn_forward_seg(self.code, s, c.e, heads, dim, _lib.ptr(self.q),
                                                     _lib.ptr(self.k), _lib.ptr(self.v), _lib.ptr(c.dst_rowptr),
                                                     _lib.ptr(c.dst_src), None, _lib.ptr(self.out),
                                                     _lib.ptr(self.z), _lib.ptr(self.ns), self.ns.numel(),
                                                     c.seg_edges, _lib.ptr(fd), _lib.ptr(rd), nd,
                                                     _lib.ptr(self.part_f), _lib.stream_of(self.q)),
                   "ngt_spattn_forward_seg")
        return self.out, self.ns

    def backward(self, dout):
        s, heads, dim = self.shape
        c = self.csr
        (fd, rd, nd), (fs, rs, ns_) = self.segs
        _lib.check(_lib.lib().ngt_spattn_backward_seg(self.code, s, c.e, heads, dim, _lib.ptr(self.q),
                                                      _lib.ptr(self.k), _lib.ptr(self.v), _lib.ptr(self.out),
                                                      _lib.ptr(dout), _lib.ptr(self.z), _lib.ptr(c.dst_rowptr),
                                                      _lib.ptr(c.dst_src), _lib.ptr(c.src_rowptr),
                                                      _lib.ptr(c.src_dst), None, None, _lib.ptr(self.delta),
                                                      _lib.ptr(self.dq), _lib.ptr(self.dk), _lib.ptr(self.dv), None,
                                                      c.seg_edges, _lib.ptr(fd), _lib.ptr(rd), nd, _lib.ptr(fs),
                                                      _lib.ptr(rs), ns_, _lib.ptr(self.part_b),
                                                      _lib.stream_of(self.q)), "ngt_spattn_backward_seg")
        return self.dq, self.dk, self.dv


def sparse_attention_bias(q, k, v, edge_index, attn_bias=None, num_heads=None):
    """Drop-in for `CoreAttention.sparse_attention_bias` (see module docstring)."""
    heads = num_heads if num_heads is not None else q.shape[-2]
    dim = q.shape[-1]
    _lib.require_cuda(q, k, v, edge_index, attn_bias)
    q3 = q.reshape(-1, heads, dim)
    k3 = k.reshape(-1, heads, dim)
    v3 = v.reshape(-1, heads, dim)
    if not (q3.dtype == k3.dtype == v3.dtype):
        raise TypeError(f"q, k, v dtypes differ: {q3.dtype}, {k3.dtype}, {v3.dtype}")
    _lib.dtype_code(q3.dtype)
    s = q3.shape[0]
    if k3.shape[0] != s or v3.shape[0] != s:
        raise ValueError("q, k and v must have the same number of rows")
    csr = edge_csr_for(edge_index, s)
    edge_bias = None
    if attn_bias is not None:
        if attn_bias.dim() != 4 or attn_bias.shape[0] != 1:
            raise ValueError("attn_bias must be [1, H, s, s] (windows are one sequence)")
        src, dst = csr.dst_major_pairs()
        edge_bias = attn_bias[0][:, src, dst].transpose(0, 1).to(torch.float32).contiguous()
    x, ns = _SparseWindowAttention.apply(q3.contiguous(), k3.contiguous(), v3.contiguous(), edge_bias, csr)
    return x, ns


class CoreAttention(nn.Module):
    """Mirror of the reference `CoreAttention` (`…single_window.py:30-227`).

    Same constructor and `forward(q, k, v, attn_bias, edge_index, attn_type, mask,
    pruning_mask) -> (x [b, s, H*D], score)`.  `attn_type == "sparse"` runs the CUDA
    sparse window attention; the dense paths (`"full"`, `"flash"`) run
    `dense_attention.full_attention`.
    """

    def __init__(self, hidden_size, attention_dropout_rate, num_heads):
        super().__init__()
        self.hidden_size_per_attention_head = hidden_size // num_heads
        self.num_attention_heads_per_partition = num_heads
        self.hidden_size_per_partition = hidden_size
        self.scale = math.sqrt(self.hidden_size_per_attention_head)
        self.num_heads = num_heads
        self.att_dropout = nn.Dropout(attention_dropout_rate)
        self.attention_dropout_rate = attention_dropout_rate

    def sparse_attention_bias(self, q, k, v, edge_index, attn_bias):
        # heads come from the [b, s, H, D] tensor itself, so a head-group shard (after the
        # Ulysses exchange) works too; without sequence parallelism H == num_heads
        return sparse_attention_bias(q, k, v, edge_index, attn_bias,
                                     num_heads=q.shape[-2] if q.dim() == 4 else self.num_heads)

    def full_attention(self, k, q, v, attn_bias, mask=None, pruning_mask=None):
        from .dense_attention import full_attention
        p = self.attention_dropout_rate if self.training else 0.0
        return full_attention(k, q, v, attn_bias, mask=mask, pruning_mask=pruning_mask,
                              scale=self.scale, dropout_p=p)

    def forward(self, q, k, v, attn_bias=None, edge_index=None, attn_type=None, mask=None,
                pruning_mask=None):
        batch_size, s_len = q.size(0), q.size(1)
        score = None
        if attn_type == "sparse":
            x, score = self.sparse_attention_bias(q, k, v, edge_index, attn_bias)
        else:
            x, score = self.full_attention(k, q, v, attn_bias, mask=mask, pruning_mask=pruning_mask)
        x = x.reshape(batch_size, s_len, -1)
        return x, score
