"""Ulysses sequence parallelism for dense attention windows: head-scatter / sequence-gather.

`_SeqAllToAll` and `DistributedAttentionNodeLevel` keep the interfaces of
`NeutronGT/gt_sp/gt_layer.py:31-51` and `:211-303`.  Forward of `_SeqAllToAll(group, x,
scatter_idx, gather_idx)`: split `x` into P equal chunks along `scatter_idx`, send chunk r to
rank r, and concatenate what arrives along `gather_idx` in rank order; backward is the same
exchange with the two dims swapped.  With q, k, v of shape [1, S/P, H, D] per rank, the
forward exchange gives every rank [1, S, H/P, D] (all positions, its head group); the output
[1, S, H/P * D] goes back to [1, S/P, H * D].

Mechanism: the P chunks are packed into one contiguous buffer and moved with a single
`all_to_all_single` (one NCCL call over NVLink per tensor, instead of P tensors), which
also lets the same code run on gloo for CPU tests.  Chunks must be equal (dims divisible
by P), which the reference's receive buffers assume as well (`gt_layer.py:42-43`).

Node scores: the reference's score exchange (`gt_layer.py:297`) applies a 2-D all-to-all to
the 1-D score vector, which cannot run; here each rank's partial head-mean over its head
group is all-reduced (sum / P gives the mean over all heads) and the rank keeps its own
S/P slice, the shape the reference's exchange was meant to return.

Overlap (`head_chunks` > 1): every rank's head group is cut into chunks; q, k and v of one
chunk travel in one packed `all_to_all_single` issued asynchronously, so NCCL moves chunk c + 1
over NVLink on its own stream while the attention kernels of chunk c run, and each chunk's
output goes back while the next chunk computes.  The backward pipelines the same way in
reverse.  Results equal the unchunked exchange exactly (the chunks are disjoint heads).
"""
from __future__ import annotations

from typing import Any

import torch
import torch.distributed as dist
from torch import Tensor


def _world(group) -> int:
    return dist.get_world_size(group=group)


def seq_all_to_all(x: Tensor, scatter_idx: int, gather_idx: int, group=None) -> Tensor:
    p = _world(group)
    if p == 1:
        return x
    if x.shape[scatter_idx] % p != 0:
        raise ValueError(f"dim {scatter_idx} of size {x.shape[scatter_idx]} does not split into {p} ranks")
    send = torch.stack(torch.tensor_split(x, p, dim=scatter_idx), dim=0).contiguous()
    recv = torch.empty_like(send)
    dist.all_to_all_single(recv, send, group=group)
    return torch.cat(list(recv.unbind(0)), dim=gather_idx).contiguous()


class _SeqAllToAll(torch.autograd.Function):
    @staticmethod
    def forward(ctx: Any, group, input: Tensor, scatter_idx: int, gather_idx: int) -> Tensor:
        ctx.group = group
        ctx.scatter_idx = scatter_idx
        ctx.gather_idx = gather_idx
        return seq_all_to_all(input, scatter_idx, gather_idx, group)

    @staticmethod
    def backward(ctx: Any, *grad_output: Tensor):
        return (None, _SeqAllToAll.apply(ctx.group, *grad_output, ctx.gather_idx, ctx.scatter_idx), None, None)


class _PipelinedAttention(torch.autograd.Function):
    """Head-chunked exchange + local attention with the exchanges overlapping the kernels."""

    @staticmethod
    def forward(ctx: Any, group, local_attn, attn_type, chunks: int, edge_index, query: Tensor, key: Tensor,
                value: Tensor):
        p = _world(group)
        b, s_loc, heads, d = query.shape
        if b != 1 or heads % (p * chunks) != 0:
            raise ValueError(f"{heads} heads do not split into {p} ranks x {chunks} chunks (batch must be 1)")
        hp, hc = heads // p, heads // (p * chunks)
        qkv = torch.stack((query, key, value), dim=2)[0].view(s_loc, 3, p, hp, d)

        def send_in(c):   # [p, s_loc, 3, hc, d]: rank j gets my rows of its head group's chunk c
            return qkv[:, :, :, c * hc:(c + 1) * hc].permute(2, 0, 1, 3, 4).contiguous()

        def exchange(send):
            recv = torch.empty_like(send)
            return recv, dist.all_to_all_single(recv, send, group=group, async_op=True)

        pending = exchange(send_in(0))
        leaves, outputs, back, score = [], [], [], None
        for c in range(chunks):
            recv, work = pending
            if c + 1 < chunks:   # the next chunk's exchange runs while this chunk computes
                pending = exchange(send_in(c + 1))
            work.wait()
            full = recv.view(p * s_loc, 3, hc, d)
            qc, kc, vc = (full[:, i].unsqueeze(0).detach().requires_grad_(query.requires_grad) for i in range(3))
            with torch.enable_grad():
                xc, sc = local_attn(qc, kc, vc, None, edge_index, attn_type)
            leaves.append((qc, kc, vc))
            outputs.append(xc)
            if sc is not None:
                sc = sc.detach() * (hc / hp)
                score = sc if score is None else score + sc
            send = xc.detach().reshape(p, s_loc, hc, d)      # rank j gets its rows
            back.append(exchange(send.contiguous()))
        out = query.new_empty(s_loc, p, hp, d)
        for c, (recv, work) in enumerate(back):
            work.wait()
            out[:, :, c * hc:(c + 1) * hc] = recv.permute(1, 0, 2, 3)
        ctx.group, ctx.chunks, ctx.shape = group, chunks, (s_loc, p, hp, hc, d)
        ctx.leaves, ctx.outputs = leaves, outputs
        if score is not None:
            if p > 1:
                dist.all_reduce(score, op=dist.ReduceOp.SUM, group=group)
                score = score / p
            score = torch.tensor_split(score, p)[dist.get_rank(group=group)].contiguous()
            ctx.mark_non_differentiable(score)
        return out.view(1, s_loc, heads * d), score

    @staticmethod
    def backward(ctx: Any, grad_out: Tensor, _grad_score):
        s_loc, p, hp, hc, d = ctx.shape
        group = ctx.group
        g = grad_out.contiguous().view(s_loc, p, hp, d)

        def send_out(c):  # [p, s_loc, hc, d]: rank j gets my rows' gradient of its chunk c
            return g[:, :, c * hc:(c + 1) * hc].permute(1, 0, 2, 3).contiguous()

        def exchange(send):
            recv = torch.empty_like(send)
            return recv, dist.all_to_all_single(recv, send, group=group, async_op=True)

        pending = exchange(send_out(0))
        back = []
        for c in range(ctx.chunks):
            recv, work = pending
            if c + 1 < ctx.chunks:
                pending = exchange(send_out(c + 1))
            work.wait()
            qc, kc, vc = ctx.leaves[c]
            gx = recv.view(1, p * s_loc, hc * d)
            torch.autograd.backward([ctx.outputs[c]], [gx.to(ctx.outputs[c].dtype)])
            gqkv = torch.stack([t.grad if t.grad is not None else torch.zeros_like(t) for t in (qc, kc, vc)], dim=3)
            back.append(exchange(gqkv[0].reshape(p, s_loc, hc, 3, d).contiguous()))
        dqkv = grad_out.new_empty(s_loc, p, hp, 3, d)
        for c, (recv, work) in enumerate(back):
            work.wait()
            dqkv[:, :, c * hc:(c + 1) * hc] = recv.permute(1, 0, 2, 3, 4)
        ctx.leaves = ctx.outputs = None
        dq, dk, dv = (dqkv[:, :, :, i].reshape(1, s_loc, p * hp, d) for i in range(3))
        return None, None, None, None, None, dq, dk, dv


class DistributedAttentionNodeLevel(torch.nn.Module):
    """`gt_layer.py:211-303`: exchange q/k/v (and a dense attn_bias) to head groups, run the
    local attention on the full sequence, exchange the output back.  In eval mode, as in the
    reference, no exchange happens."""

    def __init__(self, local_attention, sequence_process_group, scatter_idx: int = 2, gather_idx: int = 1,
                 head_chunks: int = 1):
        super().__init__()
        self.local_attn = local_attention
        self.spg = sequence_process_group
        self.scatter_idx = scatter_idx
        self.gather_idx = gather_idx
        self.head_chunks = int(head_chunks)   # > 1: pipelined exchange (module docstring)

    def forward(self, query, key, value, attn_bias, edge_index, attn_type, mask=None, pruning_mask=None, *args):
        if not self.training:
            return self.local_attn(query, key, value, attn_bias, edge_index, attn_type, mask=mask,
                                   pruning_mask=pruning_mask, *args)
        plain = attn_bias is None and mask is None and pruning_mask is None and not args
        if (self.head_chunks > 1 and plain and (self.scatter_idx, self.gather_idx) == (2, 1)
                and query.dim() == 4 and query.shape[2] % (_world(self.spg) * self.head_chunks) == 0):
            return _PipelinedAttention.apply(self.spg, self.local_attn, attn_type, self.head_chunks, edge_index,
                                             query, key, value)
        q = _SeqAllToAll.apply(self.spg, query, self.scatter_idx, self.gather_idx)
        k = _SeqAllToAll.apply(self.spg, key, self.scatter_idx, self.gather_idx)
        v = _SeqAllToAll.apply(self.spg, value, self.scatter_idx, self.gather_idx)
        bias = _SeqAllToAll.apply(self.spg, attn_bias, 1, 2) if attn_bias is not None else None
        context, score = self.local_attn(q, k, v, bias, edge_index, attn_type, mask=mask, pruning_mask=pruning_mask,
                                         *args)
        output = _SeqAllToAll.apply(self.spg, context, self.gather_idx, self.scatter_idx)
        if score is not None:
            p = _world(self.spg)
            score = score.detach().clone()
            if p > 1:
                dist.all_reduce(score, op=dist.ReduceOp.SUM, group=self.spg)
                score = score / p
                rank = dist.get_rank(group=self.spg)
                score = torch.tensor_split(score, p)[rank]
        return output, score
