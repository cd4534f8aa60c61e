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


class DistributedAttentionNodeLevel(torch.nn.Module):
    """`gt_layer.py:211-303`: exchange q/k/v (and a dense attn_bias) to head groups, run the
    local attention on the full sequence, exchange the output back.  In eval mode, as in the
    reference, no exchange happens."""

    def __init__(self, local_attention, sequence_process_group, scatter_idx: int = 2, gather_idx: int = 1):
        super().__init__()
        self.local_attn = local_attention
        self.spg = sequence_process_group
        self.scatter_idx = scatter_idx
        self.gather_idx = gather_idx

    def forward(self, query, key, value, attn_bias, edge_index, attn_type, mask=None, pruning_mask=None, *args):
        if not self.training:
            return self.local_attn(query, key, value, attn_bias, edge_index, attn_type, mask=mask,
                                   pruning_mask=pruning_mask, *args)
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
