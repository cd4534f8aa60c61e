"""Ulysses exchange and distributed attention on CPU ranks (gloo, world size 2).

A torch restatement of dense attention stands in for the CUDA kernel, so the test checks the
exchange pattern of `gt_sp/gt_layer.py:31-51, 236-303`: the distributed result on each
rank's sequence shard equals single-process attention over the whole sequence, forward and
backward.  The CUDA kernel under the same exchange is covered by tests/test_ulysses_gpu.py.
"""
import math
import os
import socket

import torch
import torch.distributed as dist
import torch.multiprocessing as mp


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    port = s.getsockname()[1]
    s.close()
    return port


class _TorchDense(torch.nn.Module):
    """CoreAttention-shaped stand-in: x [b, s, H*D], node scores [s] (head mean of |S|)."""

    def forward(self, q, k, v, attn_bias, edge_index, attn_type, mask=None, pruning_mask=None):
        b, s, h, d = q.shape
        qt, kt, vt = (t.transpose(1, 2) for t in (q, k, v))
        score = torch.matmul(qt * math.sqrt(d), kt.transpose(2, 3))
        x = torch.matmul(torch.softmax(score, -1), vt).transpose(1, 2).reshape(b, s, h * d)
        return x, score.detach().abs().mean(dim=1).squeeze(0).sum(dim=0)


def _worker(rank, world, port, out, chunks=1):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    from neutrongt_b200.ulysses import DistributedAttentionNodeLevel, _SeqAllToAll
    S, H, D = 12, 4, 3
    g = torch.Generator().manual_seed(0)
    q, k, v, dy = (torch.randn(1, S, H, D, generator=g, dtype=torch.float64) for _ in range(4))
    sl = slice(rank * S // world, (rank + 1) * S // world)
    # the raw exchange: rank r gets all positions of head group r
    x = _SeqAllToAll.apply(None, q[:, sl].contiguous(), 2, 1)
    hs = slice(rank * H // world, (rank + 1) * H // world)
    exch_ok = torch.equal(x, q[:, :, hs])
    layer = DistributedAttentionNodeLevel(_TorchDense(), None, head_chunks=chunks).train()
    ql, kl, vl = (t[:, sl].clone().requires_grad_(True) for t in (q, k, v))
    y, score = layer(ql, kl, vl, None, None, "full")
    y.backward(dy[:, sl].reshape(y.shape))
    out[rank] = (exch_ok, y.detach(), score, ql.grad, kl.grad, vl.grad)
    dist.destroy_process_group()


import pytest


@pytest.mark.parametrize("chunks", [1, 2])
def test_distributed_attention_matches_single_process(chunks):
    """chunks == 2: the pipelined exchange (one head per chunk and rank) gives the same values."""
    port = _free_port()
    with mp.get_context("spawn").Manager() as m:
        res = m.dict()
        mp.spawn(_worker, args=(2, port, res, chunks), nprocs=2, join=True)
        res = dict(res)
    S, H, D = 12, 4, 3
    g = torch.Generator().manual_seed(0)
    q, k, v, dy = (torch.randn(1, S, H, D, generator=g, dtype=torch.float64) for _ in range(4))
    qr, kr, vr = (t.clone().requires_grad_(True) for t in (q, k, v))
    y, score = _TorchDense()(qr, kr, vr, None, None, "full")
    y.backward(dy.reshape(y.shape))
    for r in range(2):
        sl = slice(r * S // 2, (r + 1) * S // 2)
        ok, yr, sr, gq, gk, gv = res[r]
        assert ok
        assert torch.allclose(yr, y[:, sl].detach(), atol=1e-12)
        assert torch.allclose(sr, score[sl], atol=1e-12)
        assert torch.allclose(gq, qr.grad[:, sl], atol=1e-12)
        assert torch.allclose(gk, kr.grad[:, sl], atol=1e-12)
        assert torch.allclose(gv, vr.grad[:, sl], atol=1e-12)
