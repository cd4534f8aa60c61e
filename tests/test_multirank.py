"""Multi-rank host logic of the window-parallel loop on CPU (gloo, world size 2).

Ranks own disjoint windows (round-robin, `window_state.py:210`), take the same number of
steps (zero-gradient steps on the rank with fewer windows, `train_eval.py:211-217`), and
average gradients every step (`:289-295`); after each epoch the replicas stay identical.
"""
import os
import socket
from types import SimpleNamespace

import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    port = s.getsockname()[1]
    s.close()
    return port


class _ToyModel(torch.nn.Module):
    """Same call signature and return tuple as the window models; ignores the edges."""

    def __init__(self, d, c):
        super().__init__()
        self.lin = torch.nn.Linear(d, c)

    def forward(self, x, attn_bias, edge_index, *a, attn_type=None, **k):
        out = torch.log_softmax(self.lin(x), dim=1)
        return out, None, [out.detach().sum(1)], None


def _worker(rank, world, port, results):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    from neutrongt_b200.train import FlatGradients, WindowState, train_epoch
    torch.manual_seed(0)                      # identical replicas
    n, d, c = 60, 6, 3
    g = torch.Generator().manual_seed(1)
    feature = torch.randn(n, d, generator=g)
    y = torch.randint(0, c, (n,), generator=g)
    split = {"train": torch.arange(0, n, 2)}
    parts = [torch.arange(i * 12, (i + 1) * 12) for i in range(5)]    # 5 windows: 3 on rank 0, 2 on rank 1
    ids = list(range(rank, 5, world))
    ws = WindowState(ids, [parts[i] for i in ids], [torch.empty(2, 0, dtype=torch.long)] * len(ids),
                     [torch.empty(0, dtype=torch.long)] * len(ids), feature.new_empty(0, d))
    model = _ToyModel(d, c)
    grads = FlatGradients(model)
    opt = torch.optim.SGD(model.parameters(), lr=0.1)
    sched = torch.optim.lr_scheduler.StepLR(opt, 10)
    args = SimpleNamespace(use_cache=1, attn_type="sparse")
    loss, scores, _, stats = train_epoch(args, model, ws.local_partition_ids, ws.local_partitions, feature, y, opt,
                                         sched, world, split, torch.device("cpu"), 0, ws, grads=grads)
    results[rank] = (torch.cat([p.detach().flatten() for p in model.parameters()]), stats["max_window_steps"],
                     sorted(scores))
    dist.destroy_process_group()


def test_two_ranks_stay_in_lockstep_and_identical():
    port = _free_port()
    with mp.get_context("spawn").Manager() as m:
        results = m.dict()
        mp.spawn(_worker, args=(2, port, results), nprocs=2, join=True)
        r0, r1 = results[0], results[1]
    assert torch.equal(r0[0], r1[0])          # replicas identical after averaged steps
    assert r0[1] == r1[1] == 3                # rank 1 took one zero-gradient step
    assert r0[2] == [0, 2, 4] and r1[2] == [1, 3]


def test_flat_gradients_are_views():
    from neutrongt_b200.train import FlatGradients
    model = torch.nn.Sequential(torch.nn.Linear(3, 4), torch.nn.Linear(4, 2))
    fg = FlatGradients(model)
    model(torch.randn(5, 3)).sum().backward()
    assert fg.flat.abs().sum() > 0
    assert all(p.grad.data_ptr() >= fg.flat.data_ptr() for p in model.parameters())
    fg.zero()
    assert all(float(p.grad.abs().sum()) == 0 for p in model.parameters())


def _partitions():
    g = torch.Generator().manual_seed(3)
    return [torch.randperm(100, generator=g)[: 5 + 3 * i] for i in range(7)] + [torch.empty(0, dtype=torch.long)]


def _bcast_worker(rank, world, port, results):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    from neutrongt_b200.train import broadcast_partitions
    got = broadcast_partitions(_partitions() if rank == 0 else None)
    results[rank] = ([p.clone() for p in got], list(range(rank, len(got), world)))
    results[f"empty{rank}"] = len(broadcast_partitions([] if rank == 0 else None))
    dist.destroy_process_group()


def test_window_node_lists_broadcast_from_rank_zero():
    """The collective replacement of the reference's per-rank bundle files: every rank receives
    rank 0's window node lists (order, lengths and ids, an empty window included) and owns
    windows pid mod world_size of them."""
    port = _free_port()
    with mp.get_context("spawn").Manager() as m:
        results = m.dict()
        mp.spawn(_bcast_worker, args=(2, port, results), nprocs=2, join=True)
        out = {k: results[k] for k in results.keys()}
    expected = _partitions()
    for r in range(2):
        got, owned = out[r]
        assert len(got) == len(expected)
        assert all(torch.equal(a, b) and a.dtype == torch.long for a, b in zip(got, expected))
        assert owned == list(range(r, 8, 2))
        assert out[f"empty{r}"] == 0


def _bucket_worker(rank, world, port, results):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    from neutrongt_b200.train import FlatGradients
    torch.manual_seed(0)
    model = torch.nn.Sequential(torch.nn.Linear(16, 32), torch.nn.ReLU(), torch.nn.Linear(32, 32), torch.nn.ReLU(),
                                torch.nn.Linear(32, 4))
    unused = torch.nn.Linear(4, 4)          # a parameter without a gradient: its bucket goes in average()
    model.add_module("unused", unused)
    out = {}
    for mode in ("plain", "buckets"):
        grads = FlatGradients(model, bucket_bytes=600 if mode == "buckets" else None)
        if mode == "buckets":
            assert len(grads.buckets) >= 3
        per_step = []
        for step in range(3):
            grads.zero()
            g = torch.Generator().manual_seed(100 * step + rank)
            x = torch.randn(8, 16, generator=g)
            model(x).square().sum().backward()
            grads.average(world)
            per_step.append(grads.flat.clone())
        out[mode] = per_step
    results[rank] = out
    dist.destroy_process_group()


def test_bucketed_allreduce_overlapped_with_backward_matches_one_flat_allreduce():
    """Gradient buckets all-reduced from post-accumulate hooks while backward runs give the same
    averaged gradients, bit for bit, as one all-reduce after backward (two gloo ranks)."""
    port = _free_port()
    with mp.get_context("spawn").Manager() as m:     # no fork of the test process
        results = m.dict()
        mp.spawn(_bucket_worker, args=(2, port, results), nprocs=2, join=True)
        results = dict(results)
    for r in range(2):
        for a, b in zip(results[r]["plain"], results[r]["buckets"]):
            assert torch.equal(a, b)
    for a, b in zip(results[0]["buckets"], results[1]["buckets"]):
        assert torch.equal(a, b)
