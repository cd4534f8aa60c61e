"""Window membership and window edge lists on the device.

* `subgraph_from_csr(node_set, rowptr, col)` — same contract and output order as the
  reference's `_subgraph_from_csr` (`NeutronGT/core/node_level_pipeline/window_state.py:92-119`),
  computed by `ngt_window_subgraph_count/_fill` (`csrc/csr.cu`).  Returns an int64
  [2, E_w] tensor on the device of `rowptr` (moved to CUDA when given on the host).
* `compute_local_duplicate_nodes(local_partitions)` — `window_state.py:52-73`:
  nodes that occur in two or more of a rank's windows move to the front of every
  window (both groups keep their order); returns (reranged windows, dup nodes per window).
  Computed by `ngt_duplicate_rerange` (`csrc/windows.cu`); results on the input's device.
* `build_adj_format(sorted_ppr_matrix)` — `NeutronGT/core/ppr_preprocess.py:30-71`
  (`build_adj_fromat`): the symmetric, integer-weighted PPR adjacency, by `ngt_ppr_adjacency`.
  Returns (CSRAdjacency(adj_starts, adjacent), eweights, None) with int32 CUDA tensors where the
  reference returns a pymetis CSRAdjacency of lists and a list.
* `merge_related_nodes(partition, csr_adjacency, eweights, topk_percent)` —
  `NeutronGT/core/metisPartition.py:397-425`: the window plus the topk_percent % of its external
  neighbours with the largest summed edge weight, sorted (`ngt_halo_degree`, `ngt_halo_merge`).
* `find_duplicate_nodes_and_rerange(child_partitions)` — `metisPartition.py:333-363` over the
  nested [parent][child] window lists; returns (reranged child_partitions, dup nodes per window).
* `add_isolated_connections(ppr_result, original_edge_index, num_nodes, connect_prob,
  ppr_fill_value, device, seed)` — `NeutronGT/core/ppr_preprocess.py:94-132`: random links from
  isolated nodes to appearing ones, by `ngt_isolated_connections_count/_fill`, with a seeded
  counter-based draw per pair instead of a dense torch.rand matrix.
"""
from __future__ import annotations

from dataclasses import dataclass

import torch

from . import _lib


@dataclass
class CSRAdjacency:
    """The fields of pymetis.CSRAdjacency that the window code reads, as int32 device tensors."""
    adj_starts: torch.Tensor
    adjacent: torch.Tensor


def _cuda(device=None):
    return torch.device(device) if device is not None else torch.device("cuda", torch.cuda.current_device())


def subgraph_from_csr(node_set, rowptr, col, device=None):
    device = torch.device(device) if device is not None else (
        rowptr.device if rowptr.is_cuda else torch.device("cuda"))
    nodes = torch.as_tensor(node_set, dtype=torch.long).to(device).contiguous()
    if nodes.numel() == 0:
        return torch.empty((2, 0), dtype=torch.long, device=device)
    rp = rowptr.to(device=device, dtype=torch.long).contiguous()
    cl = col.to(device=device, dtype=torch.long).contiguous()
    n_global = int(rp.numel() - 1)
    w = int(nodes.numel())
    L = _lib.lib()
    nbytes = _lib.size_query(L.ngt_window_subgraph_workspace_size, n_global, w)
    ws = _lib.workspace(nbytes, device)
    out_rowptr = torch.empty(w + 1, dtype=torch.long, device=device)
    info = torch.empty(1, dtype=torch.int32, device=device)
    st = _lib.stream_of(rp)
    _lib.check(L.ngt_window_subgraph_count(n_global, _lib.ptr(rp), _lib.ptr(cl), _lib.ptr(nodes), w,
                                           _lib.ptr(out_rowptr), _lib.ptr(info), _lib.ptr(ws), ws.numel(), st),
               "ngt_window_subgraph_count")
    total = int(out_rowptr[-1].item())
    if int(info.item()) != 0:
        raise ValueError(f"window node list has {int(info.item())} out-of-range or repeated entries")
    out = torch.empty((2, total), dtype=torch.long, device=device)
    _lib.check(L.ngt_window_subgraph_fill(n_global, _lib.ptr(rp), _lib.ptr(cl), _lib.ptr(nodes), w,
                                          _lib.ptr(out_rowptr), _lib.ptr(out), total, _lib.ptr(ws),
                                          ws.numel(), st),
               "ngt_window_subgraph_fill")
    return out


def duplicate_rerange(partitions, device=None):
    """Duplicate-first order of a list of windows on the device: (reranged, dup nodes) per window,
    as int64 tensors on `device` (default: the current CUDA device)."""
    dev = _cuda(device)
    parts = [torch.as_tensor(p, dtype=torch.long).reshape(-1) for p in partitions]
    if not parts:
        return [], []
    lens = torch.tensor([p.numel() for p in parts], dtype=torch.long)
    offsets = torch.zeros(len(parts) + 1, dtype=torch.long)
    offsets[1:] = torch.cumsum(lens, 0)
    total = int(offsets[-1])
    nodes = torch.cat(parts).to(dev).contiguous() if total else torch.empty(0, dtype=torch.long, device=dev)
    if total and int(nodes.min()) < 0:
        raise ValueError("window node ids must be non-negative")
    n = int(nodes.max()) + 1 if total else 0
    L = _lib.lib()
    ws = _lib.workspace(_lib.size_query(L.ngt_duplicate_rerange_workspace_size, n, total), dev)
    out = torch.empty_like(nodes)
    dup_counts = torch.empty(len(parts), dtype=torch.long, device=dev)
    bad = torch.empty(1, dtype=torch.int32, device=dev)
    off_d = offsets.to(dev)
    _lib.check(L.ngt_duplicate_rerange(n, len(parts), _lib.ptr(off_d), _lib.ptr(nodes), total, _lib.ptr(out),
                                       _lib.ptr(dup_counts), _lib.ptr(bad), _lib.ptr(ws), ws.numel(),
                                       _lib.stream_of(nodes)), "ngt_duplicate_rerange")
    nd = dup_counts.tolist()
    reranged, dups = [], []
    for k in range(len(parts)):
        a, b = int(offsets[k]), int(offsets[k + 1])
        reranged.append(out[a:b])
        dups.append(out[a:a + nd[k]])
    return reranged, dups


def compute_local_duplicate_nodes(local_partitions):
    if not local_partitions:
        return [], []
    src_dev = torch.as_tensor(local_partitions[0]).device
    reranged, dups = duplicate_rerange(local_partitions)
    return [r.to(src_dev) for r in reranged], [d.to(src_dev) for d in dups]


def find_duplicate_nodes_and_rerange(child_partitions):
    """`metisPartition.py:333-363`: duplicate-first order over every child window of every parent.
    Returns (reranged child_partitions, dup nodes per window in flattened order); with no windows,
    or no nodes at all, the input and an empty list, as the reference leaves them."""
    flat = [p for group in child_partitions for p in group]
    if not flat or sum(torch.as_tensor(p).numel() for p in flat) == 0:
        return child_partitions, []
    src_dev = torch.as_tensor(flat[0]).device
    reranged, dups = duplicate_rerange(flat)
    it = iter(reranged)
    groups = [[next(it).to(src_dev) for _ in group] for group in child_partitions]
    return groups, [d.to(src_dev) for d in dups]


def build_adj_format(sorted_ppr_matrix, device=None):
    edge_index, ppr_val = sorted_ppr_matrix
    assert edge_index.shape[0] == 2
    dev = _cuda(device)
    if edge_index.numel() == 0:
        return (CSRAdjacency(torch.zeros(1, dtype=torch.int32, device=dev), torch.empty(0, dtype=torch.int32, device=dev)),
                torch.empty(0, dtype=torch.int32, device=dev), None)
    if ppr_val.dtype != torch.float32:
        raise TypeError(f"PPR values must be float32 (the PPR backends' output), got {ppr_val.dtype}")
    ei = edge_index.to(device=dev, dtype=torch.long).contiguous()
    val = ppr_val.to(dev).contiguous()
    m = int(ei.shape[1])
    n = int(ei.max()) + 1
    L = _lib.lib()
    ws = _lib.workspace(_lib.size_query(L.ngt_ppr_adjacency_workspace_size, m, n), dev)
    i32 = dict(dtype=torch.int32, device=dev)
    xadj = torch.empty(n + 1, **i32)
    adjncy = torch.empty(2 * m, **i32)
    eweights = torch.empty(2 * m, **i32)
    info = torch.empty(2, **i32)
    _lib.check(L.ngt_ppr_adjacency(m, n, _lib.ptr(ei), _lib.ptr(val), _lib.ptr(xadj), _lib.ptr(adjncy),
                                   _lib.ptr(eweights), _lib.ptr(info), _lib.ptr(ws), ws.numel(), _lib.stream_of(ei)),
               "ngt_ppr_adjacency")
    bad, u = (int(x) for x in info.tolist())
    if bad:
        raise IndexError(f"PPR edge_index holds {bad} negative entries")
    return CSRAdjacency(xadj, adjncy[:2 * u]), eweights[:2 * u], None


def merge_related_nodes(partition, csr_adjacency, eweights, topk_percent, device=None):
    dev = _cuda(device)
    xadj = torch.as_tensor(csr_adjacency.adj_starts).to(device=dev, dtype=torch.int32).contiguous()
    adjncy = torch.as_tensor(csr_adjacency.adjacent).to(device=dev, dtype=torch.int32).contiguous()
    ew = torch.as_tensor(eweights).to(device=dev, dtype=torch.int32).contiguous()
    part = torch.as_tensor(partition).to(device=dev, dtype=torch.long).reshape(-1).contiguous()
    n, p = int(xadj.numel()) - 1, int(part.numel())
    if p and (int(part.min()) < 0 or int(part.max()) >= n):
        raise IndexError(f"window node ids must lie in [0, {n})")
    pct = int(topk_percent)
    L = _lib.lib()
    st = _lib.stream_of(xadj)
    total = torch.zeros(1, dtype=torch.long, device=dev)
    ws0 = _lib.workspace(_lib.size_query(L.ngt_halo_merge_workspace_size, n, p, 0), dev)
    _lib.check(L.ngt_halo_degree(n, _lib.ptr(xadj), p, _lib.ptr(part), _lib.ptr(total), _lib.ptr(ws0), ws0.numel(), st),
               "ngt_halo_degree")
    t = int(total.item())
    ws = _lib.workspace(_lib.size_query(L.ngt_halo_merge_workspace_size, n, p, t), dev)
    out = torch.empty(max(p + t, 1), dtype=torch.long, device=dev)
    counts = torch.zeros(3, dtype=torch.long, device=dev)
    _lib.check(L.ngt_halo_merge(n, _lib.ptr(xadj), _lib.ptr(adjncy), _lib.ptr(ew), p, _lib.ptr(part), t, pct,
                                _lib.ptr(out), _lib.ptr(counts), _lib.ptr(ws), ws.numel(), st), "ngt_halo_merge")
    merged = int(counts[0].item())
    return out[:merged]


def add_isolated_connections(ppr_result, original_edge_index, num_nodes, connect_prob=0.01, ppr_fill_value=0.001,
                             device="cuda", seed=0):
    edge_index, edge_values = ppr_result
    dev = torch.device(device)
    if dev.type != "cuda":
        raise RuntimeError("add_isolated_connections runs on CUDA devices (there is no CPU path)")
    if dev.index is None:
        dev = _cuda()
    edge_index = edge_index.to(dev)
    edge_values = edge_values.to(dev)
    ppr = edge_index.to(torch.long).contiguous()
    orig = original_edge_index.to(device=dev, dtype=torch.long).contiguous()
    n = int(num_nodes)
    L = _lib.lib()
    ws = _lib.workspace(_lib.size_query(L.ngt_isolated_connections_workspace_size, n), dev)
    counts = torch.zeros(3, dtype=torch.long, device=dev)
    bad = torch.zeros(1, dtype=torch.int32, device=dev)
    st = _lib.stream_of(ppr)
    seed64 = int(seed) & 0xFFFFFFFFFFFFFFFF
    _lib.check(L.ngt_isolated_connections_count(n, int(ppr.shape[1]), _lib.ptr(ppr), int(orig.shape[1]),
                                                _lib.ptr(orig), float(connect_prob), seed64, _lib.ptr(counts),
                                                _lib.ptr(bad), _lib.ptr(ws), ws.numel(), st),
               "ngt_isolated_connections_count")
    n_iso, n_app, e_new = (int(x) for x in counts.tolist())
    if int(bad.item()):
        raise IndexError(f"edge lists hold node ids outside [0, {n})")
    if n_iso == 0 or n_app == 0 or e_new == 0:
        return edge_index, edge_values
    new_edges = torch.empty((2, e_new), dtype=torch.long, device=dev)
    _lib.check(L.ngt_isolated_connections_fill(n, float(connect_prob), seed64, _lib.ptr(counts), e_new,
                                               _lib.ptr(new_edges), _lib.ptr(ws), ws.numel(), st),
               "ngt_isolated_connections_fill")
    new_values = torch.full((e_new,), ppr_fill_value, device=dev, dtype=edge_values.dtype)
    return torch.cat([edge_index, new_edges.to(edge_index.dtype)], dim=1), torch.cat([edge_values, new_values], dim=0)
