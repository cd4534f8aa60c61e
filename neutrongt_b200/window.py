"""Window membership and window edge lists on the device.

* `subgraph_from_csr(node_set, rowptr, col)` — same contract and output order as the
  reference's `_subgraph_from_csr` (`NeutronGT/core/node_level_pipeline/window_state.py:92-119`),
  computed by `ngt_window_subgraph_count/_fill` (`csrc/csr.cu`).  Returns an int64
  [2, E_w] tensor on the device of `rowptr` (moved to CUDA when given on the host).
* `compute_local_duplicate_nodes(local_partitions)` — `window_state.py:52-73`:
  nodes that occur in two or more of a rank's windows move to the front of every
  window (both groups keep their order); returns (reranged windows, dup nodes per window).
"""
from __future__ import annotations

import torch

from . import _lib


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


def compute_local_duplicate_nodes(local_partitions):
    if not local_partitions:
        return [], []
    parts = [p.to(torch.long) for p in local_partitions]
    all_nodes = torch.cat(parts)
    if all_nodes.numel() == 0:
        return [p.clone() for p in parts], [p.new_empty(0) for p in parts]
    uniq, counts = torch.unique(all_nodes, return_counts=True, sorted=True)
    dup = uniq[counts >= 2]
    if dup.numel() == 0:
        return [p.clone() for p in parts], [p.new_empty(0) for p in parts]
    reranged, dups = [], []
    for p in parts:
        m = torch.isin(p, dup)
        reranged.append(torch.cat([p[m], p[~m]]))
        dups.append(p[m])
    return reranged, dups
