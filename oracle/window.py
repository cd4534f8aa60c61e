"""CPU restatement of window membership and window edge-list construction (test oracle only).

* `duplicate_first` follows `_compute_local_duplicate_nodes`,
  `NeutronGT/core/node_level_pipeline/window_state.py:52-73`: nodes present in two
  or more of a rank's windows move to the front of each window, both groups
  keeping their previous relative order.
* `subgraph_from_csr` follows `_subgraph_from_csr`, `window_state.py:92-119`:
  for each window node in window order (local source i), its global neighbours
  in CSR order that are also in the window, relabelled to their window
  position.  Output [2, E_w], row 0 = local source, row 1 = local destination.
* `subgraph_edge_filter` follows PyG `subgraph(subset, edge_index,
  relabel_nodes=True)` as called at `window_state.py:122-134` (torch_geometric
  2.4.0, not part of the reference tree): keep global edges whose two ends are
  in the window, in global edge order, relabelled to window positions.
* `stable_csr` builds the destination-major (or source-major) CSR of an edge
  list with ties kept in edge order — the layout the attention kernels read.
"""
from __future__ import annotations

import numpy as np
import torch


def duplicate_first(local_partitions):
    if not local_partitions:
        return [], []
    allnodes = np.concatenate([np.asarray(p, dtype=np.int64) for p in local_partitions])
    uniq, counts = np.unique(allnodes, return_counts=True)
    dup_set = uniq[counts >= 2]
    reranged, dups = [], []
    for p in local_partitions:
        arr = np.asarray(p, dtype=np.int64)
        m = np.isin(arr, dup_set)
        reranged.append(torch.from_numpy(np.concatenate([arr[m], arr[~m]])))
        dups.append(torch.from_numpy(arr[m].copy()))
    return reranged, dups


def subgraph_from_csr(node_set, rowptr, col):
    nodes = np.asarray(node_set, dtype=np.int64)
    rowptr = np.asarray(rowptr, dtype=np.int64)
    col = np.asarray(col, dtype=np.int64)
    if nodes.size == 0:
        return torch.empty((2, 0), dtype=torch.long)
    n_global = rowptr.size - 1
    local = np.full(n_global, -1, dtype=np.int64)
    local[nodes] = np.arange(nodes.size)
    starts = rowptr[nodes]
    ends = rowptr[nodes + 1]
    lengths = ends - starts
    src_rep = np.repeat(np.arange(nodes.size), lengths)
    offs = np.arange(lengths.sum()) - np.repeat(np.cumsum(lengths) - lengths, lengths)
    neigh = col[np.repeat(starts, lengths) + offs]
    loc = local[neigh]
    keep = loc >= 0
    return torch.from_numpy(np.stack([src_rep[keep], loc[keep]]).astype(np.int64))


def subgraph_edge_filter(subset, edge_index, num_nodes):
    subset = np.asarray(subset, dtype=np.int64)
    ei = np.asarray(edge_index, dtype=np.int64)
    local = np.full(int(num_nodes), -1, dtype=np.int64)
    local[subset] = np.arange(subset.size)
    a = local[ei[0]]
    b = local[ei[1]]
    keep = (a >= 0) & (b >= 0)
    return torch.from_numpy(np.stack([a[keep], b[keep]]).astype(np.int64))


def stable_csr(edge_index, n, by="dst"):
    """(rowptr [n+1], other-end [E], edge id [E]) sorted by `by` endpoint, ties in edge order."""
    ei = np.asarray(edge_index, dtype=np.int64)
    key = ei[1] if by == "dst" else ei[0]
    other = ei[0] if by == "dst" else ei[1]
    order = np.argsort(key, kind="stable")
    counts = np.bincount(key, minlength=int(n)) if key.size else np.zeros(int(n), dtype=np.int64)
    rowptr = np.zeros(int(n) + 1, dtype=np.int64)
    np.cumsum(counts, out=rowptr[1:])
    return torch.from_numpy(rowptr), torch.from_numpy(other[order]), torch.from_numpy(order.astype(np.int64))
