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
* `ppr_adjacency` follows `build_adj_fromat`, `NeutronGT/core/ppr_preprocess.py:30-71`:
  undirected keys (min, max) of the PPR list, each key's values summed in entry order
  (the reference's CPU scatter_add_) in float32, weight int32(max(sum * 1000, 1)); both
  directions listed and ordered by row with a stable sort (the reference's argsort is not
  stable, so it fixes no order inside a row; the oracle pins the stable one).
* `merge_related_nodes` follows `_merge_related_nodes`, `NeutronGT/core/metisPartition.py:397-425`:
  external neighbours of the window with their summed weights, ordered by weight (descending)
  with ties in first-encounter order, the first len * percent // 100 added, result sorted.
* `duplicate_rerange_nested` follows `_find_duplicate_nodes_and_rerange`,
  `metisPartition.py:333-363`: `duplicate_first` over every child window of every parent.
* `isolated_connections` follows `add_isolated_connections`, `NeutronGT/core/ppr_preprocess.py:94-132`,
  with the reference's dense torch.rand mask replaced by the per-pair SplitMix64 draw the device
  uses (Steele, Lea & Flood 2014), so its new edges are the device's exactly.
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


def ppr_adjacency(edge_index, values):
    """Returns (xadj int32 [n+1], adjncy int32 [2U], eweights int32 [2U]), n = max index + 1."""
    ei = np.asarray(edge_index, dtype=np.int64)
    val = np.asarray(values, dtype=np.float32)
    if ei.size == 0:
        return np.zeros(1, np.int32), np.zeros(0, np.int32), np.zeros(0, np.int32)
    n = int(ei.max()) + 1
    u = np.minimum(ei[0], ei[1])
    v = np.maximum(ei[0], ei[1])
    key = u * n + v
    order = np.argsort(key, kind="stable")
    uniq, first = np.unique(key[order], return_index=True)
    bounds = list(first) + [len(order)]
    sums = np.zeros(len(uniq), np.float32)
    for s in range(len(uniq)):
        acc = np.float32(0.0)
        for t in order[bounds[s]:bounds[s + 1]]:
            acc = np.float32(acc + val[t])
        sums[s] = acc
    w = np.maximum(sums * np.float32(1000.0), np.float32(1.0)).astype(np.int32)
    uu, vv = uniq // n, uniq % n
    rows = np.concatenate([uu, vv])
    cols = np.concatenate([vv, uu])
    ww = np.concatenate([w, w])
    o = np.argsort(rows, kind="stable")
    xadj = np.zeros(n + 1, np.int64)
    xadj[1:] = np.cumsum(np.bincount(rows, minlength=n))
    return xadj.astype(np.int32), cols[o].astype(np.int32), ww[o].astype(np.int32)


def merge_related_nodes(partition, xadj, adjncy, eweights, topk_percent):
    part = [int(x) for x in np.asarray(partition).reshape(-1)]
    inside = set(part)
    total, first = {}, {}
    pos = 0
    for x in part:
        for j in range(int(xadj[x]), int(xadj[x + 1])):
            nb = int(adjncy[j])
            if nb not in inside:
                total[nb] = total.get(nb, 0) + int(eweights[j])
                first.setdefault(nb, pos)
            pos += 1
    ranked = sorted(total, key=lambda nb: (-total[nb], first[nb]))
    k = len(ranked) * topk_percent // 100 if topk_percent > 0 else 0
    return torch.tensor(sorted(inside | set(ranked[:k])), dtype=torch.long)


def duplicate_rerange_nested(child_partitions):
    flat = [p for group in child_partitions for p in group]
    if not flat or sum(len(p) for p in flat) == 0:
        return child_partitions, []
    reranged, dups = duplicate_first(flat)
    it = iter(reranged)
    return [[next(it) for _ in group] for group in child_partitions], dups


_M64 = (1 << 64) - 1


def splitmix64(z):
    """Vectorised over uint64 arrays (wrap-around arithmetic)."""
    z = np.asarray(z, dtype=np.uint64)
    with np.errstate(over="ignore"):
        z = z + np.uint64(0x9E3779B97F4A7C15)
        z = (z ^ (z >> np.uint64(30))) * np.uint64(0xBF58476D1CE4E5B9)
        z = (z ^ (z >> np.uint64(27))) * np.uint64(0x94D049BB133111EB)
    return z ^ (z >> np.uint64(31))


def isolated_connections(ppr_edge_index, graph_edge_index, num_nodes, connect_prob, seed):
    """New edges [2, e_new] (int64): isolated nodes x appearing nodes, row-major, pair (a, b) kept
    when the top 32 bits of splitmix64(seed ^ splitmix64(a << 32 ^ b)) < floor(p * 2^32)."""
    seen = np.zeros(num_nodes, bool)
    for ei in (ppr_edge_index, graph_edge_index):
        ei = np.asarray(ei, dtype=np.int64).reshape(-1)
        seen[ei] = True
    iso = np.nonzero(~seen)[0]
    app = np.nonzero(seen)[0]
    if iso.size == 0 or app.size == 0:
        return np.zeros((2, 0), np.int64)
    thr = 0 if connect_prob <= 0 else (1 << 32 if connect_prob >= 1 else int(connect_prob * 4294967296.0))
    a = np.arange(iso.size, dtype=np.uint64)[:, None]
    b = np.arange(app.size, dtype=np.uint64)[None, :]
    inner = splitmix64((a << np.uint64(32)) ^ b)
    h = splitmix64(np.uint64(seed & _M64) ^ inner)
    mask = (h >> np.uint64(32)) < np.uint64(min(thr, (1 << 64) - 1))
    i, j = np.nonzero(mask)
    return np.stack([iso[i], app[j]])
