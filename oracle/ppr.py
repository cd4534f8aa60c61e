"""CPU oracles for the two PPR backends (test infrastructure only).

APPNP PPR with per-iteration top-k:

`personal_pagerank_appnp` keeps the reference's call signature and argument
normalisation (`NeutronGT/core/ppr_backends/appnp_backend.py:203-310`) and runs the
arithmetic in `appnp_oracle.c` (canonical fp64 order; see that file's header).
Outputs follow the reference's format: edge_index [2, M] int64 (row 0 = seed,
row 1 = neighbour) and values [M] float32, seeds ascending, each seed's entries
in (value desc, column asc) order.

Push-based approximate PPR (`personal_pagerank_push`, the reference's `torch_geometric`
backend, `NeutronGT/core/ppr_backends/torch_geometric_backend.py:5-30`): `push_oracle.c`
restates the published push method (Andersen, Chung & Lang 2006, PPRGo variant) that PyG's
unvendored `get_ppr` implements; parity with PyG itself is unpinned (PyG is absent), the
restatement is checked against the method's error guarantee instead.
"""
from __future__ import annotations

import ctypes
import os
import subprocess

import numpy as np
import torch

_HERE = os.path.dirname(os.path.abspath(__file__))
_LIB_PATH = os.path.join(_HERE, "liboracle_appnp.so")
_lib = None


def build():
    subprocess.run(["make", "-s", "-C", _HERE], check=True)


def _load():
    global _lib
    if _lib is None:
        srcs = [os.path.join(_HERE, f) for f in ("appnp_oracle.c", "push_oracle.c")]
        if not os.path.exists(_LIB_PATH) or os.path.getmtime(_LIB_PATH) < max(os.path.getmtime(f) for f in srcs):
            build()
        lib = ctypes.CDLL(_LIB_PATH)
        f = lib.ngt_oracle_appnp
        f.restype = ctypes.c_int64
        i64, p = ctypes.c_int64, ctypes.c_void_p
        f.argtypes = [i64, p, p, ctypes.c_double, i64, i64, i64, i64, i64, i64, p, p, p, p, ctypes.c_double,
                      ctypes.c_int, p]
        g = lib.ngt_oracle_ppr_push
        g.restype = ctypes.c_int
        g.argtypes = [i64, p, p, ctypes.c_double, ctypes.c_double, i64, i64, i64, p, p, p, ctypes.c_int, p]
        _lib = lib
    return _lib


def normalize_args(num_nodes, topk, num_iterations, iter_topk, source_start, source_end):
    """Argument normalisation of `appnp_backend.py:219-248, :291`."""
    num_iterations = max(1, int(num_iterations))
    source_start = 0 if source_start is None else max(0, min(int(source_start), num_nodes))
    source_end = num_nodes if source_end is None else max(source_start, min(int(source_end), num_nodes))
    topk = min(int(topk), num_nodes)
    it = topk if iter_topk is None else int(iter_topk)
    it = None if it <= 0 else min(it, num_nodes)
    final_keep = topk if it is None else min(topk, it)
    return num_iterations, source_start, source_end, it, final_keep


def csr_from_edge_index(edge_index, num_nodes=None):
    """`_build_csr_from_edge_index` (`appnp_backend.py:36-58`): rows = src, cols sorted by (src, dst)."""
    ei = np.asarray(edge_index, dtype=np.int64)
    if ei.size == 0:
        return np.zeros(1, dtype=np.int64), np.zeros(0, dtype=np.int64), 0
    n = int(ei.max()) + 1 if num_nodes is None else int(num_nodes)
    order = np.lexsort((ei[1], ei[0]))
    src, dst = ei[0][order], ei[1][order]
    rowptr = np.zeros(n + 1, dtype=np.int64)
    np.cumsum(np.bincount(src, minlength=n), out=rowptr[1:])
    return rowptr, dst, n


def personal_pagerank_appnp(edge_index, alpha, topk=100, num_iterations=10, batch_size=8, device="cpu",
                            csr_data=None, num_nodes=None, iter_topk=None, source_start=None,
                            source_end=None, nthreads=1, return_fp64=False, stats=None, tie_rtol=1e-5):
    del batch_size, device  # seed batches do not change values (see appnp_oracle.c)
    if csr_data is not None:
        rowptr = np.ascontiguousarray(np.asarray(csr_data["rowptr"], dtype=np.int64))
        col = np.ascontiguousarray(np.asarray(csr_data["col"], dtype=np.int64))
        n = rowptr.size - 1
        if num_nodes is not None and int(num_nodes) != n:
            raise ValueError(f"CSR num_nodes mismatch: expected {num_nodes}, got {n}")
    else:
        if edge_index is None:
            raise ValueError("edge_index must be provided when csr_data is None")
        rowptr, col, n = csr_from_edge_index(edge_index, num_nodes)
    if n == 0:
        return torch.empty((2, 0), dtype=torch.long), torch.empty((0,), dtype=torch.float32)
    T, s0, s1, it, final_keep = normalize_args(n, topk, num_iterations, iter_topk, source_start, source_end)
    if s0 >= s1:
        return torch.empty((2, 0), dtype=torch.long), torch.empty((0,), dtype=torch.float32)
    stride = final_keep if final_keep > 0 else n + 1
    nseeds = s1 - s0
    out_col = np.zeros(nseeds * stride, dtype=np.int64)
    out_val = np.zeros(nseeds * stride, dtype=np.float64)
    out_cnt = np.zeros(nseeds, dtype=np.int32)
    out_tie = np.zeros(nseeds, dtype=np.uint8)
    st = np.zeros(2, dtype=np.int64)
    rc = _load().ngt_oracle_appnp(n, rowptr.ctypes.data, col.ctypes.data, float(alpha), T,
                                  it if it is not None else 0, final_keep, s0, s1, stride,
                                  out_col.ctypes.data, out_val.ctypes.data, out_cnt.ctypes.data,
                                  out_tie.ctypes.data, float(tie_rtol), int(nthreads), st.ctypes.data)
    if rc != 0:
        raise RuntimeError(f"oracle APPNP failed ({rc})")
    if stats is not None:
        stats["edges_touched"] = int(st[0])
        stats["state_entries"] = int(st[1])
        # seeds whose pruning boundary was a near tie at some iteration (the
        # reference's torch.topk may legitimately keep a different entry there)
        stats["near_tie_seeds"] = torch.from_numpy(np.nonzero(out_tie)[0] + s0)
    mask = np.arange(stride)[None, :] < out_cnt[:, None]
    cols = out_col.reshape(nseeds, stride)[mask]
    vals = out_val.reshape(nseeds, stride)[mask]
    seeds = np.repeat(np.arange(s0, s1, dtype=np.int64), out_cnt)
    ei = torch.from_numpy(np.stack([seeds, cols]))
    if return_fp64:
        return ei, torch.from_numpy(vals)
    return ei, torch.from_numpy(vals.astype(np.float32))


def personal_pagerank_push(edge_index, alpha, topk=100, eps=1e-6, csr_data=None, num_nodes=None, source_start=None,
                           source_end=None, nthreads=1, return_fp64=False, stats=None):
    """Push PPR of every seed in [source_start, source_end) (all nodes by default), then the
    reference's per-seed top-k (`torch_geometric_backend.py:14-28`).  Graph from `edge_index`
    (rows = sources, columns sorted by (src, dst), as PyG's get_ppr sorts it) or `csr_data`.
    Returns (edge_index [2, M] int64, values [M] float32, or fp64 with return_fp64)."""
    if csr_data is not None:
        rowptr = np.ascontiguousarray(np.asarray(csr_data["rowptr"], dtype=np.int64))
        col = np.asarray(csr_data["col"], dtype=np.int64)
        n = rowptr.size - 1
    else:
        rowptr, col, n = csr_from_edge_index(edge_index, num_nodes)
    col32 = np.ascontiguousarray(col.astype(np.int32))
    s0 = 0 if source_start is None else max(0, min(int(source_start), n))
    s1 = n if source_end is None else max(s0, min(int(source_end), n))
    topk = int(topk)
    if topk <= 0:
        raise ValueError("topk must be positive")
    nseeds = s1 - s0
    if nseeds == 0:
        return torch.empty((2, 0), dtype=torch.long), torch.empty((0,), dtype=torch.float64 if return_fp64 else
                                                                   torch.float32)
    cnt = np.zeros(nseeds, dtype=np.int64)
    idx = np.zeros(nseeds * topk, dtype=np.int64)
    val = np.zeros(nseeds * topk, dtype=np.float64)
    st = np.zeros(2, dtype=np.int64)
    rc = _load().ngt_oracle_ppr_push(n, rowptr.ctypes.data, col32.ctypes.data, float(alpha), float(eps), s0, s1,
                                     topk, cnt.ctypes.data, idx.ctypes.data, val.ctypes.data, int(nthreads),
                                     st.ctypes.data)
    if rc != 0:
        raise RuntimeError(f"oracle push PPR failed ({rc})")
    if stats is not None:
        stats["pushes"] = int(st[0])
        stats["edges_touched"] = int(st[1])
    mask = np.arange(topk)[None, :] < cnt[:, None]
    cols = idx.reshape(nseeds, topk)[mask]
    vals = val.reshape(nseeds, topk)[mask]
    seeds = np.repeat(np.arange(s0, s1, dtype=np.int64), cnt)
    ei = torch.from_numpy(np.stack([seeds, cols]))
    return ei, torch.from_numpy(vals if return_fp64 else vals.astype(np.float32))
