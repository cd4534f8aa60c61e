"""Personalised PageRank on the B200: APPNP with per-iteration top-k, and push-based approximate PPR.

`personal_pagerank_appnp` and `personal_pagerank` keep the reference's signatures and
argument handling (`NeutronGT/core/ppr_backends/appnp_backend.py:203-310`,
`NeutronGT/core/ppr_preprocess.py:135-172`); the propagation, merge and top-k run in
the `ngt_ppr_appnp_topk` kernel (`csrc/ppr.cu`).

Output format as the reference: edge_index [2, M] int64 (row 0 = seed, row 1 =
neighbour) and values [M] float32 on `device`, seeds ascending.  Within a seed the
entries come in (value desc, column asc) order — the reference leaves rows that did
not need pruning unsorted, so the sets are what correspond.  Values are computed in
fp64 in a fixed order and rounded to float32 at the end.

`personal_pagerank_torch_geometric` is the reference's default backend
(`NeutronGT/core/ppr_backends/torch_geometric_backend.py:5-30`: PyG `get_ppr(edge_index, alpha, eps)`
and a per-source top-k): the push method of Andersen, Chung & Lang (PPRGo variant) runs in the
`ngt_ppr_push_topk` kernel (`csrc/ppr_push.cu`), bit-identical to the sequential method in fp64.
Seeds with more than `topk` entries keep the top `topk` by (value desc, node asc); others keep
the method's insertion order, as the reference leaves them.
"""
from __future__ import annotations

import torch

from . import _lib
from .edge_csr import build_edge_csr


def _graph_from_csr(csr_data, device, num_nodes):
    if csr_data is None:
        raise ValueError("csr_data must not be None when loading a CSR graph")
    if not isinstance(csr_data, dict):
        raise TypeError(f"Unsupported csr_data type: {type(csr_data)}")
    if "rowptr" not in csr_data or "col" not in csr_data:
        raise KeyError(f"CSR data must contain rowptr and col, got keys={list(csr_data.keys())}")
    rowptr = torch.as_tensor(csr_data["rowptr"], dtype=torch.long, device=device)
    col = torch.as_tensor(csr_data["col"], dtype=torch.long, device=device)
    if rowptr.dim() != 1 or col.dim() != 1:
        raise ValueError("CSR rowptr and col must be 1-D")
    n = int(rowptr.numel() - 1)
    if num_nodes is not None and n != int(num_nodes):
        raise ValueError(f"CSR num_nodes mismatch: expected {num_nodes}, got {n}")
    return rowptr, col, n


def _graph_from_edge_index(edge_index, device, num_nodes):
    """Rows = sources, columns sorted by (src, dst) (`appnp_backend.py:36-58`)."""
    if edge_index.numel() == 0:
        return torch.zeros(1, dtype=torch.long, device=device), torch.empty(0, dtype=torch.long, device=device), 0
    ei = edge_index.to(device=device, dtype=torch.long)
    n = int(ei.max().item()) + 1 if num_nodes is None else int(num_nodes)
    key = ei[0] * max(n, 1) + ei[1]
    key, _ = torch.sort(key)
    src = key // max(n, 1)
    dst = key % max(n, 1)
    rowptr = torch.zeros(n + 1, dtype=torch.long, device=device)
    rowptr[1:] = torch.cumsum(torch.bincount(src, minlength=n), 0)
    return rowptr, dst, n


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


def personal_pagerank_appnp(edge_index, alpha, topk=100, num_iterations: int = 10, batch_size: int = 8,
                            device="cuda", csr_data=None, num_nodes=None, iter_topk=None,
                            source_start=None, source_end=None, return_fp64: bool = False):
    device = torch.device(device) if not isinstance(device, torch.device) else device
    if device.type != "cuda":
        raise RuntimeError("APPNP backend requires a CUDA device")
    del batch_size  # every seed owns one CTA; batching does not change any value
    if csr_data is not None:
        rowptr, col, n = _graph_from_csr(csr_data, device, num_nodes)
    else:
        if edge_index is None:
            raise ValueError("edge_index must be provided when csr_data is None")
        rowptr, col, n = _graph_from_edge_index(edge_index, device, num_nodes)
    empty = (torch.empty((2, 0), dtype=torch.long, device=device),
             torch.empty((0,), dtype=torch.float64 if return_fp64 else torch.float32, device=device))
    if n == 0:
        return empty
    if n >= 2**31 - 1 or col.numel() >= 2**31 - 1:
        raise RuntimeError("graph exceeds the int32 index range of the PPR kernel")
    # the kernel indexes rowptr by every column it meets: reject malformed graphs up front
    if int(rowptr[0].item()) != 0 or int(rowptr[-1].item()) != col.numel() or bool((rowptr[1:] < rowptr[:-1]).any()):
        raise ValueError("CSR rowptr must start at 0, be non-decreasing and end at col.numel()")
    if col.numel() and (int(col.min().item()) < 0 or int(col.max().item()) >= n):
        raise ValueError(f"CSR col holds indices outside [0, {n})")
    T, s0, s1, it, final_keep = normalize_args(n, topk, num_iterations, iter_topk, source_start, source_end)
    if s0 >= s1:
        return empty
    col32 = col.to(torch.int32).contiguous()
    deg = rowptr[1:] - rowptr[:-1]
    max_deg = int(deg.max().item()) if n > 0 else 0
    dense = it is None
    in_rowptr = in_col = None
    if dense:
        if final_keep <= 0 or final_keep > 32:
            raise NotImplementedError("unpruned APPNP keeps 1..32 entries per seed on this backend")
        src = torch.repeat_interleave(torch.arange(n, device=device), deg)
        tcsr = build_edge_csr(torch.stack([src, col]), n)   # dst-major view = in-adjacency
        in_rowptr = tcsr.dst_rowptr.to(torch.long)
        in_col = tcsr.dst_src
    else:
        if it > 32:
            raise NotImplementedError("iter_topk above 32 is not supported by the PPR kernel")
        # the pruned kernel merges adjacency rows, so each row's columns must ascend (the
        # reference's CSR writer emits them that way); sort the rows of any other input once
        if col.numel() > 1:
            row_of = torch.repeat_interleave(torch.arange(n, device=device), deg)
            desc = (col[1:] < col[:-1]) & (row_of[1:] == row_of[:-1])
            if bool(desc.any()):
                order = torch.argsort(row_of * n + col, stable=True)
                col32 = col32[order].contiguous()
    stride = final_keep if final_keep > 0 else it
    nseeds = s1 - s0
    L = _lib.lib()
    nbytes = _lib.size_query(L.ngt_ppr_workspace_size, n, max_deg, it if it is not None else 0, nseeds)
    ws = _lib.workspace(nbytes, device)
    out_col = torch.empty(nseeds * stride, dtype=torch.long, device=device)
    out_val = torch.empty(nseeds * stride, dtype=torch.float32, device=device)
    out_val64 = torch.empty(nseeds * stride, dtype=torch.float64, device=device) if return_fp64 else None
    out_cnt = torch.empty(nseeds, dtype=torch.int32, device=device)
    info = torch.empty(1, dtype=torch.int32, device=device)
    _lib.check(L.ngt_ppr_appnp_topk(n, _lib.ptr(rowptr), _lib.ptr(col32), _lib.ptr(in_rowptr), _lib.ptr(in_col),
                                    float(alpha), T, it if it is not None else 0, final_keep, s0, s1, max_deg,
                                    stride, _lib.ptr(out_col), _lib.ptr(out_val), _lib.ptr(out_val64),
                                    _lib.ptr(out_cnt), _lib.ptr(info), _lib.ptr(ws), ws.numel(),
                                    _lib.stream_of(rowptr)),
               "ngt_ppr_appnp_topk")
    if int(info.item()) != 0:
        raise RuntimeError(f"PPR rows of {int(info.item())} seeds did not fit the workspace")
    cnt = out_cnt.to(torch.long)
    mask = torch.arange(stride, device=device)[None, :] < cnt[:, None]
    cols = out_col.view(nseeds, stride)[mask]
    vals = (out_val64 if return_fp64 else out_val).view(nseeds, stride)[mask]
    seeds = torch.repeat_interleave(torch.arange(s0, s1, device=device), cnt)
    return torch.stack([seeds, cols], dim=0), vals


def _col32_checked(rowptr, col, n):
    """col as int32 with its rows ascending, checked in one device pass (`ngt_csr_col32_checked`);
    rows out of order are sorted first (the order PyG's get_ppr sorts the edge list into).  Needs a
    validated rowptr."""
    col32 = torch.empty(col.numel(), dtype=torch.int32, device=col.device)
    flags = torch.empty(1, dtype=torch.int32, device=col.device)
    _lib.check(_lib.lib().ngt_csr_col32_checked(n, col.numel(), _lib.ptr(rowptr), _lib.ptr(col), _lib.ptr(col32),
                                                _lib.ptr(flags), _lib.stream_of(col)), "ngt_csr_col32_checked")
    f = int(flags.item())
    if f & 1:
        raise ValueError(f"CSR col holds indices outside [0, {n})")
    if f & 2:
        col32 = _sorted_rows(rowptr, col, n).to(torch.int32).contiguous()
    return col32


def _sorted_rows(rowptr, col, n):
    """Columns ascending within each row (the order PyG's get_ppr sorts the edge list into)."""
    if col.numel() <= 1:
        return col
    deg = rowptr[1:] - rowptr[:-1]
    row_of = torch.repeat_interleave(torch.arange(n, device=col.device), deg)
    if bool(((col[1:] < col[:-1]) & (row_of[1:] == row_of[:-1])).any()):
        col = col[torch.argsort(row_of * n + col, stable=True)]
    return col


def _push_slots(n, nseeds, device, slots=None):
    """Concurrent seeds (one warp and ~29 n bytes of workspace each): eight warps per SM (more slots
    measured slower: their scattered per-node arrays thrash the L2), capped at a quarter of the free
    device memory (16 GiB at most)."""
    if slots is not None:
        return max(1, min(int(slots), nseeds))
    sms = torch.cuda.get_device_properties(device).multi_processor_count
    free, _ = torch.cuda.mem_get_info(device)
    per = _lib.size_query(_lib.lib().ngt_ppr_push_workspace_size, n, 1)
    cap = max(1, int(min(free // 4, 16 << 30) // max(per, 1)))
    return max(1, min(nseeds, 8 * sms, cap))


def personal_pagerank_torch_geometric(edge_index, alpha, topk=100, eps: float = 1e-6, device="cuda", csr_data=None,
                                      num_nodes=None, source_start=None, source_end=None, return_fp64: bool = False,
                                      slots=None, stats=None):
    """Drop-in for `personal_pagerank_torch_geometric` (`torch_geometric_backend.py:5-30`), on the
    device.  Beyond the reference: a CSR graph (`csr_data`), a seed range (`source_start`,
    `source_end`, for sharding seeds over ranks) and fp64 values (`return_fp64`)."""
    device = torch.device(device) if not isinstance(device, torch.device) else device
    if device.type != "cuda":
        raise RuntimeError("the push PPR backend runs on a CUDA device")
    if csr_data is not None:
        rowptr, col, n = _graph_from_csr(csr_data, device, num_nodes)
    else:
        if edge_index is None:
            raise ValueError("edge_index must be provided when csr_data is None")
        rowptr, col, n = _graph_from_edge_index(edge_index, device, num_nodes)
    vdt = torch.float64 if return_fp64 else torch.float32
    empty = (torch.empty((2, 0), dtype=torch.long, device=device), torch.empty((0,), dtype=vdt, device=device))
    topk = int(topk)
    if topk <= 0:
        raise ValueError("topk must be positive")
    if not (0.0 < float(alpha) <= 1.0) or not float(eps) > 0.0:
        raise ValueError("alpha must lie in (0, 1] and eps must be positive")
    if n == 0:
        return empty
    if n >= 2**31 - 1 or col.numel() >= 2**31 - 1:
        raise RuntimeError("graph exceeds the int32 index range of the PPR kernel")
    if int(rowptr[0].item()) != 0 or int(rowptr[-1].item()) != col.numel() or bool((rowptr[1:] < rowptr[:-1]).any()):
        raise ValueError("CSR rowptr must start at 0, be non-decreasing and end at col.numel()")
    col32 = _col32_checked(rowptr, col.contiguous(), n)
    s0 = 0 if source_start is None else max(0, min(int(source_start), n))
    s1 = n if source_end is None else max(s0, min(int(source_end), n))
    if s0 >= s1:
        return empty
    nseeds = s1 - s0
    slots = _push_slots(n, nseeds, device, slots)
    L = _lib.lib()
    ws = _lib.workspace(_lib.size_query(L.ngt_ppr_push_workspace_size, n, slots), device)
    out_idx = torch.empty(nseeds * topk, dtype=torch.long, device=device)
    out_val = torch.empty(nseeds * topk, dtype=torch.float32, device=device)
    out_val64 = torch.empty(nseeds * topk, dtype=torch.float64, device=device) if return_fp64 else None
    out_cnt = torch.empty(nseeds, dtype=torch.int32, device=device)
    info = torch.empty(1, dtype=torch.int32, device=device)
    st = _lib.stream_of(rowptr)
    _lib.check(L.ngt_ppr_push_topk(n, _lib.ptr(rowptr), _lib.ptr(col32), float(alpha), float(eps), s0, s1, topk, slots,
                                   _lib.ptr(out_idx), _lib.ptr(out_val), _lib.ptr(out_val64), _lib.ptr(out_cnt),
                                   _lib.ptr(info), _lib.ptr(ws), ws.numel(), st), "ngt_ppr_push_topk")
    if int(info.item()) != 0:
        raise RuntimeError(f"push PPR stopped {int(info.item())} seeds at the termination guard")
    if stats is not None:
        import ctypes
        pr = (ctypes.c_int64 * 2)()
        _lib.check(L.ngt_ppr_push_stats(_lib.ptr(ws), n, slots, pr, st), "ngt_ppr_push_stats")
        stats["pushes"], stats["edges_touched"], stats["slots"] = int(pr[0]), int(pr[1]), slots
    cnt = out_cnt.to(torch.long)
    mask = torch.arange(topk, device=device)[None, :] < cnt[:, None]
    cols = out_idx.view(nseeds, topk)[mask]
    vals = (out_val64 if return_fp64 else out_val).view(nseeds, topk)[mask]
    seeds = torch.repeat_interleave(torch.arange(s0, s1, device=device), cnt)
    return torch.stack([seeds, cols], dim=0), vals


def personal_pagerank(edge_index, alpha, topk=100, max_iter: int = 100, device="cuda",
                      backend: str = "torch_geometric", num_iterations=None, batch_size: int = 8,
                      eps: float = 1e-6, csr_data=None, num_nodes=None, iter_topk=None,
                      source_start=None, source_end=None):
    """Dispatcher with the signature of `NeutronGT/core/ppr_preprocess.py:135-172`."""
    if backend == "torch_geometric":
        if source_start is not None or source_end is not None:
            raise NotImplementedError("torch_geometric backend does not support distributed source sharding")
        # the reference reads edge_index only; a CSR graph is accepted when no edge list is given
        return personal_pagerank_torch_geometric(edge_index, alpha, topk=topk, eps=eps, device=device,
                                                 csr_data=csr_data if edge_index is None else None,
                                                 num_nodes=num_nodes)
    if backend == "appnp":
        if num_iterations is None:
            num_iterations = max_iter
        return personal_pagerank_appnp(edge_index, alpha, topk=topk, num_iterations=num_iterations,
                                       batch_size=batch_size, device=device, csr_data=csr_data,
                                       num_nodes=num_nodes, iter_topk=iter_topk,
                                       source_start=source_start, source_end=source_end)
    raise ValueError(f"Unsupported PPR backend: {backend}")
