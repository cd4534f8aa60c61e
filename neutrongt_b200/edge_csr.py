"""Per-window CSR views of an attention edge list, built on the device and cached.

The reference indexes Q/K/V by `edge_index` and scatters by destination on every call
(`NeutronGT/models/gt_dist_node_level_single_window.py:130-178`).  The kernels here
read two CSR views instead — destination-major (forward, dq) and source-major
(dk, dv) — built once per edge-list tensor by `ngt_edge_csr_build` and reused by every
layer of the window's forward and backward.

The cache is keyed by the edge_index tensor object itself (weak reference) plus its
version counter and the node count, so a freed tensor whose memory is reused can never
hit a stale entry, and an in-place edit invalidates it.
"""
from __future__ import annotations

import ctypes
import weakref
from dataclasses import dataclass

import torch

from . import _lib


@dataclass
class EdgeCSR:
    n: int
    e: int
    dst_rowptr: torch.Tensor      # int32 [n+1]
    dst_src: torch.Tensor         # int32 [e]
    src_rowptr: torch.Tensor      # int32 [n+1]
    src_dst: torch.Tensor         # int32 [e]
    src_to_dst_slot: torch.Tensor  # int32 [e]
    max_dst: int                  # -1 when e == 0
    # heavy-row segments (ngt_edge_csr_segments): rows with more than seg_edges entries are
    # processed as segments of seg_edges entries by separate warps
    seg_edges: int = 0
    seg_first: torch.Tensor | None = None   # int32 [2n]: destination view, then source view
    seg_row: torch.Tensor | None = None     # int32 [2 * seg_cap]
    seg_cap: int = 0
    nseg_dst: int = 0
    nseg_src: int = 0

    def seg_tables(self, view: int):
        """(first, row, nseg) of one view (0 destination, 1 source); Nones when it has no segments."""
        nseg = self.nseg_dst if view == 0 else self.nseg_src
        if nseg == 0:
            return None, None, 0
        return (self.seg_first[view * self.n:(view + 1) * self.n],
                self.seg_row[view * self.seg_cap:(view + 1) * self.seg_cap], nseg)

    @property
    def node_scores_len(self) -> int:
        """torch_scatter's output length without dim_size: max(index) + 1 (0 if empty)."""
        return self.max_dst + 1

    def dst_major_pairs(self):
        """(src, dst) int64 of every dst-major slot, for gathering per-edge tensors."""
        counts = (self.dst_rowptr[1:] - self.dst_rowptr[:-1]).to(torch.long)
        dst = torch.repeat_interleave(torch.arange(self.n, device=counts.device), counts)
        return self.dst_src.to(torch.long), dst


def build_edge_csr(edge_index: torch.Tensor, n: int) -> EdgeCSR:
    _lib.require_cuda(edge_index)
    if edge_index.dim() != 2 or edge_index.shape[0] != 2:
        raise ValueError(f"edge_index must be [2, E], got {tuple(edge_index.shape)}")
    ei = edge_index.to(torch.long).contiguous()
    e = int(ei.shape[1])
    dev = ei.device
    L = _lib.lib()
    nbytes = _lib.size_query(L.ngt_edge_csr_workspace_size, n, e)
    ws = _lib.workspace(nbytes, dev)
    i32 = dict(dtype=torch.int32, device=dev)
    dst_rowptr = torch.empty(n + 1, **i32)
    src_rowptr = torch.empty(n + 1, **i32)
    dst_src = torch.empty(e, **i32)
    src_dst = torch.empty(e, **i32)
    s2d = torch.empty(e, **i32)
    info = torch.empty(4, **i32)       # [bad entries, max dst, segments dst view, segments src view]
    _lib.check(L.ngt_edge_csr_build(n, e, _lib.ptr(ei), _lib.ptr(dst_rowptr), _lib.ptr(dst_src),
                                    _lib.ptr(src_rowptr), _lib.ptr(src_dst), _lib.ptr(s2d),
                                    _lib.ptr(info), _lib.ptr(ws), ws.numel(), _lib.stream_of(ei)),
               "ngt_edge_csr_build")
    seg_edges = segment_edges(n, e)
    cap = ctypes.c_int64(0)
    _lib.check(L.ngt_edge_csr_segment_capacity(e, seg_edges, ctypes.byref(cap)), "ngt_edge_csr_segment_capacity")
    seg_first = torch.empty(max(2 * n, 1), **i32)
    seg_row = torch.empty(max(2 * cap.value, 1), **i32)
    _lib.check(L.ngt_edge_csr_segments(n, e, _lib.ptr(dst_rowptr), _lib.ptr(src_rowptr), seg_edges,
                                       _lib.ptr(seg_first), _lib.ptr(seg_row), _lib.ptr(info[2:]),
                                       _lib.stream_of(ei)), "ngt_edge_csr_segments")
    bad, max_dst, nseg_dst, nseg_src = (int(x) for x in info.tolist())
    if bad:
        raise IndexError(f"edge_index holds {bad} entries outside [0, {n})")
    return EdgeCSR(n, e, dst_rowptr, dst_src, src_rowptr, src_dst, s2d, max_dst, seg_edges, seg_first, seg_row,
                   int(cap.value), nseg_dst, nseg_src)


def segment_edges(n: int, e: int) -> int:
    """Entries per heavy-row segment: four times the mean degree, at least 16.  Rows up to that
    length stay one warp's work (uniform-degree windows never split); a hub row of a power-law
    window is spread over ceil(degree / seg_edges) warps."""
    mean = -(-e // max(n, 1))
    return max(16, 4 * mean)


# id(edge_index) -> (weak reference to it, (version, n), csr).  Identity is checked through
# the weak reference, never with tensor ==; the entry leaves when the tensor is freed.
_cache: dict = {}


def edge_csr_for(edge_index: torch.Tensor, n: int) -> EdgeCSR:
    """Cached `build_edge_csr` for this edge_index tensor object."""
    k = id(edge_index)
    key = (edge_index._version, int(n))
    hit = _cache.get(k)
    if hit is not None and hit[0]() is edge_index and hit[1] == key:
        return hit[2]
    csr = build_edge_csr(edge_index, n)

    def _drop(ref, k=k):
        cur = _cache.get(k)
        if cur is not None and cur[0] is ref:
            del _cache[k]

    _cache[k] = (weakref.ref(edge_index, _drop), key, csr)
    return csr


def clear_cache() -> None:
    _cache.clear()
