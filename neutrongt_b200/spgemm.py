"""`csr_spgemm` with the reference's contract, on the B200.

Same signature, checks and results as `csr_spgemm` (`NeutronGT/core/ppr_backends/cusparse_ops.py:
76-114`): six 1-D CUDA tensors (A's and B's rowptr / col / val; indices must fit int32, values are
taken as float32), B square; returns (rowptr_c int64 [m+1], col_c int64, val_c float32) with the
product's structural entries, columns ascending per row.  The product runs in `csrc/spgemm.cu`
(row-wise, one warp per row; every value summed in A's entry order in fp32).
"""
from __future__ import annotations

import torch

from . import _lib

_INT32_MAX = 2**31 - 1


def _require_cuda_tensor(tensor, name):
    if not isinstance(tensor, torch.Tensor):
        raise TypeError(f"{name} must be a torch.Tensor")
    if not tensor.is_cuda:
        raise RuntimeError(f"{name} must be a CUDA tensor for cuSPARSE")
    if tensor.dim() != 1:
        raise ValueError(f"{name} must be a 1-D tensor")


def _index(tensor, name, dtype):
    _require_cuda_tensor(tensor, name)
    if tensor.numel() > 0 and int(tensor.max().item()) > _INT32_MAX:
        raise RuntimeError(f"{name} contains indices that exceed the cuSPARSE int32 limit")
    return tensor.to(dtype=dtype).contiguous()


def _value(tensor, name):
    _require_cuda_tensor(tensor, name)
    return tensor.to(dtype=torch.float32).contiguous()


def _slots(m, n, device):
    sms = torch.cuda.get_device_properties(device).multi_processor_count
    free, _ = torch.cuda.mem_get_info(device)
    per = _lib.size_query(_lib.lib().ngt_csr_spgemm_workspace_size, 0, n, 1)
    cap = max(1, int(min(free // 4, 8 << 30) // per))
    return max(1, min(max(m, 1), 8 * sms, cap))


def csr_spgemm(rowptr_a, col_a, val_a, rowptr_b, col_b, val_b):
    ra = _index(rowptr_a, "rowptr_a", torch.int64)
    ca = _index(col_a, "col_a", torch.int32)
    va = _value(val_a, "val_a")
    rb = _index(rowptr_b, "rowptr_b", torch.int64)
    cb = _index(col_b, "col_b", torch.int32)
    vb = _value(val_b, "val_b")
    dev = ra.device
    if not all(t.device == dev for t in (ca, va, rb, cb, vb)):
        raise RuntimeError("A and B must be on the same CUDA device")
    m, n = ra.numel() - 1, rb.numel() - 1
    if m < 0 or n < 0:
        raise ValueError("rowptr tensors need at least one entry")
    if ca.numel() != va.numel() or cb.numel() != vb.numel():
        raise ValueError("col and val of a matrix must have the same length")
    if int(ra[-1].item()) != ca.numel() or int(rb[-1].item()) != cb.numel():
        raise ValueError("rowptr must end at the number of entries")
    if (ca.numel() and (int(ca.min().item()) < 0 or int(ca.max().item()) >= n)) or \
            (cb.numel() and (int(cb.min().item()) < 0 or int(cb.max().item()) >= n)):
        raise ValueError(f"column indices must lie in [0, {n}) (B is {n} x {n})")
    L = _lib.lib()
    slots = _slots(m, n, dev)
    ws = _lib.workspace(_lib.size_query(L.ngt_csr_spgemm_workspace_size, m, n, slots), dev)
    rowptr_c = torch.empty(m + 1, dtype=torch.long, device=dev)
    st = _lib.stream_of(ra)
    _lib.check(L.ngt_csr_spgemm_symbolic(m, n, _lib.ptr(ra), _lib.ptr(ca), _lib.ptr(rb), _lib.ptr(cb), slots,
                                         _lib.ptr(rowptr_c), _lib.ptr(ws), ws.numel(), st), "ngt_csr_spgemm_symbolic")
    nnz = int(rowptr_c[-1].item())
    col_c = torch.empty(nnz, dtype=torch.long, device=dev)
    val_c = torch.empty(nnz, dtype=torch.float32, device=dev)
    _lib.check(L.ngt_csr_spgemm_numeric(m, n, _lib.ptr(ra), _lib.ptr(ca), _lib.ptr(va), _lib.ptr(rb), _lib.ptr(cb),
                                        _lib.ptr(vb), slots, _lib.ptr(rowptr_c), _lib.ptr(col_c), _lib.ptr(val_c),
                                        _lib.ptr(ws), ws.numel(), st), "ngt_csr_spgemm_numeric")
    return rowptr_c, col_c, val_c
