"""ctypes binding of the C ABI in include/neutrongt_b200.h (libneutrongt_b200.so).

The library is built in-tree by `make -C neutrongt_b200/csrc` (or
`__graft_entry__.build()`).  There is no fallback: if the shared library is missing,
every entry point raises.
"""
from __future__ import annotations

import ctypes
import os
import threading

import torch

_HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(_HERE, "libneutrongt_b200.so")

_i64 = ctypes.c_int64
_i32 = ctypes.c_int
_p = ctypes.c_void_p
_dbl = ctypes.c_double
_sz_p = ctypes.POINTER(ctypes.c_size_t)

# symbol -> argtypes (every declaration of include/neutrongt_b200.h)
SIGNATURES = {
    "ngt_abi_version": [],
    "ngt_status_string": [_i32],
    "ngt_edge_csr_workspace_size": [_i64, _i64, _sz_p],
    "ngt_edge_csr_build": [_i64, _i64, _p, _p, _p, _p, _p, _p, _p, _p, ctypes.c_size_t, _p],
    "ngt_spattn_forward": [_i32, _i64, _i64, _i32, _i32, _p, _p, _p, _p, _p, _p, _p, _p, _p, _i64, _p],
    "ngt_spattn_backward": [_i32, _i64, _i64, _i32, _i32, _p, _p, _p, _p, _p, _p, _p, _p, _p, _p, _p,
                            _p, _p, _p, _p, _p, _p, _p],
    "ngt_spattn_backward_noalloc": [_i32, _i64, _i64, _i32, _i32, _p, _p, _p, _p, _p, _p, _p, _p, _p, _p,
                                    _p, _p, _p, _p, _p, _p, _p],
    "ngt_edge_csr_segment_capacity": [_i64, _i32, ctypes.POINTER(ctypes.c_int64)],
    "ngt_edge_csr_segments": [_i64, _i64, _p, _p, _i32, _p, _p, _p, _p],
    "ngt_spattn_seg_part_size": [_i32, _i32, _i32, _i64, _i64, _sz_p],
    "ngt_spattn_forward_seg": [_i32, _i64, _i64, _i32, _i32, _p, _p, _p, _p, _p, _p, _p, _p, _p, _i64,
                               _i32, _p, _p, _i64, _p, _p],
    "ngt_spattn_backward_seg": [_i32, _i64, _i64, _i32, _i32, _p, _p, _p, _p, _p, _p, _p, _p, _p, _p,
                                _p, _p, _p, _p, _p, _p, _p, _i32, _p, _p, _i64, _p, _p, _i64, _p, _p],
    "ngt_dense_attn_forward": [_i64, _i32, _i32, ctypes.c_float, ctypes.c_float, ctypes.c_float, ctypes.c_uint64,
                               _p, _p, _p, _p, _p, _p, _p, _p],
    "ngt_dense_attn_backward": [_i64, _i32, _i32, ctypes.c_float, ctypes.c_float, ctypes.c_uint64, _p, _p, _p, _p,
                                _p, _p, _p, _p, _p, _p, _p, _p, _p],
    "ngt_dense_attn_forward_bias": [_i64, _i32, _i32, ctypes.c_float, ctypes.c_float, ctypes.c_float,
                                    ctypes.c_uint64, _p, _p, _p, _p, _i64, _p, _p, _p, _p, _p],
    "ngt_dense_attn_backward_bias": [_i64, _i32, _i32, ctypes.c_float, ctypes.c_float, ctypes.c_uint64, _p, _p, _p, _p,
                                     _p, _p, _p, _i64, _p, _p, _p, _p, _p, _p, _p, _p],
    "ngt_window_subgraph_workspace_size": [_i64, _i64, _sz_p],
    "ngt_window_subgraph_count": [_i64, _p, _p, _p, _i64, _p, _p, _p, ctypes.c_size_t, _p],
    "ngt_window_subgraph_fill": [_i64, _p, _p, _p, _i64, _p, _p, _i64, _p, ctypes.c_size_t, _p],
    "ngt_ppr_workspace_size": [_i64, _i64, _i64, _i64, _sz_p],
    "ngt_ppr_appnp_topk": [_i64, _p, _p, _p, _p, _dbl, _i64, _i64, _i64, _i64, _i64, _i64, _i64, _p, _p,
                           _p, _p, _p, _p, ctypes.c_size_t, _p],
    "ngt_ppr_adjacency_workspace_size": [_i64, _i64, _sz_p],
    "ngt_ppr_adjacency": [_i64, _i64, _p, _p, _p, _p, _p, _p, _p, ctypes.c_size_t, _p],
    "ngt_halo_degree": [_i64, _p, _i64, _p, _p, _p, ctypes.c_size_t, _p],
    "ngt_halo_merge_workspace_size": [_i64, _i64, _i64, _sz_p],
    "ngt_halo_merge": [_i64, _p, _p, _p, _i64, _p, _i64, _i32, _p, _p, _p, ctypes.c_size_t, _p],
    "ngt_duplicate_rerange_workspace_size": [_i64, _i64, _sz_p],
    "ngt_duplicate_rerange": [_i64, _i32, _p, _p, _i64, _p, _p, _p, _p, ctypes.c_size_t, _p],
    "ngt_isolated_connections_workspace_size": [_i64, _sz_p],
    "ngt_isolated_connections_count": [_i64, _i64, _p, _i64, _p, _dbl, ctypes.c_uint64, _p, _p, _p, ctypes.c_size_t,
                                       _p],
    "ngt_isolated_connections_fill": [_i64, _dbl, ctypes.c_uint64, _p, _i64, _p, _p, ctypes.c_size_t, _p],
    "ngt_rowops_workspace_size": [_i64, _i32, _sz_p],
    "ngt_layernorm_forward": [_i64, _i32, _p, _p, _p, ctypes.c_float, _p, _p, _p, _p],
    "ngt_layernorm_backward": [_i64, _i32, _p, _p, _p, _p, _p, _p, _p, _p, _p, ctypes.c_size_t, _p],
    "ngt_column_sum": [_i64, _i32, _p, _p, _p, ctypes.c_size_t, _p],
    "ngt_linear_forward": [_i64, _i32, _i32, _p, _p, _p, _p, _p],
    "ngt_linear_backward_input": [_i64, _i32, _i32, _p, _p, _p, _p],
    "ngt_linear_weight_workspace_size": [_i64, _i32, _i32, _sz_p],
    "ngt_linear_backward_weight": [_i64, _i32, _i32, _p, _p, _p, _p, _p, ctypes.c_size_t, _p],
    "ngt_linear_bf16_forward": [_i64, _i32, _i32, _p, _p, _p, _p, _p],
    "ngt_linear_bf16_backward_input": [_i64, _i32, _i32, _p, _p, _p, _p],
    "ngt_linear_bf16_weight_workspace_size": [_i64, _i32, _i32, _sz_p],
    "ngt_linear_bf16_backward_weight": [_i64, _i32, _i32, _p, _p, _p, _p, _p, ctypes.c_size_t, _p],
    "ngt_linear_status": [_p],
    "ngt_ppr_push_workspace_size": [_i64, _i64, _sz_p],
    "ngt_ppr_push_topk": [_i64, _p, _p, _dbl, _dbl, _i64, _i64, _i64, _i64, _p, _p, _p, _p, _p, _p, ctypes.c_size_t,
                          _p],
    "ngt_ppr_push_stats": [_p, _i64, _i64, _p, _p],
    "ngt_csr_col32_checked": [_i64, _i64, _p, _p, _p, _p, _p],
    "ngt_csr_spgemm_workspace_size": [_i64, _i64, _i64, _sz_p],
    "ngt_csr_spgemm_symbolic": [_i64, _i64, _p, _p, _p, _p, _i64, _p, _p, ctypes.c_size_t, _p],
    "ngt_csr_spgemm_numeric": [_i64, _i64, _p, _p, _p, _p, _p, _p, _i64, _p, _p, _p, _p, ctypes.c_size_t, _p],
}

NGT_F32 = 0
NGT_BF16 = 1

_lib = None
_lock = threading.Lock()


class NGTError(RuntimeError):
    """A neutrongt_b200 entry point returned a non-zero status."""


def lib():
    global _lib
    if _lib is None:
        with _lock:
            if _lib is None:
                if not os.path.exists(LIB_PATH):
                    raise RuntimeError(
                        f"neutrongt_b200 CUDA library not found at {LIB_PATH}; build it with "
                        "`make -C neutrongt_b200/csrc` (there is no CPU fallback)")
                h = ctypes.CDLL(LIB_PATH)
                for name, args in SIGNATURES.items():
                    fn = getattr(h, name)
                    fn.argtypes = args
                    fn.restype = ctypes.c_char_p if name == "ngt_status_string" else ctypes.c_int
                _lib = h
    return _lib


def status_name(rc: int) -> str:
    return lib().ngt_status_string(int(rc)).decode()


def check(rc: int, what: str) -> None:
    if rc != 0:
        raise NGTError(f"{what} failed with {status_name(rc)} ({rc})")


def ptr(t):
    """Device pointer of a tensor, or None for a missing optional argument."""
    return None if t is None else ctypes.c_void_p(t.data_ptr())


def stream_of(t: torch.Tensor):
    return ctypes.c_void_p(torch.cuda.current_stream(t.device).cuda_stream)


def require_cuda(*tensors):
    for t in tensors:
        if t is not None and not t.is_cuda:
            raise RuntimeError("neutrongt_b200 kernels need CUDA tensors (there is no CPU path)")


def dtype_code(dt: torch.dtype) -> int:
    if dt == torch.float32:
        return NGT_F32
    if dt == torch.bfloat16:
        return NGT_BF16
    raise TypeError(f"sparse window attention supports float32 and bfloat16, got {dt}")


def workspace(nbytes: int, device) -> torch.Tensor:
    return torch.empty(max(int(nbytes), 1), dtype=torch.uint8, device=device)


def size_query(fn, *args) -> int:
    out = ctypes.c_size_t(0)
    check(fn(*args, ctypes.byref(out)), fn.__name__)
    return int(out.value)
