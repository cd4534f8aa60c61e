"""The C-ABI library loads and exports every symbol include/neutrongt_b200.h declares (no GPU)."""
import os
import re

from conftest import ROOT

HEADER = os.path.join(ROOT, "include", "neutrongt_b200.h")


def _declared():
    text = open(HEADER).read()
    return sorted(set(re.findall(r"^NGT_API\s+(?:int|const char \*)\s*(ngt_\w+)\(", text, flags=re.M)))


def test_header_declares_the_entry_points():
    names = _declared()
    assert "ngt_spattn_forward" in names and "ngt_ppr_appnp_topk" in names
    assert len(names) >= 11


def test_library_exports_every_declared_symbol():
    from neutrongt_b200 import _lib
    lib = _lib.lib()
    for name in _declared():
        assert hasattr(lib, name), name
        assert name in _lib.SIGNATURES, f"{name} has no ctypes signature"


def test_version_status_and_size_queries():
    from neutrongt_b200 import _lib
    lib = _lib.lib()
    assert lib.ngt_abi_version() == 1
    assert _lib.status_name(0) == "NGT_OK"
    assert _lib.status_name(3) == "NGT_ERR_WORKSPACE"
    assert _lib.size_query(lib.ngt_edge_csr_workspace_size, 65536, 2_000_000) > 2_000_000 * 28
    assert _lib.size_query(lib.ngt_window_subgraph_workspace_size, 169343, 10000) >= 169343 * 4
    # pruned PPR on a hub-heavy graph reserves per-CTA overflow tables
    # pruned PPR keeps every row on chip (a work counter only); unpruned needs two dense
    # fp64 vectors and presence flags per CTA
    assert 0 < _lib.size_query(lib.ngt_ppr_workspace_size, 169343, 11702, 8, 169343) < 4096
    assert _lib.size_query(lib.ngt_ppr_workspace_size, 10000, 100, 0, 100) >= 100 * 2 * 10000 * 9


def test_invalid_arguments_are_rejected_without_a_gpu():
    import ctypes

    from neutrongt_b200 import _lib
    lib = _lib.lib()
    out = ctypes.c_size_t(0)
    assert lib.ngt_edge_csr_workspace_size(-1, 5, ctypes.byref(out)) == 1
    assert lib.ngt_spattn_forward(7, 1, 1, 8, 8, *([None] * 9), 0, None) == 1   # bad dtype
    # row-wise operators: size query, unsupported widths and null pointers fail before any launch
    assert _lib.size_query(lib.ngt_rowops_workspace_size, 10583, 128) >= 2 * 128 * 4
    assert lib.ngt_layernorm_forward(10, 130, *([None] * 3), 1e-5, *([None] * 3), None) == 2
    assert lib.ngt_layernorm_forward(10, 2048, *([None] * 3), 1e-5, *([None] * 3), None) == 2
    assert lib.ngt_layernorm_forward(10, 128, *([None] * 3), 1e-5, *([None] * 3), None) == 1
    assert lib.ngt_layernorm_forward(0, 128, *([None] * 3), 1e-5, *([None] * 3), None) == 0
    assert lib.ngt_column_sum(-1, 128, None, None, None, 0, None) == 1
    # fp32 Linear: workspace query; inner dimensions above 256 are refused before any launch
    assert _lib.size_query(lib.ngt_linear_weight_workspace_size, 10583, 128, 256) >= (128 * 256 + 256) * 4
    assert lib.ngt_linear_forward(4, 260, 8, *([None] * 4), None) == 2
    assert lib.ngt_linear_backward_input(4, 8, 260, *([None] * 3), None) == 2
    assert lib.ngt_linear_forward(4, 6, 8, *([None] * 4), None) == 1           # features % 4 != 0
    assert lib.ngt_linear_forward(0, 8, 8, *([None] * 4), None) == 0
    assert lib.ngt_linear_status(None) == 1                                     # null output pointer
    # window construction: size queries; invalid arguments are refused before any launch
    assert _lib.size_query(lib.ngt_ppr_adjacency_workspace_size, 1000, 100) > 1000 * 4
    assert _lib.size_query(lib.ngt_halo_merge_workspace_size, 1000, 10, 50) >= 1000 * 4
    assert _lib.size_query(lib.ngt_duplicate_rerange_workspace_size, 1000, 50) >= 1000 * 4
    assert lib.ngt_halo_merge(10, None, None, None, 1, None, 0, 5, None, None, None, 0, None) == 1
    assert lib.ngt_duplicate_rerange(10, 1, None, None, 0, None, None, None, None, 0, None) == 1
    # CSR column check: negative sizes, entries without rows and null pointers are refused
    assert lib.ngt_csr_col32_checked(-1, 0, None, None, None, None, None) == 1
    assert lib.ngt_csr_col32_checked(0, 5, None, None, None, None, None) == 1
    assert lib.ngt_csr_col32_checked(4, 5, None, None, None, None, None) == 1


def test_bf16_linear_shape_checks_without_a_gpu():
    import ctypes

    from neutrongt_b200 import _lib
    lib = _lib.lib()
    out = ctypes.c_size_t(0)
    assert lib.ngt_linear_bf16_weight_workspace_size(1000, 30, 16, ctypes.byref(out)) == 1   # 30 % 8 != 0
    assert lib.ngt_linear_bf16_weight_workspace_size(32768, 768, 768, ctypes.byref(out)) == 0
    assert out.value >= 768 * 768 * 4
    assert lib.ngt_linear_bf16_forward(10, 64, 12, None, None, None, None, None) == 1        # 12 % 8 != 0


def test_new_entry_points_reject_bad_arguments_without_a_gpu():
    """Argument checks of the push PPR, SpGEMM and biased dense attention entry points run before any
    CUDA call (NGT_ERR_INVALID_ARGUMENT = 1, NGT_ERR_UNSUPPORTED = 2)."""
    import ctypes

    from neutrongt_b200 import _lib
    lib = _lib.lib()
    out = ctypes.c_size_t(0)
    assert lib.ngt_ppr_push_workspace_size(100, 0, ctypes.byref(out)) == 1
    assert lib.ngt_ppr_push_workspace_size(100, 4, ctypes.byref(out)) == 0 and out.value >= 4 * 100 * 29
    info = ctypes.c_void_p(16)      # never dereferenced: the checks fail first
    for alpha, eps in ((0.0, 1e-4), (1.5, 1e-4), (0.15, 0.0), (0.15, -1.0)):
        assert lib.ngt_ppr_push_topk(10, None, None, alpha, eps, 0, 10, 4, 1, None, None, None, None, info, None, 0,
                                     None) == 1
    assert lib.ngt_ppr_push_topk(10, None, None, 0.15, 1e-4, 5, 3, 4, 1, None, None, None, None, info, None, 0,
                                 None) == 1
    assert lib.ngt_csr_spgemm_workspace_size(-1, 10, 1, ctypes.byref(out)) == 1
    assert lib.ngt_csr_spgemm_workspace_size(10, 10, 2, ctypes.byref(out)) == 0 and out.value > 0
    assert lib.ngt_csr_spgemm_symbolic(4, 4, None, None, None, None, 1, None, None, 0, None) == 1
    st = ctypes.c_int32(0)
    dummy = ctypes.c_void_p(256)
    assert lib.ngt_dense_attn_forward_bias(64, 2, 72, 1.0, 0.5, 0.0, 0, dummy, dummy, dummy, dummy, 0, dummy, dummy,
                                           dummy, ctypes.byref(st), None) == 2          # head_dim > 64
    assert lib.ngt_dense_attn_forward_bias(64, 2, 16, 1.0, 0.5, 0.0, 0, dummy, dummy, dummy, dummy, 7, dummy, dummy,
                                           dummy, ctypes.byref(st), None) == 1          # bad head stride
