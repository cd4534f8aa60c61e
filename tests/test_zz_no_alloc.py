"""The allocation-free attention backward (`ngt_spattn_backward_noalloc`) on the GPU.

That entry point is for callers that cannot allocate device memory at the point where
they run the backward (a fixed memory budget with no allocator handle, or a host
runtime that does not own a CUDA allocator); it takes the per-row scratch from a fixed
array inside the library instead of a caller buffer.  These tests call it through the
C ABI and compare it with the regular `ngt_spattn_backward`, twice in a row, since the
array is shared between calls.  Both entry points run the same kernels on the same inputs, so
their gradients must be bitwise equal.  The file is named to be collected last.
"""
import ctypes

import pytest
import torch

pytestmark = pytest.mark.gpu

NOALLOC_MAX = 2097152        # NGT_NOALLOC_MAX_ROWS_X_HEADS in include/neutrongt_b200.h


def _window(n, e, heads, dim, dtype, seed):
    from neutrongt_b200.attention import WindowAttentionBuffers
    from neutrongt_b200.edge_csr import build_edge_csr
    g = torch.Generator(device="cuda").manual_seed(seed)
    q, k, v = (torch.randn(n, heads, dim, generator=g, device="cuda").to(dtype) for _ in range(3))
    ei = torch.randint(0, n, (2, e), generator=g, device="cuda")
    buf = WindowAttentionBuffers(q, k, v, build_edge_csr(ei, n))
    buf.forward()
    return buf


def _call(fn_name, buf, dout, with_delta):
    from neutrongt_b200 import _lib
    s, heads, dim = buf.shape
    c = buf.csr
    dq, dk, dv = torch.empty_like(buf.q), torch.empty_like(buf.k), torch.empty_like(buf.v)
    args = [buf.code, s, c.e, heads, dim, _lib.ptr(buf.q), _lib.ptr(buf.k), _lib.ptr(buf.v), _lib.ptr(buf.out),
            _lib.ptr(dout), _lib.ptr(buf.z), _lib.ptr(c.dst_rowptr), _lib.ptr(c.dst_src), _lib.ptr(c.src_rowptr),
            _lib.ptr(c.src_dst), None, None]
    if with_delta:
        delta = torch.empty(s, heads, dtype=torch.float32, device="cuda")
        args.append(_lib.ptr(delta))
    args += [_lib.ptr(dq), _lib.ptr(dk), _lib.ptr(dv), None, _lib.stream_of(buf.q)]
    rc = getattr(_lib.lib(), fn_name)(*args)
    torch.cuda.synchronize()
    return rc, (dq, dk, dv)


@pytest.mark.parametrize("dtype", [torch.float32, torch.bfloat16])
def test_noalloc_backward_matches_regular_entry_point(cuda, dtype):
    buf = _window(5000, 120000, 8, 16, dtype, seed=3)
    g = torch.Generator(device="cuda").manual_seed(4)
    douts = [torch.randn(buf.shape, generator=g, device="cuda").to(dtype) for _ in range(2)]
    for dout in douts:   # two calls in a row: the shared scratch keeps the previous call's data
        rc_ref, ref = _call("ngt_spattn_backward", buf, dout, with_delta=True)
        rc, got = _call("ngt_spattn_backward_noalloc", buf, dout, with_delta=False)
        assert rc_ref == 0 and rc == 0
        for a, b in zip(got, ref):
            assert torch.equal(a, b)


def test_noalloc_rejects_sizes_beyond_its_scratch(cuda):
    from neutrongt_b200 import _lib
    n, heads, dim = NOALLOC_MAX // 8 + 1, 8, 8
    x = torch.zeros(n, heads, dim, device="cuda")
    grads = [torch.full_like(x, 7.0) for _ in range(3)]
    rowptr = torch.zeros(n + 1, dtype=torch.int32, device="cuda")
    z = torch.zeros(n, heads, device="cuda")
    p = _lib.ptr
    rc = _lib.lib().ngt_spattn_backward_noalloc(0, n, 0, heads, dim, p(x), p(x), p(x), p(x), p(x), p(z), p(rowptr),
                                                None, p(rowptr), None, None, None, p(grads[0]), p(grads[1]),
                                                p(grads[2]), None, ctypes.c_void_p(0))
    torch.cuda.synchronize()
    assert _lib.status_name(rc) == "NGT_ERR_TOO_LARGE"
    for t in grads:      # rejected before any work: outputs untouched
        assert bool((t == 7.0).all())
