"""Heavy-row segments: the tables of `ngt_edge_csr_segments` and the segmented attention kernels.

Power-law windows put hundreds of entries in a few hub rows; those rows are cut into segments
of `seg_edges` entries handled by separate warps and added back in segment order.  Checked here:
the tables cover every entry of every heavy row exactly once with dense segment numbers; the
segmented kernels match the CPU oracle (fp32 1e-5, bf16 2e-2, max|a-b| / max|b|) and the
unsegmented entry points, with and without an attention bias; reruns are bitwise identical.
"""
import ctypes

import pytest
import torch

from conftest import rel_err
from oracle import attention as oatt

pytestmark = pytest.mark.gpu

F32_TOL = 1e-5
BF16_TOL = 2e-2


def _hub_edges(n, e, seed):
    """Uniform edges plus destination hubs (rows 7, 11) and a source hub (row 5)."""
    g = torch.Generator().manual_seed(seed)
    src = torch.randint(0, n, (e,), generator=g)
    dst = torch.randint(0, n, (e,), generator=g)
    dst[:900] = 7
    dst[900:1200] = 11
    src[1200:2000] = 5
    return torch.stack([src, dst])


def test_segment_tables_cover_heavy_rows(cuda):
    from neutrongt_b200.edge_csr import build_edge_csr, segment_edges
    n, e = 1500, 6000
    ei = _hub_edges(n, e, seed=1).cuda()
    csr = build_edge_csr(ei, n)
    T = segment_edges(n, e)
    assert csr.seg_edges == T == 16
    for view, rowptr, nseg in ((0, csr.dst_rowptr, csr.nseg_dst), (1, csr.src_rowptr, csr.nseg_src)):
        deg = (rowptr[1:] - rowptr[:-1]).cpu()
        first, rows, cnt = csr.seg_tables(view)
        assert cnt == nseg > 0
        first, rows = first.cpu(), rows[:cnt].cpu()
        heavy = deg > T
        assert torch.equal(first < 0, ~heavy)
        expect = ((deg[heavy] + T - 1) // T).sum().item()
        assert cnt == expect
        covered = torch.zeros(cnt, dtype=torch.int32)
        for r in torch.nonzero(heavy).flatten().tolist():
            k = (int(deg[r]) + T - 1) // T
            f = int(first[r])
            assert torch.all(rows[f:f + k] == r)
            covered[f:f + k] += 1
        assert torch.all(covered == 1)         # dense numbering, no overlap


def _run(fn_seg, q, k, v, ei, bias, dout):
    from neutrongt_b200 import _lib, sparse_attention_bias
    from neutrongt_b200.edge_csr import edge_csr_for
    qd, kd, vd = (t.clone().requires_grad_(True) for t in (q, k, v))
    bd = bias.clone().requires_grad_(True) if bias is not None else None
    if fn_seg:
        x, ns = sparse_attention_bias(qd, kd, vd, ei, bd)
        x.backward(dout)
        return x, ns, qd.grad, kd.grad, vd.grad, None if bd is None else bd.grad
    # unsegmented C entry points on the same CSR
    s, H, D = q.shape
    csr = edge_csr_for(ei, s)
    L = _lib.lib()
    st = _lib.stream_of(q)
    code = _lib.dtype_code(q.dtype)
    eb = None
    if bias is not None:
        src, dst = csr.dst_major_pairs()
        eb = bias[0].permute(1, 2, 0)[src, dst].contiguous()
    out = torch.empty_like(q)
    z = torch.empty(s, H, device=q.device)
    ns = torch.empty(csr.node_scores_len, device=q.device)
    assert L.ngt_spattn_forward(code, s, csr.e, H, D, _lib.ptr(q), _lib.ptr(k), _lib.ptr(v), _lib.ptr(csr.dst_rowptr),
                                _lib.ptr(csr.dst_src), _lib.ptr(eb), _lib.ptr(out), _lib.ptr(z), _lib.ptr(ns),
                                ns.numel(), st) == 0
    delta = torch.empty(s, H, device=q.device)
    dq, dk, dv = torch.empty_like(q), torch.empty_like(k), torch.empty_like(v)
    deb = torch.empty_like(eb) if eb is not None else None
    assert L.ngt_spattn_backward(code, s, csr.e, H, D, _lib.ptr(q), _lib.ptr(k), _lib.ptr(v), _lib.ptr(out),
                                 _lib.ptr(dout.contiguous()), _lib.ptr(z), _lib.ptr(csr.dst_rowptr),
                                 _lib.ptr(csr.dst_src), _lib.ptr(csr.src_rowptr), _lib.ptr(csr.src_dst),
                                 _lib.ptr(csr.src_to_dst_slot), _lib.ptr(eb), _lib.ptr(delta), _lib.ptr(dq),
                                 _lib.ptr(dk), _lib.ptr(dv), _lib.ptr(deb), st) == 0
    return out, ns, dq, dk, dv, deb


@pytest.mark.parametrize("H,D", [(8, 16), (8, 8), (4, 32)])
@pytest.mark.parametrize("dtype", [torch.float32, torch.bfloat16])
def test_segmented_matches_oracle_and_unsegmented(cuda, H, D, dtype):
    n, e = 1500, 6000
    g = torch.Generator().manual_seed(H * D)
    q, k, v, dout = (torch.randn(n, H, D, generator=g) * (1.5 if i < 2 else 1.0) for i in range(4))
    ei = _hub_edges(n, e, seed=H + D)
    q, k, v = (t.to(dtype) for t in (q, k, v))
    dd = [t.cuda() for t in (q, k, v)]
    x, ns, dq, dk, dv, _ = _run(True, *dd, ei.cuda(), None, dout.to(dtype).cuda())
    rx, rns, _, _ = oatt.sparse_attention_forward(q.double(), k.double(), v.double(), ei)
    rdq, rdk, rdv, _ = oatt.sparse_attention_backward(q.double(), k.double(), v.double(), ei, dout.to(dtype).double())
    tol = F32_TOL if dtype == torch.float32 else BF16_TOL
    for a, b in ((x, rx), (ns, rns), (dq, rdq), (dk, rdk), (dv, rdv)):
        assert rel_err(a, b) < tol
    ux, uns, udq, udk, udv, _ = _run(False, *dd, ei.cuda(), None, dout.to(dtype).cuda())
    same = 2e-6 if dtype == torch.float32 else 1e-2   # only the fp32 summation order differs
    for a, b in ((x, ux), (ns, uns), (dq, udq), (dk, udk), (dv, udv)):
        assert rel_err(a, b) < same


def test_segmented_with_bias_and_reruns(cuda):
    n, e, H, D = 1500, 6000, 8, 16
    g = torch.Generator().manual_seed(3)
    q, k, v, dout = (torch.randn(n, H, D, generator=g) for _ in range(4))
    ei = _hub_edges(n, e, seed=3)
    bias = torch.randn(1, H, n, n, generator=g) * 0.5
    dd = [t.cuda() for t in (q, k, v)]
    a = _run(True, *dd, ei.cuda(), bias.cuda(), dout.cuda())
    b = _run(True, *dd, ei.cuda(), bias.cuda(), dout.cuda())
    for ta, tb in zip(a, b):
        assert torch.equal(ta, tb)
    rx, rns, _, _ = oatt.sparse_attention_forward(q.double(), k.double(), v.double(), ei, bias.double())
    rdq, rdk, rdv, rdb = oatt.sparse_attention_backward(q.double(), k.double(), v.double(), ei, dout.double(),
                                                        bias.double())
    x, ns, dq, dk, dv, db = a
    for t, r in ((x, rx), (ns, rns), (dq, rdq), (dk, rdk), (dv, rdv), (db, rdb)):
        assert rel_err(t, r) < F32_TOL


def test_uniform_window_has_no_segments(cuda):
    from neutrongt_b200 import synthetic
    from neutrongt_b200.edge_csr import build_edge_csr
    rowptr, col = synthetic.poisson_window_csr(65536, 32.0, seed=0)
    ei = synthetic.edge_index_from_dst_csr(rowptr, col).cuda()
    csr = build_edge_csr(ei, 65536)
    assert csr.seg_edges == 128 and csr.nseg_dst == 0 and csr.nseg_src == 0
