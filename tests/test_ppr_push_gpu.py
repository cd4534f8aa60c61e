"""Push PPR (`personal_pagerank_torch_geometric`, the reference's default backend) on the GPU.

Checked bit for bit (fp64 values, entry order) against the CPU restatement of the push method
(oracle/push_oracle.c), which the CPU tests pin to the method's statement and its error guarantee.
Parity with PyG's own get_ppr is unpinned (PyG is not available here).
"""
import pytest
import torch

from oracle import ppr as oppr

pytestmark = pytest.mark.gpu


def _check(csr, alpha, eps, topk, s0=None, s1=None, slots=None):
    from neutrongt_b200.ppr import personal_pagerank_torch_geometric
    dev = torch.device("cuda")
    ei, v = personal_pagerank_torch_geometric(None, alpha, topk=topk, eps=eps, device=dev,
                                              csr_data={k: t.to(dev) for k, t in csr.items()}, source_start=s0,
                                              source_end=s1, return_fp64=True, slots=slots)
    rei, rv = oppr.personal_pagerank_push(None, alpha, topk=topk, eps=eps, csr_data=csr, source_start=s0,
                                          source_end=s1, return_fp64=True, nthreads=8)
    assert torch.equal(ei.cpu(), rei)
    assert torch.equal(v.cpu(), rv)
    return ei


@pytest.mark.parametrize("alpha,eps,topk", [(0.15, 1e-4, 10), (0.15, 1e-4, 100000), (0.85, 1e-5, 5), (0.3, 1e-3, 1)])
def test_matches_oracle_power_law(cuda, alpha, eps, topk):
    from neutrongt_b200 import synthetic
    rowptr, col = synthetic.chung_lu_graph(3000, 20000, seed=5)
    ei = _check({"rowptr": rowptr, "col": col}, alpha, eps, topk)
    assert ei.shape[1] > 0


def test_repeated_edges_and_sinks(cuda):
    """Repeated edges (equal neighbouring lanes: the sequential step) and nodes without out-edges."""
    g = torch.Generator().manual_seed(3)
    n = 500
    src = torch.randint(0, n, (6000,), generator=g)
    dst = torch.randint(0, n, (6000,), generator=g)
    src[:300] = 7
    dst[:300] = torch.randint(0, 40, (300,), generator=g)      # a hub row with many repeats
    keep = src % 11 != 0                                        # rows of multiples of 11 stay empty
    src, dst = src[keep], dst[keep]
    order = torch.argsort(src * n + dst, stable=True)
    src, dst = src[order], dst[order]
    rowptr = torch.zeros(n + 1, dtype=torch.long)
    rowptr[1:] = torch.cumsum(torch.bincount(src, minlength=n), 0)
    _check({"rowptr": rowptr, "col": dst}, 0.15, 1e-4, 16)
    _check({"rowptr": rowptr, "col": dst}, 0.2, 1e-6, 1000)


def test_seed_range_and_few_slots(cuda):
    from neutrongt_b200 import synthetic
    rowptr, col = synthetic.chung_lu_graph(20000, 150000, seed=8)
    _check({"rowptr": rowptr, "col": col}, 0.15, 1e-4, 10, s0=1234, s1=5678)
    _check({"rowptr": rowptr, "col": col}, 0.15, 1e-4, 10, s0=0, s1=700, slots=3)


def test_dispatcher_contract(cuda):
    from neutrongt_b200 import personal_pagerank
    from neutrongt_b200 import synthetic
    rowptr, col = synthetic.chung_lu_graph(400, 1600, seed=9)
    ei_in = synthetic.edge_index_from_src_csr(rowptr, col)
    ei, v = personal_pagerank(ei_in.cuda(), 0.15, topk=8, backend="torch_geometric", eps=1e-4)
    rei, rv = oppr.personal_pagerank_push(ei_in, 0.15, topk=8, eps=1e-4)
    assert torch.equal(ei.cpu(), rei) and torch.equal(v.cpu(), rv) and v.dtype == torch.float32
    with pytest.raises(NotImplementedError):
        personal_pagerank(ei_in.cuda(), 0.15, topk=8, backend="torch_geometric", source_start=0, source_end=10)


def test_csr_check_flags_and_unsorted_rows(cuda):
    """`ngt_csr_col32_checked` (one pass: range check, row order, int32 narrowing) directly, and
    through the wrapper: rows out of order give the sorted graph's result, a column outside [0, n)
    is refused."""
    from neutrongt_b200 import _lib, synthetic
    from neutrongt_b200.ppr import personal_pagerank_torch_geometric
    dev = torch.device("cuda")
    rowptr, col = synthetic.chung_lu_graph(3000, 60000, seed=9)
    rp, cl = rowptr.to(dev), col.to(dev)
    n, nnz = rp.numel() - 1, cl.numel()

    def flags_of(c):
        out = torch.empty(nnz, dtype=torch.int32, device=dev)
        f = torch.empty(1, dtype=torch.int32, device=dev)
        _lib.check(_lib.lib().ngt_csr_col32_checked(n, nnz, _lib.ptr(rp), _lib.ptr(c), _lib.ptr(out), _lib.ptr(f),
                                                    _lib.stream_of(c)), "ngt_csr_col32_checked")
        return int(f.item()), out

    f, out = flags_of(cl)
    assert f == 0 and torch.equal(out.long(), cl)
    # reverse every row: out of order wherever a row holds two or more distinct columns
    deg = rp[1:] - rp[:-1]
    row_of = torch.repeat_interleave(torch.arange(n, device=dev), deg)
    rev = cl[torch.argsort(row_of * n + (n - 1 - cl), stable=True)].contiguous()
    assert flags_of(rev)[0] == 2
    bad = cl.clone()
    bad[nnz // 2] = n
    assert flags_of(bad)[0] & 1
    bad[nnz // 2] = -1
    assert flags_of(bad)[0] & 1
    # through the wrapper
    args = dict(topk=10, eps=1e-4, device=dev, return_fp64=True)
    ei, v = personal_pagerank_torch_geometric(None, 0.15, csr_data={"rowptr": rp, "col": cl}, **args)
    ei2, v2 = personal_pagerank_torch_geometric(None, 0.15, csr_data={"rowptr": rp, "col": rev}, **args)
    assert torch.equal(ei, ei2) and torch.equal(v, v2)
    with pytest.raises(ValueError):
        personal_pagerank_torch_geometric(None, 0.15, csr_data={"rowptr": rp, "col": bad}, **args)
