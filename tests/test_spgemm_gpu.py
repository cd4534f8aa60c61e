"""`csr_spgemm` (the reference's cuSPARSE SpGEMM contract) on the GPU, bit for bit against the
row-wise restatement in oracle/spgemm.py (itself held to SciPy's row-wise product on the CPU), and
against SciPy directly where no entry cancels."""
import numpy as np
import pytest
import scipy.sparse as sp
import torch

from oracle import spgemm as osg

pytestmark = pytest.mark.gpu


def _rand_csr(rows, cols, nnz, seed, positive=True, dups=False):
    g = np.random.default_rng(seed)
    r = g.integers(0, rows, nnz)
    c = g.integers(0, cols, nnz)
    v = (g.random(nnz) + 0.1 if positive else g.standard_normal(nnz)).astype(np.float32)
    if dups:      # CSR built directly, so repeated (row, column) entries stay separate
        r[: nnz // 8], c[: nnz // 8] = r[nnz // 8: nnz // 4], c[nnz // 8: nnz // 4]
        order = np.lexsort((c, r))
        indptr = np.zeros(rows + 1, dtype=np.int64)
        np.cumsum(np.bincount(r, minlength=rows), out=indptr[1:])
        return sp.csr_matrix((v[order], c[order], indptr), shape=(rows, cols))
    mat = sp.csr_matrix((v, (r, c)), shape=(rows, cols))
    mat.sum_duplicates()
    mat.sort_indices()
    return mat


def _ours(a, b):
    from neutrongt_b200.spgemm import csr_spgemm
    t = lambda x, dt: torch.from_numpy(np.asarray(x).astype(dt)).cuda()  # noqa: E731
    rp, cl, vl = csr_spgemm(t(a.indptr, np.int64), t(a.indices, np.int64), t(a.data, np.float32),
                            t(b.indptr, np.int64), t(b.indices, np.int32), t(b.data, np.float32))
    assert rp.dtype == torch.long and cl.dtype == torch.long and vl.dtype == torch.float32
    return rp.cpu().numpy(), cl.cpu().numpy(), vl.cpu().numpy()


@pytest.mark.parametrize("m,n,nnz_a,nnz_b,seed", [(40, 60, 200, 500, 1), (1, 30, 5, 100, 2), (25, 25, 0, 100, 3),
                                                  (300, 2000, 3000, 40000, 4), (64, 5000, 640, 400000, 5)])
def test_matches_oracle_and_scipy(cuda, m, n, nnz_a, nnz_b, seed):
    a = _rand_csr(m, n, nnz_a, seed)
    b = _rand_csr(n, n, nnz_b, seed + 100)
    rp, cl, vl = _ours(a, b)
    orp, ocl, ovl = osg.csr_spgemm(a.indptr, a.indices, a.data, b.indptr, b.indices, b.data)
    assert np.array_equal(rp, orp) and np.array_equal(cl, ocl)
    assert np.array_equal(vl.view(np.uint32), ovl.view(np.uint32))
    c = (a @ b).tocsr()
    c.sort_indices()
    assert np.array_equal(rp, c.indptr) and np.array_equal(cl, c.indices)
    assert np.array_equal(vl.view(np.uint32), c.data.astype(np.float32).view(np.uint32))


def test_repeated_entries_signed_values_and_long_rows(cuda):
    """Repeated columns inside a row (the sequential step), cancelling sums kept as 0, and output
    rows longer than the shared-memory sort buffer (sorted in global memory)."""
    a = _rand_csr(20, 3000, 400, 7, positive=False, dups=True)
    b = _rand_csr(3000, 3000, 200000, 8, positive=False, dups=True)
    rp, cl, vl = _ours(a, b)
    orp, ocl, ovl = osg.csr_spgemm(a.indptr, a.indices, a.data, b.indptr, b.indices, b.data)
    assert np.array_equal(rp, orp) and np.array_equal(cl, ocl)
    assert np.array_equal(vl.view(np.uint32), ovl.view(np.uint32))
    assert int(np.diff(rp).max()) > 1024


@pytest.mark.parametrize("case", ["merged runs", "many A entries", "unsorted B rows"])
def test_rows_longer_than_the_shared_sort_buffer(cuda, case):
    """Output rows of ~7,000 columns, beyond the 4,096-column shared-memory sort: merged from their
    ascending per-A-entry runs (B's rows ascending, <= 32 A entries per row), or sorted in global
    memory (an A row with more entries, or B rows out of order)."""
    n = 20000
    b = _rand_csr(n, n, n * 300, 11)
    if case == "unsorted B rows":   # the same entries, each row's order shuffled
        g = np.random.default_rng(12)
        rows = np.repeat(np.arange(n), np.diff(b.indptr))
        order = np.lexsort((g.random(b.nnz), rows))
        b = sp.csr_matrix((b.data[order], b.indices[order], b.indptr.copy()), shape=(n, n))
        assert not b.has_sorted_indices
    per_row = 40 if case == "many A entries" else 30
    g = np.random.default_rng(13)
    m = 12
    a_cols = np.stack([g.choice(n, per_row, replace=False) for _ in range(m)]).ravel()
    a = sp.csr_matrix(((g.random(m * per_row) + 0.1).astype(np.float32), a_cols,
                       np.arange(0, m * per_row + 1, per_row)), shape=(m, n))
    rp, cl, vl = _ours(a, b)
    assert int(np.diff(rp).min()) > 4096
    orp, ocl, ovl = osg.csr_spgemm(a.indptr, a.indices, a.data, b.indptr, b.indices, b.data)
    assert np.array_equal(rp, orp) and np.array_equal(cl, ocl)
    assert np.array_equal(vl.view(np.uint32), ovl.view(np.uint32))


def test_contract_checks(cuda):
    from neutrongt_b200.spgemm import csr_spgemm
    z = torch.zeros(1, dtype=torch.long, device="cuda")
    with pytest.raises(RuntimeError):
        csr_spgemm(z.cpu(), z, z.float(), z, z, z.float())
    with pytest.raises(ValueError):
        csr_spgemm(z.view(1, 1), z, z.float(), z, z, z.float())
    rp, cl, vl = csr_spgemm(z, z[:0], z[:0].float(), z, z[:0], z[:0].float())   # 0 x 0 product
    assert rp.tolist() == [0] and cl.numel() == 0 and vl.numel() == 0
