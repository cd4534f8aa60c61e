"""The CPU oracle, pinned against outputs of the reference's own code (tests/golden).

The fixtures were produced by `tests/golden/make_golden.py`, which imports the
reference modules unmodified (absent third-party packages replaced by the shims in
`tests/golden/reference_shims.py`).
"""
import pytest
import torch

from conftest import golden, rel_err
from oracle import attention as oatt
from oracle import ppr as oppr
from oracle import window as owin

ATTN_CASES = ["slim_d8", "gt_d16_clamp", "bias_h4", "empty"]


@pytest.mark.parametrize("case", ATTN_CASES)
def test_attention_forward_matches_reference(case):
    g = golden(f"attention_{case}.pt")
    x, ns, _, _ = oatt.sparse_attention_forward(g["q"].double(), g["k"].double(), g["v"].double(),
                                                g["edge_index"],
                                                None if g["attn_bias"] is None else g["attn_bias"].double())
    assert x.shape == g["x64"].shape
    assert ns.shape == g["node_scores64"].shape          # length = max(dst) + 1
    assert rel_err(x, g["x64"]) < 1e-12
    assert rel_err(ns, g["node_scores64"]) < 1e-12
    # fp32 oracle against the reference's own fp32 run
    x32, ns32, _, _ = oatt.sparse_attention_forward(g["q"], g["k"], g["v"], g["edge_index"], g["attn_bias"])
    assert rel_err(x32, g["x32"]) < 1e-5
    assert rel_err(ns32, g["node_scores32"]) < 1e-5


@pytest.mark.parametrize("case", ATTN_CASES)
def test_attention_backward_matches_reference_autograd(case):
    g = golden(f"attention_{case}.pt")
    bias = None if g["attn_bias"] is None else g["attn_bias"].double()
    dq, dk, dv, db = oatt.sparse_attention_backward(g["q"].double(), g["k"].double(), g["v"].double(),
                                                    g["edge_index"], g["dout"].double(), bias)
    s, H, D = g["s"], g["H"], g["D"]
    for mine, ref in ((dq, g["dq64"]), (dk, g["dk64"]), (dv, g["dv64"])):
        assert rel_err(mine.reshape(1, s, H, D), ref) < 1e-10
    if bias is not None:
        assert rel_err(db, g["dbias64"]) < 1e-10


def test_attention_forward_dispatch_shape():
    g = golden("attention_slim_d8.pt")
    assert g["forward_x"].shape == (1, g["s"], g["H"] * g["D"])
    assert torch.equal(g["forward_score"], g["node_scores32"])


def test_window_subgraph_matches_reference():
    g = golden("window_subgraph.pt")
    reranged, dups = owin.duplicate_first(g["windows"])
    for a, b in zip(reranged, g["reranged"]):
        assert torch.equal(a, b)
    for a, b in zip(dups, g["dup_nodes"]):
        assert torch.equal(a, b)
    for w, ref in zip(g["reranged"], g["sub_edge_index"]):
        assert torch.equal(owin.subgraph_from_csr(w, g["rowptr"], g["col"]), ref)


def test_stable_csr_orders_ties_by_edge_position():
    ei = torch.tensor([[3, 1, 2, 1, 0], [2, 2, 0, 2, 1]])
    rp, src, eid = owin.stable_csr(ei, 4, by="dst")
    assert rp.tolist() == [0, 1, 2, 5, 5]
    assert eid.tolist() == [2, 4, 0, 1, 3]
    assert src.tolist() == [2, 0, 3, 1, 1]


def _per_seed(ei, val):
    d = {}
    for s, c, v in zip(ei[0].tolist(), ei[1].tolist(), val.tolist()):
        d.setdefault(s, {})[c] = v
    return d


def _check_appnp_against_reference(ref_ei, ref_val, csr=None, edge_index=None, **params):
    stats = {}
    ei, val = oppr.personal_pagerank_appnp(edge_index, csr_data=csr, stats=stats, **params)
    mine, ref = _per_seed(ei, val), _per_seed(ref_ei, ref_val)
    assert set(mine) == set(ref)
    ties = set(stats["near_tie_seeds"].tolist())
    pinned = [s for s in ref if s not in ties]
    for s in pinned:  # no near-tie at any pruning boundary: sets equal, values to fp32 precision
        assert set(mine[s]) == set(ref[s]), s
        for c, v in ref[s].items():
            assert abs(mine[s][c] - v) <= 2e-6 * abs(v), (s, c)
    for s in ties:    # a near tie: torch.topk may keep either entry; sizes still agree
        assert len(mine[s]) == len(ref[s])
    return len(pinned)


def test_appnp_matches_reference():
    g = golden("appnp.pt")
    csr = {"rowptr": g["rowptr"], "col": g["col"]}
    pinned = 0
    for name, case in g["cases"].items():
        pinned += _check_appnp_against_reference(case["edge_index"], case["values"], csr=csr, **case["params"])
    d = g["dense"]
    for name, case in d["cases"].items():
        pinned += _check_appnp_against_reference(case["edge_index"], case["values"],
                                                 csr={"rowptr": d["rowptr"], "col": d["col"]}, **case["params"])
    c = g["edge_index_case"]
    pinned += _check_appnp_against_reference(c["edge_index"], c["values"], edge_index=c["edge_index_in"],
                                             **c["params"])
    assert pinned >= 500


def test_appnp_unpruned_matches_reference_everywhere():
    g = golden("appnp.pt")
    case = g["cases"]["unpruned"]
    stats = {}
    ei, val = oppr.personal_pagerank_appnp(None, csr_data={"rowptr": g["rowptr"], "col": g["col"]},
                                           stats=stats, **case["params"])
    mine, ref = _per_seed(ei, val), _per_seed(case["edge_index"], case["values"])
    assert len(stats["near_tie_seeds"]) == 0
    for s in ref:
        assert set(mine[s]) == set(ref[s])


def test_appnp_isolated_seed_keeps_teleport_only():
    rowptr = torch.tensor([0, 1, 2, 2])     # 0 <-> 1, node 2 isolated
    col = torch.tensor([1, 0])
    ei, val = oppr.personal_pagerank_appnp(None, 0.15, topk=4, num_iterations=3,
                                           csr_data={"rowptr": rowptr, "col": col})
    seed2 = ei[0] == 2
    assert ei[1][seed2].tolist() == [2]
    assert val[seed2].tolist() == [pytest.approx(0.15)]


def test_appnp_source_range_and_empty():
    rowptr = torch.tensor([0, 1, 2])
    col = torch.tensor([1, 0])
    ei, val = oppr.personal_pagerank_appnp(None, 0.5, topk=2, csr_data={"rowptr": rowptr, "col": col},
                                           source_start=1, source_end=1)
    assert ei.shape == (2, 0) and val.numel() == 0


# ---------------- dense full attention (oracle/dense.py) against the reference's outputs ----------------

@pytest.mark.parametrize("case", ["d24_h4", "d16_h2", "d8_h3", "d64_h2", "d40_h1", "bias_d16",
                                  "bias_pruning_mask_d24", "mask_d64"])
def test_dense_oracle_matches_reference(case):
    from oracle import dense as odense
    c = golden("dense_attention.pt")[case]
    q, k, v, g = (c[n].double().requires_grad_(n != "dout") for n in ("q", "k", "v", "dout"))
    b = c["attn_bias"].double().requires_grad_(True) if c["attn_bias"] is not None else None
    pm = c["pruning_mask"].double().requires_grad_(True) if c["pruning_mask"] is not None else None
    x, ns = odense.full_attention(k, q, v, b, c["mask"], pm)
    (x * g).sum().backward()
    tol = 1e-6     # the fixture holds fp64 results rounded to fp32
    assert rel_err(x, c["x"]) < tol and rel_err(ns, c["node_scores"]) < tol
    assert rel_err(q.grad, c["dq"]) < tol and rel_err(k.grad, c["dk"]) < tol and rel_err(v.grad, c["dv"]) < tol
    if b is not None:
        assert rel_err(b.grad, c["dbias"]) < tol
    if pm is not None:
        assert rel_err(pm.grad, c["dpruning"]) < tol
    if c["attn_bias"] is None and c["mask"] is None:      # the chunked form (no bias / mask)
        out, ns2, dq, dk, dv = odense.full_attention_chunked(q[0].detach(), k[0].detach(), v[0].detach(),
                                                             g[0].detach(), rows=37)
        assert rel_err(out, c["x"][0]) < tol and rel_err(ns2, c["node_scores"]) < tol
        assert rel_err(dq, c["dq"][0]) < tol and rel_err(dk, c["dk"][0]) < tol and rel_err(dv, c["dv"][0]) < tol


def test_dense_reference_dispatch_matches_full_attention():
    """`CoreAttention.forward(attn_type="full")` reshapes the full_attention output to [b, s, H*D]."""
    c = golden("dense_attention.pt")["d24_h4"]
    assert c["forward_x"].shape == (1, c["s"], c["H"] * c["D"])
    assert rel_err(c["forward_x"].reshape(c["x"].shape), c["x"]) < 1e-5
    assert rel_err(c["forward_score"], c["node_scores"]) < 1e-5


# ---------------- push PPR (oracle/push_oracle.c): the published method and its guarantee ----------------

def _push_python(rowptr, col, alpha, eps, seed):
    """The push method written with Python dicts and a list stack, line by line as the published
    algorithm states it (PPRGo variant of Andersen, Chung & Lang); returns p in insertion order."""
    deg = [rowptr[i + 1] - rowptr[i] for i in range(len(rowptr) - 1)]
    p, r, q = {seed: 0.0}, {seed: alpha}, [seed]
    while q:
        u = q.pop()
        res = r.get(u, 0.0)
        p[u] = p[u] + res if u in p else res
        r[u] = 0.0
        for v in col[rowptr[u]:rowptr[u + 1]]:
            val = (1 - alpha) * res / deg[u]
            r[v] = r[v] + val if v in r else val
            if r[v] >= alpha * eps * deg[v] and v not in q:
                q.append(v)
    return list(p.items())


@pytest.mark.parametrize("alpha,eps", [(0.15, 1e-3), (0.85, 1e-4), (0.2, 1e-5)])
def test_push_oracle_matches_the_python_statement(alpha, eps):
    import numpy as np
    from neutrongt_b200 import synthetic
    rowptr, col = synthetic.chung_lu_graph(120, 500, seed=17)
    rp, cl = rowptr.tolist(), col.tolist()
    big = 10 ** 6
    ei, v = oppr.personal_pagerank_push(None, alpha, topk=big, eps=eps, csr_data={"rowptr": rowptr, "col": col},
                                        return_fp64=True)
    for seed in (0, 1, 7, 63, 119):
        want = _push_python(rp, cl, alpha, eps, seed)
        sel = (ei[0] == seed).nonzero().flatten()
        got = list(zip(ei[1, sel].tolist(), v[sel].tolist()))
        assert got == want                     # same entries, same insertion order, same bits
    # top-k: (value desc, node asc) when a seed has more entries than topk
    ei5, v5 = oppr.personal_pagerank_push(None, alpha, topk=5, eps=eps, csr_data={"rowptr": rowptr, "col": col},
                                          return_fp64=True)
    for seed in (0, 7):
        want = sorted(_push_python(rp, cl, alpha, eps, seed), key=lambda t: (-t[1], t[0]))[:5]
        sel = (ei5[0] == seed).nonzero().flatten()
        assert list(zip(ei5[1, sel].tolist(), v5[sel].tolist())) == want
    assert np.all(np.diff(ei5[0].numpy()) >= 0)


@pytest.mark.parametrize("n,m,alpha,eps", [(200, 900, 0.15, 1e-4), (150, 2000, 0.85, 1e-3), (400, 1200, 0.3, 1e-5)])
def test_push_oracle_meets_the_error_guarantee(n, m, alpha, eps):
    """Undirected graph: 0 <= pi_s(v) - p_s(v) < eps * deg(v) for every seed s and node v, with pi_s the
    exact PPR (teleport alpha) from a dense solve."""
    import numpy as np
    from neutrongt_b200 import synthetic
    rowptr, col = synthetic.chung_lu_graph(n, m, seed=n + m)
    ei, v = oppr.personal_pagerank_push(None, alpha, topk=n, eps=eps, csr_data={"rowptr": rowptr, "col": col},
                                        return_fp64=True, nthreads=4)
    A = np.zeros((n, n))
    rp, cl = rowptr.numpy(), col.numpy()
    for u in range(n):
        np.add.at(A[u], cl[rp[u]:rp[u + 1]], 1.0)
    assert np.array_equal(A, A.T)
    deg = A.sum(1)
    P = A / np.maximum(deg, 1.0)[:, None]
    pi = alpha * np.linalg.inv(np.eye(n) - (1 - alpha) * P)
    got = np.zeros((n, n))
    got[ei[0].numpy(), ei[1].numpy()] = v.numpy()
    diff = pi - got
    assert diff.min() > -1e-12
    assert (diff < eps * deg[None, :] + 1e-12).all()


# ---------------- sparse product (oracle/spgemm.py) against SciPy's row-wise product ----------------

def _rand_csr(rows, cols, nnz, seed, positive=True):
    import numpy as np
    import scipy.sparse as sp
    g = np.random.default_rng(seed)
    r = g.integers(0, rows, nnz)
    c = g.integers(0, cols, nnz)
    v = (g.random(nnz) + 0.1 if positive else g.standard_normal(nnz)).astype(np.float32)
    mat = sp.csr_matrix((v, (r, c)), shape=(rows, cols))
    mat.sum_duplicates()
    mat.sort_indices()
    return mat


@pytest.mark.parametrize("m,n,nnz_a,nnz_b,seed", [(40, 60, 200, 500, 1), (1, 30, 5, 100, 2), (25, 25, 0, 100, 3),
                                                  (80, 50, 600, 900, 4)])
def test_spgemm_oracle_matches_scipy(m, n, nnz_a, nnz_b, seed):
    import numpy as np
    from oracle import spgemm as osg
    a = _rand_csr(m, n, nnz_a, seed)
    b = _rand_csr(n, n, nnz_b, seed + 100)
    c = (a @ b).tocsr()
    c.sort_indices()
    rp, cl, vl = osg.csr_spgemm(a.indptr, a.indices, a.data, b.indptr, b.indices, b.data)
    assert np.array_equal(rp, c.indptr) and np.array_equal(cl, c.indices)
    assert np.array_equal(vl.view(np.uint32), c.data.astype(np.float32).view(np.uint32))   # bit for bit


def test_spgemm_oracle_keeps_cancelled_entries():
    """A row whose two products cancel: SciPy drops the entry, cuSPARSE (and this) keeps it as 0."""
    from oracle import spgemm as osg
    rp, cl, vl = osg.csr_spgemm([0, 2], [0, 1], [1.0, -1.0], [0, 1, 2], [0, 0], [2.0, 2.0])
    assert rp.tolist() == [0, 1] and cl.tolist() == [0] and vl.tolist() == [0.0]
