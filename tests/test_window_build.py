"""Window construction oracle (PPR adjacency, halo merge, duplicate-first order) against the
reference's own outputs (tests/golden/window_build.pt, made by tests/golden/make_golden.py)."""
import numpy as np
import torch

from conftest import golden
from oracle import window as ow


def _rows(xadj, adjncy, eweights):
    xadj, adjncy, eweights = (np.asarray(t) for t in (xadj, adjncy, eweights))
    return [sorted(zip(adjncy[xadj[r]:xadj[r + 1]].tolist(), eweights[xadj[r]:xadj[r + 1]].tolist()))
            for r in range(len(xadj) - 1)]


def test_ppr_adjacency_matches_reference():
    g = golden("window_build.pt")
    x, a, e = ow.ppr_adjacency(g["ppr_edge_index"].numpy(), g["ppr_val"].numpy())
    assert np.array_equal(x, g["xadj"].numpy())
    # the reference orders a row with a non-stable argsort: compare each row as a multiset
    assert _rows(x, a, e) == _rows(g["xadj"], g["adjncy"], g["eweights"])


def test_halo_merge_matches_reference():
    g = golden("window_build.pt")
    for pct, halos in g["halos"].items():
        for win, ref in zip(g["windows"], halos):
            assert torch.equal(ow.merge_related_nodes(win, g["xadj"], g["adjncy"], g["eweights"], pct), ref)


def test_duplicate_rerange_matches_reference():
    g = golden("window_build.pt")
    groups, dups = ow.duplicate_rerange_nested(g["child_partitions"])
    for ga, gb in zip(groups, g["reranged"]):
        for a, b in zip(ga, gb):
            assert torch.equal(a, b)
    assert len(dups) == len(g["dup_nodes"])
    for a, b in zip(dups, g["dup_nodes"]):
        assert torch.equal(a, b)


def test_oracle_edge_cases():
    x, a, e = ow.ppr_adjacency(np.zeros((2, 0), np.int64), np.zeros(0, np.float32))
    assert x.tolist() == [0] and a.size == 0
    # ties broken by first encounter; percent rounds down
    ei = np.array([[0, 0, 0], [1, 2, 3]])
    x, a, e = ow.ppr_adjacency(ei, np.array([0.0005, 0.0002, 0.004], np.float32))
    assert e.tolist()[:3] == [1, 1, 4]
    assert ow.merge_related_nodes([0], x, a, e, 34).tolist() == [0, 3]     # 3 * 34 // 100 = 1
    assert ow.merge_related_nodes([0], x, a, e, 67).tolist() == [0, 1, 3]  # then node 1 (seen first)
    assert ow.merge_related_nodes([0, 1, 2, 3], x, a, e, 100).tolist() == [0, 1, 2, 3]


def test_isolated_connections_oracle_properties():
    # SplitMix64 published first outputs for state 0 and 1 (Steele, Lea & Flood 2014)
    assert ow.splitmix64(np.array([0, 1], np.uint64)).tolist() == [0xE220A8397B1DCDAF, 0x910A2DEC89025CC1]
    ppr = np.array([[0, 1, 5], [1, 2, 7]])
    graph = np.array([[9], [10]])
    e = ow.isolated_connections(ppr, graph, 3000, 0.02, seed=3)
    iso = np.setdiff1d(np.arange(3000), [0, 1, 2, 5, 7, 9, 10])
    assert np.all(np.isin(e[0], iso)) and np.all(np.isin(e[1], [0, 1, 2, 5, 7, 9, 10]))
    order = e[0] * 3000 + e[1]
    assert np.all(np.diff(order) > 0)                              # row-major, no repeats
    expect = iso.size * 7 * 0.02
    assert abs(e.shape[1] - expect) < 5 * np.sqrt(expect)          # Bernoulli(p) per pair
    assert ow.isolated_connections(ppr, graph, 11, 0.5, seed=3).shape[1] > 0
    assert ow.isolated_connections(np.array([[0], [1]]), np.zeros((2, 0), np.int64), 2, 1.0, 0).shape[1] == 0
