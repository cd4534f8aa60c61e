"""Window construction on the device (csrc/windows.cu) against the reference fixtures and the
CPU oracle: bit-exact (integer weights, node ids and orders)."""
import numpy as np
import pytest
import torch

from conftest import golden
from oracle import window as ow

pytestmark = pytest.mark.gpu


def _rows(xadj, adjncy, eweights):
    xadj, adjncy, eweights = (np.asarray(t.cpu() if torch.is_tensor(t) else t) for t in (xadj, adjncy, eweights))
    return [sorted(zip(adjncy[xadj[r]:xadj[r + 1]].tolist(), eweights[xadj[r]:xadj[r + 1]].tolist()))
            for r in range(len(xadj) - 1)]


def _ppr_like(n, k, seed):
    g = torch.Generator().manual_seed(seed)
    src = torch.arange(n).repeat_interleave(k)
    dst = torch.randint(0, n, (n * k,), generator=g)
    vals = (torch.rand(n * k, generator=g) ** 6 * 0.3).to(torch.float32)
    mirror = torch.randperm(n * k, generator=g)[: n * k // 4]
    ei = torch.stack([torch.cat([src, dst[mirror]]), torch.cat([dst, src[mirror]])])
    return ei, torch.cat([vals, (torch.rand(mirror.numel(), generator=g) * 0.01).to(torch.float32)])


def test_ppr_adjacency_reference_and_oracle(cuda):
    from neutrongt_b200.window import build_adj_format
    g = golden("window_build.pt")
    csr, ew, _ = build_adj_format((g["ppr_edge_index"], g["ppr_val"]))
    assert torch.equal(csr.adj_starts.cpu(), g["xadj"])
    assert _rows(csr.adj_starts, csr.adjacent, ew) == _rows(g["xadj"], g["adjncy"], g["eweights"])
    x, a, e = ow.ppr_adjacency(g["ppr_edge_index"].numpy(), g["ppr_val"].numpy())
    assert np.array_equal(csr.adjacent.cpu().numpy(), a) and np.array_equal(ew.cpu().numpy(), e)


@pytest.mark.parametrize("n,k,seed", [(20000, 8, 1), (3, 1, 2), (70000, 3, 3)])
def test_ppr_adjacency_random_vs_oracle(cuda, n, k, seed):
    from neutrongt_b200.window import build_adj_format
    ei, val = _ppr_like(n, k, seed)
    csr, ew, _ = build_adj_format((ei, val))
    x, a, e = ow.ppr_adjacency(ei.numpy(), val.numpy())
    assert np.array_equal(csr.adj_starts.cpu().numpy(), x)
    assert np.array_equal(csr.adjacent.cpu().numpy(), a)
    assert np.array_equal(ew.cpu().numpy(), e)


def test_ppr_adjacency_empty(cuda):
    from neutrongt_b200.window import build_adj_format
    csr, ew, extra = build_adj_format((torch.empty(2, 0, dtype=torch.long), torch.empty(0)))
    assert csr.adj_starts.tolist() == [0] and csr.adjacent.numel() == 0 and ew.numel() == 0 and extra is None


def test_halo_merge_reference(cuda):
    from neutrongt_b200.window import CSRAdjacency, merge_related_nodes
    g = golden("window_build.pt")
    csr = CSRAdjacency(g["xadj"], g["adjncy"])
    for pct, halos in g["halos"].items():
        for win, ref in zip(g["windows"], halos):
            assert torch.equal(merge_related_nodes(win, csr, g["eweights"], pct).cpu(), ref)


@pytest.mark.parametrize("pct", [0, 1, 13, 50, 100])
def test_halo_merge_random_vs_oracle(cuda, pct):
    from neutrongt_b200.window import build_adj_format, merge_related_nodes
    ei, val = _ppr_like(30000, 6, seed=pct + 7)
    csr, ew, _ = build_adj_format((ei, val))
    x, a, e = (t.cpu().numpy() for t in (csr.adj_starts, csr.adjacent, ew))
    perm = torch.randperm(30000, generator=torch.Generator().manual_seed(pct))
    for win in (perm[:2000], torch.sort(perm[2000:5000]).values, perm[5000:5001]):
        ours = merge_related_nodes(win, csr, ew, pct).cpu()
        assert torch.equal(ours, ow.merge_related_nodes(win, x, a, e, pct))


def test_halo_merge_isolated_window(cuda):
    from neutrongt_b200.window import CSRAdjacency, merge_related_nodes
    csr = CSRAdjacency(torch.tensor([0, 0, 1, 2], dtype=torch.int32), torch.tensor([2, 1], dtype=torch.int32))
    assert merge_related_nodes(torch.tensor([0]), csr, torch.tensor([5, 5]), 100).tolist() == [0]
    assert merge_related_nodes(torch.tensor([1, 2]), csr, torch.tensor([5, 5]), 100).tolist() == [1, 2]
    assert merge_related_nodes(torch.tensor([1]), csr, torch.tensor([5, 5]), 100).tolist() == [1, 2]
    assert merge_related_nodes(torch.tensor([], dtype=torch.long), csr, torch.tensor([5, 5]), 100).numel() == 0


def test_duplicate_rerange_reference_and_random(cuda):
    from neutrongt_b200.window import compute_local_duplicate_nodes, find_duplicate_nodes_and_rerange
    g = golden("window_build.pt")
    groups, dups = find_duplicate_nodes_and_rerange(g["child_partitions"])
    for ga, gb in zip(groups, g["reranged"]):
        for a, b in zip(ga, gb):
            assert torch.equal(a, b)
    assert all(torch.equal(a, b) for a, b in zip(dups, g["dup_nodes"]))
    gen = torch.Generator().manual_seed(5)
    parts = [torch.randperm(50000, generator=gen)[: int(s)] for s in (9000, 0, 12000, 1, 7000)]
    ours = compute_local_duplicate_nodes(parts)
    ref = ow.duplicate_first(parts)
    for a, b in zip(ours[0] + ours[1], ref[0] + ref[1]):
        assert torch.equal(a, b)


@pytest.mark.parametrize("n,p,seed", [(5000, 0.01, 1), (50000, 0.002, 2), (300, 1.0, 3), (300, 0.0, 4)])
def test_isolated_connections_match_oracle(cuda, n, p, seed):
    from neutrongt_b200.window import add_isolated_connections
    g = torch.Generator().manual_seed(seed)
    appear = torch.randperm(n, generator=g)[: n // 3]
    ppr = torch.stack([appear[: n // 6], appear[n // 6: 2 * (n // 6)]])
    graph = torch.stack([appear[:: 2][:50], appear[1:: 2][:50]])
    vals = torch.rand(ppr.shape[1], generator=g)
    ei, v = add_isolated_connections((ppr, vals), graph, n, connect_prob=p, ppr_fill_value=0.001, seed=seed)
    ref = ow.isolated_connections(ppr.numpy(), graph.numpy(), n, p, seed)
    m = ppr.shape[1]
    assert torch.equal(ei[:, :m].cpu(), ppr) and torch.equal(v[:m].cpu(), vals)
    assert np.array_equal(ei[:, m:].cpu().numpy(), ref)
    assert torch.all(v[m:] == torch.tensor(0.001)) and v.dtype == vals.dtype


def test_isolated_connections_none_isolated(cuda):
    from neutrongt_b200.window import add_isolated_connections
    ppr = torch.tensor([[0, 1], [1, 2]])
    vals = torch.tensor([0.5, 0.25])
    ei, v = add_isolated_connections((ppr, vals), torch.zeros((2, 0), dtype=torch.long), 3)
    assert torch.equal(ei.cpu(), ppr) and torch.equal(v.cpu(), vals)
