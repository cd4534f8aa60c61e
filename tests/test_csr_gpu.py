"""Window CSR construction on the GPU: bit-exact against the reference fixtures and the oracle."""
import pytest
import torch

from conftest import golden
from oracle import window as owin

pytestmark = pytest.mark.gpu


def _check_edge_csr(ei, n):
    from neutrongt_b200.edge_csr import build_edge_csr
    csr = build_edge_csr(ei.cuda(), n)
    rp, src, eid = owin.stable_csr(ei, n, by="dst")
    assert torch.equal(csr.dst_rowptr.cpu().long(), rp)
    assert torch.equal(csr.dst_src.cpu().long(), src)
    rp2, dst2, eid2 = owin.stable_csr(ei, n, by="src")
    assert torch.equal(csr.src_rowptr.cpu().long(), rp2)
    assert torch.equal(csr.src_dst.cpu().long(), dst2)
    # src-major slot i and dst-major slot src_to_dst_slot[i] are the same edge
    inv = torch.empty_like(eid)
    inv[eid] = torch.arange(eid.numel())
    assert torch.equal(csr.src_to_dst_slot.cpu().long(), inv[eid2])
    assert csr.max_dst == (int(ei[1].max()) if ei.shape[1] else -1)


@pytest.mark.parametrize("n,E,seed", [(1, 3, 0), (50, 0, 1), (200, 3000, 2), (5000, 70000, 3),
                                      (70000, 300000, 4), (300000, 1000000, 5)])
def test_edge_csr_matches_oracle(cuda, n, E, seed):
    g = torch.Generator().manual_seed(seed)
    ei = torch.randint(0, n, (2, E), generator=g)
    if E > 10:
        ei[:, 1:6] = ei[:, 0:1]          # repeated edges keep their order
        ei[1, 100 % E:] = torch.where(ei[1, 100 % E:] % 7 == 0, 0, ei[1, 100 % E:])  # a heavy row
    _check_edge_csr(ei, n)


def test_edge_csr_source_major_input(cuda):
    from neutrongt_b200 import synthetic
    rowptr, col = synthetic.chung_lu_graph(3000, 20000, seed=4)
    _check_edge_csr(synthetic.edge_index_from_src_csr(rowptr, col), 3000)


def test_edge_csr_rejects_out_of_range(cuda):
    from neutrongt_b200.edge_csr import build_edge_csr
    with pytest.raises(IndexError):
        build_edge_csr(torch.tensor([[0, 1], [2, -1]], device="cuda"), 3)


def test_window_subgraph_matches_reference(cuda):
    from neutrongt_b200 import compute_local_duplicate_nodes, subgraph_from_csr
    g = golden("window_subgraph.pt")
    reranged, dups = compute_local_duplicate_nodes(g["windows"])
    for a, b in zip(reranged, g["reranged"]):
        assert torch.equal(a, b)
    for a, b in zip(dups, g["dup_nodes"]):
        assert torch.equal(a, b)
    for w, ref in zip(g["reranged"], g["sub_edge_index"]):
        out = subgraph_from_csr(w, g["rowptr"].cuda(), g["col"].cuda())
        assert torch.equal(out.cpu(), ref)


def test_window_subgraph_large_matches_oracle(cuda):
    from neutrongt_b200 import subgraph_from_csr, synthetic
    rowptr, col = synthetic.chung_lu_graph(169343, 1166243, seed=0)
    parts = synthetic.random_partitions(169343, 16, seed=0)
    rp_d, col_d = rowptr.cuda(), col.cuda()
    for p in parts[:3]:
        w = p[torch.randperm(p.numel(), generator=torch.Generator().manual_seed(1))]  # arbitrary window order
        out = subgraph_from_csr(w, rp_d, col_d)
        assert torch.equal(out.cpu(), owin.subgraph_from_csr(w, rowptr, col))


def test_window_subgraph_rejects_repeated_nodes(cuda):
    from neutrongt_b200 import subgraph_from_csr
    rowptr = torch.tensor([0, 1, 2, 2]).cuda()
    col = torch.tensor([1, 0]).cuda()
    with pytest.raises(ValueError):
        subgraph_from_csr(torch.tensor([0, 1, 0]), rowptr, col)
