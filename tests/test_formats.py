"""The reference's on-disk formats: CSR file, checkpoint (CPU) and preprocess cache (GPU)."""
import os
from types import SimpleNamespace

import pytest
import torch

from conftest import golden


def test_edge_csr_file(tmp_path):
    from neutrongt_b200.formats import load_optional_edge_csr
    assert load_optional_edge_csr(str(tmp_path), "none") is None
    d = tmp_path / "ds"
    d.mkdir()
    torch.save({"rowptr": torch.tensor([0, 2, 3]), "col": torch.tensor([1, 0, 0])}, d / "edge_index_csr.pt")
    got = load_optional_edge_csr(str(tmp_path), "ds")
    assert got["rowptr"].tolist() == [0, 2, 3] and got["col"].tolist() == [1, 0, 0]
    for bad, exc in (({"rowptr": torch.tensor([0, 2])}, KeyError),
                     ({"rowptr": torch.tensor([1, 2]), "col": torch.tensor([0, 1])}, ValueError),
                     ({"rowptr": torch.tensor([0, 3]), "col": torch.tensor([0, 1])}, ValueError),
                     ({"rowptr": torch.zeros(0, dtype=torch.long), "col": torch.zeros(0, dtype=torch.long)}, ValueError)):
        torch.save(bad, d / "edge_index_csr.pt")
        with pytest.raises(exc):
            load_optional_edge_csr(str(tmp_path), "ds")


def _small_gt():
    from neutrongt_b200.models import GT_SW
    torch.manual_seed(0)
    return GT_SW(n_layers=1, num_heads=2, input_dim=8, hidden_dim=8, output_dim=3, attn_bias_dim=1, dropout_rate=0.0,
                 input_dropout_rate=0.0, attention_dropout_rate=0.0, ffn_dim=8, num_global_node=1,
                 args=SimpleNamespace(struct_enc="False"), num_in_degree=0, num_out_degree=0, num_spatial=7,
                 num_edges=512, max_dist=5, edge_dim=64)


def test_checkpoint_round_trip(tmp_path):
    from neutrongt_b200.formats import build_checkpoint_payload, load_checkpoint
    m = _small_gt()
    opt = torch.optim.AdamW(m.parameters(), lr=1e-3)
    for p in m.parameters():
        p.grad = torch.ones_like(p)
    opt.step()
    sched = torch.optim.lr_scheduler.LambdaLR(opt, lambda e: 0.5)
    run_args = SimpleNamespace(dataset="ogbn-arxiv", model="gt", n_layers=1, hidden_dim=8, num_heads=2,
                               attn_type="sparse", n_parts=16, related_nodes_topk_rate=5, ppr_topk=8, seed=0)
    payload = build_checkpoint_payload(run_args, m, opt, sched, 4, [1.0, 0.5], 2, 0.7, 0.6)
    assert payload["args_snapshot"] == {"dataset": "ogbn-arxiv", "model": "gt", "n_layers": 1, "hidden_dim": 8,
                                        "num_heads": 2, "attn_type": "sparse", "n_parts": 16,
                                        "related_nodes_topk_rate": 5, "ppr_topk": 8}
    assert set(payload) == {"epoch", "start_epoch", "model_state_dict", "optimizer_state_dict",
                            "lr_scheduler_state_dict", "args_snapshot", "loss_mean_list", "window_state_version",
                            "best_val", "best_test"}
    path = tmp_path / "last.pt"
    torch.save(payload, path)
    m2 = _small_gt()
    opt2 = torch.optim.AdamW(m2.parameters(), lr=1e-3)
    sched2 = torch.optim.lr_scheduler.LambdaLR(opt2, lambda e: 0.5)
    info = load_checkpoint(str(path), m2, opt2, sched2, args=run_args)
    assert info["start_epoch"] == 5 and info["loss_mean_list"] == [1.0, 0.5] and info["best_test"] == 0.6
    for a, b in zip(m.state_dict().values(), m2.state_dict().values()):
        assert torch.equal(a, b)
    assert opt2.state_dict()["state"][0]["step"] == opt.state_dict()["state"][0]["step"]


def test_checkpoint_rejects_incompatible_run_arguments():
    """A resume with other model arguments raises before any state is loaded
    (`checkpoint.py:77-90`); keys the snapshot does not hold are skipped."""
    from neutrongt_b200.formats import load_checkpoint
    m = _small_gt()
    before = {k: v.clone() for k, v in m.state_dict().items()}
    other = _small_gt()
    with torch.no_grad():
        for p in other.parameters():
            p.add_(1.0)
    ck = {"model_state_dict": other.state_dict(), "args_snapshot": {"model": "gt", "hidden_dim": 8, "n_parts": 16}}
    with pytest.raises(ValueError, match="hidden_dim: current=16, checkpoint=8"):
        load_checkpoint(ck, m, args=SimpleNamespace(model="gt", hidden_dim=16, n_parts=16))
    for k, v in m.state_dict().items():
        assert torch.equal(v, before[k])
    load_checkpoint(ck, m, args={"model": "gt", "hidden_dim": 8, "n_parts": 16, "dataset": "x"})


def test_reference_state_dict_loads_through_checkpoint(tmp_path):
    """A checkpoint holding the reference GT_SW's state_dict (from the golden step fixture)."""
    from neutrongt_b200.formats import load_checkpoint
    from neutrongt_b200.models import GT_SW
    g = golden("gt_sw_step.pt")
    cfg = dict(g["config"])
    cfg["args"] = SimpleNamespace(struct_enc="False")
    model = GT_SW(**cfg)
    info = load_checkpoint({"model_state_dict": g["state_dict"], "epoch": 0}, model)
    assert info["start_epoch"] == 1


@pytest.mark.gpu
def test_preprocess_cache_to_window_state(cuda, tmp_path):
    from neutrongt_b200 import synthetic
    from neutrongt_b200.formats import window_state_from_preprocess_cache
    from neutrongt_b200.train import build_window_state
    n = 2000
    rowptr, col = synthetic.chung_lu_graph(n, 8000, seed=3)
    parts = synthetic.random_partitions(n, 6, seed=1)
    payload = {"cache_version": 1, "num_nodes": n, "graph_csr_data": {"rowptr": rowptr, "col": col},
               "sorted_ppr_matrix": None, "graph_edge_index": None,
               "wm": {"partitioned_results": parts, "sub_edge_index_for_partition_results": [],
                      "dup_nodes_per_partition": []}}
    torch.save(payload, tmp_path / "preprocess_x.pt")
    feat = torch.randn(n, 4, device="cuda")
    a = window_state_from_preprocess_cache(str(tmp_path / "preprocess_x.pt"), 1, 2, feat, "cuda")
    b = build_window_state(rowptr, col, parts, 1, 2, feat, "cuda")
    assert a.local_partition_ids == b.local_partition_ids == [1, 3, 5]
    for x, y in zip(a.local_sub_edge_index_for_partition_results, b.local_sub_edge_index_for_partition_results):
        assert torch.equal(x, y)
