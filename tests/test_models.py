"""Model mirrors: the reference's state_dicts load unchanged (CPU), and one training step
reproduces the reference's loss, outputs and gradients (GPU)."""
from types import SimpleNamespace

import pytest
import torch

from conftest import golden, rel_err


def _build(kind, cfg):
    from neutrongt_b200.models import GT_SW, Graphormer
    cls = GT_SW if kind == "gt_sw" else Graphormer
    return cls(args=SimpleNamespace(struct_enc="False"), **cfg)


@pytest.mark.parametrize("kind", ["gt_sw", "graphormer"])
def test_reference_state_dict_loads_strictly(kind):
    g = golden(f"{kind}_step.pt")
    model = _build(kind, g["config"])
    model.load_state_dict(g["state_dict"], strict=True)
    assert sorted(model.state_dict()) == sorted(g["state_dict"])


@pytest.mark.gpu
@pytest.mark.parametrize("kind", ["gt_sw", "graphormer"])
def test_training_step_matches_reference(cuda, kind):
    import torch.nn.functional as F
    g = golden(f"{kind}_step.pt")
    model = _build(kind, g["config"]).cuda()
    model.load_state_dict(g["state_dict"], strict=True)
    model.train()
    out, _, scores, cache = model(g["x"].cuda(), None, g["edge_index"].cuda(), None, None, None, None,
                                  attn_type="sparse")
    loss = F.nll_loss(out, g["y"].cuda(), reduction="none")[g["train_mask"].cuda()].mean()
    loss.backward()
    assert cache is None
    assert abs(float(loss) - g["loss"]) < 1e-5 * max(1.0, abs(g["loss"]))
    assert rel_err(out, g["out"]) < 1e-5
    for mine, ref in zip(scores, g["scores"]):
        assert rel_err(mine, ref) < 1e-5
    params = dict(model.named_parameters())
    for name, ref in g["grads"].items():
        assert rel_err(params[name].grad, ref) < 1e-4, name


@pytest.mark.gpu
def test_graphed_epoch_matches_eager_epoch(cuda):
    """Two epochs replayed from CUDA graphs give the eager loop's losses and parameters."""
    import copy
    from neutrongt_b200 import synthetic
    from neutrongt_b200.train import FlatGradients, GraphedWindowTrainer, build_window_state, train_epoch
    n = 3000
    rowptr, col = synthetic.chung_lu_graph(n, 12000, seed=4)
    feature = synthetic.node_features(n, 16, seed=5).cuda()
    y = synthetic.node_labels(n, 5, seed=6).cuda()
    split = synthetic.split_idx(n, seed=7)
    parts = synthetic.random_partitions(n, 4, seed=8)
    ws = build_window_state(rowptr, col, parts, 0, 1, feature, "cuda", split)
    g = golden("gt_sw_step.pt")
    cfg = dict(g["config"])
    base = _build("gt_sw", cfg).cuda()
    eager, graphed = copy.deepcopy(base), copy.deepcopy(base)
    args = SimpleNamespace(use_cache=1, attn_type="sparse")
    opt_e = torch.optim.AdamW(eager.parameters(), lr=1e-3, weight_decay=0.01, capturable=True)
    grads_e = FlatGradients(eager)
    sched_e = torch.optim.lr_scheduler.LambdaLR(opt_e, lambda e: 1.0)
    opt_g = torch.optim.AdamW(graphed.parameters(), lr=1e-3, weight_decay=0.01, capturable=True)
    trainer = GraphedWindowTrainer(args, graphed, ws, feature, y, opt_g, 1, "cuda", split_idx=split)
    # the capture warm-up took one eager step per window: give the eager copy the same start
    for _ in range(1):
        train_epoch(args, eager, ws.local_partition_ids, ws.local_partitions, feature, y, opt_e, sched_e, 1, split,
                    "cuda", 0, ws, grads=grads_e)
    for _ in range(2):
        le, _, _, _ = train_epoch(args, eager, ws.local_partition_ids, ws.local_partitions, feature, y, opt_e,
                                  sched_e, 1, split, "cuda", 0, ws, grads=grads_e)
        lg, scores, _ = trainer.run_epoch()
        assert abs(le - lg) < 1e-4 * max(1.0, abs(le))
    for (name, pe), pg in zip(eager.named_parameters(), graphed.parameters()):
        assert rel_err(pg, pe) < 1e-4, name
    assert sorted(scores) == ws.local_partition_ids
