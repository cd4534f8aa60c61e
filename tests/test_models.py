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
