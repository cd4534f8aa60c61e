"""The reference's CPU-runnable case, end to end (the smallest benchmark configuration).

Synthetic power-law graph (10,000 nodes, mean degree 8), APPNP PPR (alpha 0.15, 20 iterations,
top-8) over every seed, 16 contiguous random windows, and one training epoch of GPH_Slim
(4 layers, hidden 64, ffn 64, 8 heads) with sparse attention.  GPU results against the CPU
oracle: PPR and window edge lists bit-exact; the epoch (fp32 on the GPU) against the same model
in fp64 on the CPU with the oracle's attention, per-window losses and the epoch loss within 1e-3.
"""
import copy
from types import SimpleNamespace

import pytest
import torch
import torch.nn.functional as F

from oracle import attention as oatt
from oracle import ppr as oppr
from oracle import window as owin

pytestmark = pytest.mark.gpu

N = 10000


@pytest.fixture(scope="module")
def graph():
    from neutrongt_b200 import synthetic
    return synthetic.chung_lu_graph(N, 40000, seed=0)


def test_ppr_all_seeds_bit_exact(cuda, graph):
    from neutrongt_b200 import personal_pagerank_appnp
    rowptr, col = graph
    p = dict(alpha=0.15, topk=8, num_iterations=20, iter_topk=8)
    ei, val = personal_pagerank_appnp(None, csr_data={"rowptr": rowptr.cuda(), "col": col.cuda()}, device="cuda",
                                      return_fp64=True, **p)
    rei, rval = oppr.personal_pagerank_appnp(None, csr_data={"rowptr": rowptr, "col": col}, return_fp64=True,
                                             nthreads=8, **p)
    assert torch.equal(ei.cpu(), rei)
    assert torch.equal(val.cpu(), rval)


def _slim(cfg_seed=0):
    from neutrongt_b200.models import Graphormer
    torch.manual_seed(cfg_seed)
    return Graphormer(n_layers=4, num_heads=8, input_dim=128, hidden_dim=64, output_dim=40, attn_bias_dim=1,
                      dropout_rate=0.0, input_dropout_rate=0.0, attention_dropout_rate=0.0, ffn_dim=64,
                      num_global_node=1, args=SimpleNamespace(struct_enc="False"), num_in_degree=0,
                      num_out_degree=0, num_spatial=7, num_edges=512, max_dist=5, edge_dim=64)


def test_windows_and_one_training_epoch(cuda, graph):
    from neutrongt_b200 import synthetic
    from neutrongt_b200.train import FlatGradients, build_window_state, train_epoch
    rowptr, col = graph
    feature = synthetic.node_features(N, 128, seed=1)
    y = synthetic.node_labels(N, 40, seed=2)
    split = synthetic.split_idx(N, seed=3)
    parts = synthetic.random_partitions(N, 16, seed=0)
    ws = build_window_state(rowptr, col, parts, 0, 1, feature.cuda(), "cuda", split)
    for w, e in zip(ws.local_partitions, ws.local_sub_edge_index_for_partition_results):
        assert torch.equal(e.cpu(), owin.subgraph_from_csr(w, rowptr, col))

    model = _slim().cuda()
    # a larger spread than init_params' 0.02/sqrt(L) so attention carries signal into the loss
    with torch.no_grad():
        for p in model.parameters():
            if p.dim() == 2:
                p.normal_(0.0, 0.2)
    ref = copy.deepcopy(model).cpu().double()

    def attn(q, k, v, ei, bias):
        x, ns, _, _ = oatt.sparse_attention_forward(q, k, v, ei, bias)
        return x, ns

    for layer in ref.layers:
        layer.self_attention.local_attn.sparse_attention_bias = attn

    args = SimpleNamespace(use_cache=1, attn_type="sparse")
    opt = torch.optim.AdamW(model.parameters(), lr=1e-3, weight_decay=0.01)
    sched = torch.optim.lr_scheduler.LambdaLR(opt, lambda e: 1.0)
    loss_gpu, _, _, _ = train_epoch(args, model, ws.local_partition_ids, ws.local_partitions, feature.cuda(),
                                    y.cuda(), opt, sched, 1, split, "cuda", 0, ws, grads=FlatGradients(model))

    ropt = torch.optim.AdamW(ref.parameters(), lr=1e-3, weight_decay=0.01)
    train = split["train"]
    losses = []
    for idx, ei in zip(ws.local_partitions, ws.local_sub_edge_index_for_partition_results):
        out, _, _, _ = ref(feature[idx].double(), None, ei.cpu(), None, None, None, None, attn_type="sparse")
        m = torch.isin(idx, train).double()
        loss = (F.nll_loss(out, y[idx], reduction="none") * m).sum() / m.sum().clamp_min(1.0)
        ropt.zero_grad(set_to_none=True)
        loss.backward()
        ropt.step()
        losses.append(float(loss.detach()))
    loss_ref = sum(losses) / len(losses)
    assert abs(loss_gpu - loss_ref) < 1e-3
    for (name, p_gpu), p_ref in zip(model.named_parameters(), ref.parameters()):
        err = float((p_gpu.detach().double().cpu() - p_ref.detach()).abs().max())
        assert err < 1e-3, name
