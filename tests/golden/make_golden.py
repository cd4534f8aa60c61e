"""Generate the golden fixtures under tests/golden/ by running the reference itself.

Run where the reference checkout exists, naming its NeutronGT/ directory:

    NEUTRONGT_REFERENCE=<checkout>/NeutronGT python tests/golden/make_golden.py [section ...]

Every output below comes from the reference's own Python, imported unmodified,
with `reference_shims.install()` standing in for packages that are absent here
(torch_scatter's sum scatter, PyG's `subgraph`, placeholders for dgl/pymetis):

* attention_*.pt  – `CoreAttention.sparse_attention_bias` and `CoreAttention.forward`
  (`models/gt_dist_node_level_single_window.py:112-179, 198-227`) forward in fp32
  and fp64, backward through torch autograd in fp64.
* dense_attention.pt – `CoreAttention.full_attention` and `CoreAttention.forward(attn_type="full")`
  (`models/gt_dist_node_level_single_window.py:56-109, 198-227`), dropout 0, on bf16-representable
  inputs: forward and fp64 autograd backward (dq, dk, dv and, where given, the gradients of
  attn_bias and pruning_mask); cases with attn_bias, an additive pruning_mask holding -inf entries,
  and a boolean mask with one fully masked row.
* window_subgraph.pt – `_subgraph_from_csr` and `_compute_local_duplicate_nodes`
  (`core/node_level_pipeline/window_state.py:92-119, 52-73`).
* appnp_*.pt – APPNP top-k PPR.  `personal_pagerank_appnp` refuses CPU devices
  (`core/ppr_backends/appnp_backend.py:217-218`), so the batch loop of
  `appnp_backend.py:259-305` is driven here while every step inside it is the
  reference's own helper (`_build_csr_from_edge_index`, `_load_csr_graph`,
  `_build_transition_csr_values`, `_cusparse_spgemm_iteration`,
  `_segment_topk_from_csr`), with cuSPARSE's `csr_spgemm` replaced by a CPU
  SciPy SpGEMM in fp32.
* window_build.pt – `build_adj_fromat` (`core/ppr_preprocess.py:30-71`) on a seeded
  PPR-shaped list, then `weightMetis_keepParent._merge_related_nodes` and
  `._find_duplicate_nodes_and_rerange` (`core/metisPartition.py:397-425, 333-363`) called on
  a stand-in `self` that holds only the attributes those methods read (the class constructor
  runs METIS, which is absent here).
* gt_sw_step.pt / graphormer_step.pt – one training step (forward, NLL loss,
  backward) of the reference `GT_SW` and `Graphormer` modules with dropout 0,
  sparse attention, together with their initial state_dicts.

Inputs are seeded; the fixtures are small enough to commit.
"""
from __future__ import annotations

import os
import sys
from types import SimpleNamespace

import numpy as np
import scipy.sparse as sp
import torch

HERE = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, HERE)
sys.path.insert(0, os.path.dirname(os.path.dirname(HERE)))

import reference_shims  # noqa: E402

reference_shims.install()

from neutrongt_b200 import synthetic  # noqa: E402


def _save(name, payload):
    path = os.path.join(HERE, name)
    torch.save(payload, path)
    print(f"wrote {path} ({os.path.getsize(path) / 1024:.1f} KiB)")


# --------------------------------------------------------------------------------------
# attention
# --------------------------------------------------------------------------------------

def _attention_case(name, s, H, D, edges, seed, in_scale=1.0, with_bias=False):
    from models.gt_dist_node_level_single_window import CoreAttention

    g = torch.Generator().manual_seed(seed)
    q = torch.randn(1, s, H, D, generator=g) * in_scale
    k = torch.randn(1, s, H, D, generator=g) * in_scale
    v = torch.randn(1, s, H, D, generator=g)
    dout = torch.randn(1, s, H, D, generator=g)
    bias = torch.randn(1, H, s, s, generator=g) if with_bias else None
    edge_index = edges

    attn = CoreAttention(H * D, 0.0, H)
    # fp32 forward
    x32, ns32 = attn.sparse_attention_bias(q, k, v, edge_index, bias)
    # fp64 forward + autograd backward
    q64 = q.double().requires_grad_(True)
    k64 = k.double().requires_grad_(True)
    v64 = v.double().requires_grad_(True)
    b64 = bias.double().requires_grad_(True) if with_bias else None
    x64, ns64 = attn.sparse_attention_bias(q64, k64, v64, edge_index, b64)
    (x64 * dout.double().view_as(x64)).sum().backward()
    # the module-level dispatch (attn_type == "sparse") reshapes to [b, s, H*D]
    xf, sf = attn.forward(q, k, v, bias, edge_index, "sparse")
    payload = {
        "s": s, "H": H, "D": D,
        "q": q, "k": k, "v": v, "dout": dout, "edge_index": edge_index, "attn_bias": bias,
        "x32": x32, "node_scores32": ns32,
        "x64": x64.detach(), "node_scores64": ns64.detach(),
        "dq64": q64.grad, "dk64": k64.grad, "dv64": v64.grad,
        "dbias64": b64.grad if with_bias else None,
        "forward_x": xf, "forward_score": sf,
    }
    _save(f"attention_{name}.pt", payload)


def make_attention():
    g = torch.Generator().manual_seed(1234)
    # A: GPH_Slim head shape (D=8), random edges with repeats and self loops; the
    # last 5 nodes receive no edge, so node_scores is shorter than s.
    s = 96
    E = 700
    src = torch.randint(0, s, (E,), generator=g)
    dst = torch.randint(0, s - 5, (E,), generator=g)
    dst[:40] = src[:40]                       # self loops
    src[40:60] = src[60:80]; dst[40:60] = dst[60:80]   # repeated edges
    _attention_case("slim_d8", s, 8, 8, torch.stack([src, dst]), seed=1)
    # B: GT head shape (D=16), window edge list from a power-law graph (source-major
    # order, as `_subgraph_from_csr` emits); inputs scaled so many scores clamp.
    rowptr, col = synthetic.chung_lu_graph(64, 300, seed=3)
    ei = synthetic.edge_index_from_src_csr(rowptr, col)
    _attention_case("gt_d16_clamp", 64, 8, 16, ei, seed=2, in_scale=2.5)
    # C: dense attention bias gathered per edge (struct_enc path), D=8, H=4.
    s = 48
    src = torch.randint(0, s, (300,), generator=g)
    dst = torch.randint(0, s, (300,), generator=g)
    _attention_case("bias_h4", s, 4, 8, torch.stack([src, dst]), seed=3, with_bias=True)
    # D: empty edge list.
    _attention_case("empty", 16, 8, 8, torch.empty(2, 0, dtype=torch.long), seed=4)


# --------------------------------------------------------------------------------------
# dense full attention
# --------------------------------------------------------------------------------------

def _dense_case(s, H, D, seed, bias=False, pruning=False, mask=False):
    from models.gt_dist_node_level_single_window import CoreAttention

    g = torch.Generator().manual_seed(seed)
    # bf16-representable inputs: the kernels compute in bf16, so the comparison measures the
    # kernels' arithmetic, not the input rounding
    mk = lambda: (torch.randn(1, s, H, D, generator=g) * 0.5).to(torch.bfloat16).double()  # noqa: E731
    q, k, v, dout = mk(), mk(), mk(), mk()
    attn_bias = torch.randn(1, H, s, s, generator=g).double() if bias else None   # fp32 values, exact in fp64
    pruning_mask = None
    if pruning:
        u = torch.rand(1, 1, s, s, generator=g)
        pruning_mask = torch.where(u < 0.1, torch.tensor(float("-inf")),
                                   torch.where(u < 0.3, torch.tensor(-3.0), torch.tensor(0.0))).double()
    mask_t = None
    if mask:
        mask_t = torch.rand(s, s, generator=g) < 0.15
        mask_t[5] = True                        # one fully masked query row: uniform softmax
    attn = CoreAttention(H * D, 0.0, H).eval()
    leaves = [t.clone().requires_grad_(True) for t in (q, k, v)]
    b_leaf = attn_bias.clone().requires_grad_(True) if bias else None
    p_leaf = pruning_mask.clone().requires_grad_(True) if pruning else None
    x, ns = attn.full_attention(leaves[1], leaves[0], leaves[2], b_leaf, mask=mask_t, pruning_mask=p_leaf)
    (x * dout).sum().backward()
    xf, sf = attn.forward(q.float(), k.float(), v.float(), None if attn_bias is None else attn_bias.float(), None,
                          "full", mask=mask_t, pruning_mask=None if pruning_mask is None else pruning_mask.float())
    # stored compactly: inputs as bf16 / fp32 (exact), the fp64 results rounded to fp32
    f32 = lambda t: None if t is None else t.detach().float()  # noqa: E731
    return {"s": s, "H": H, "D": D, "q": q.to(torch.bfloat16), "k": k.to(torch.bfloat16),
            "v": v.to(torch.bfloat16), "dout": dout.to(torch.bfloat16),
            "attn_bias": f32(attn_bias), "pruning_mask": f32(pruning_mask), "mask": mask_t,
            "x": f32(x), "node_scores": f32(ns), "dq": f32(leaves[0].grad), "dk": f32(leaves[1].grad),
            "dv": f32(leaves[2].grad), "dbias": f32(b_leaf.grad) if bias else None,
            "dpruning": f32(p_leaf.grad) if pruning else None, "forward_x": xf, "forward_score": sf}


def make_dense():
    cases = {
        "d24_h4": _dense_case(160, 4, 24, seed=31),       # the GPH_Large head shape (768 / 32)
        "d16_h2": _dense_case(300, 2, 16, seed=32),
        "d8_h3": _dense_case(96, 3, 8, seed=33),
        "d64_h2": _dense_case(130, 2, 64, seed=34),
        "d40_h1": _dense_case(200, 1, 40, seed=35),
        "bias_d16": _dense_case(144, 2, 16, seed=36, bias=True),
        "bias_pruning_mask_d24": _dense_case(136, 2, 24, seed=37, bias=True, pruning=True, mask=True),
        "mask_d64": _dense_case(150, 2, 64, seed=38, mask=True),
    }
    _save("dense_attention.pt", cases)


# --------------------------------------------------------------------------------------
# window subgraph + duplicate-first ordering
# --------------------------------------------------------------------------------------

def make_window():
    from core.node_level_pipeline.window_state import _compute_local_duplicate_nodes, _subgraph_from_csr

    rowptr, col = synthetic.chung_lu_graph(400, 1500, seed=5)
    g = torch.Generator().manual_seed(6)
    parts = synthetic.random_partitions(400, 6, seed=7)
    # grow each part with a few foreign nodes so windows overlap (duplicates exist)
    windows = []
    for p in parts:
        extra = torch.randint(0, 400, (12,), generator=g)
        windows.append(torch.unique(torch.cat([p, extra])))
    reranged, dup_nodes = _compute_local_duplicate_nodes(windows)
    sub = [_subgraph_from_csr(w, rowptr, col) for w in reranged]
    _save("window_subgraph.pt", {
        "rowptr": rowptr, "col": col, "windows": windows,
        "reranged": reranged, "dup_nodes": dup_nodes, "sub_edge_index": sub,
    })


# --------------------------------------------------------------------------------------
# APPNP PPR + top-k
# --------------------------------------------------------------------------------------

def _cpu_spgemm(rowptr_a, col_a, val_a, rowptr_b, col_b, val_b):
    """CPU stand-in for cuSPARSE SpGEMM (`cusparse_ops.py:97-114`): C = A @ B in fp32."""
    n_b = rowptr_b.numel() - 1
    a = sp.csr_matrix((val_a.numpy().astype(np.float32), col_a.numpy(), rowptr_a.numpy()),
                      shape=(rowptr_a.numel() - 1, n_b))
    b = sp.csr_matrix((val_b.numpy().astype(np.float32), col_b.numpy(), rowptr_b.numpy()),
                      shape=(n_b, n_b))
    c = (a @ b).tocsr()
    c.sort_indices()
    return (torch.from_numpy(c.indptr.astype(np.int64)), torch.from_numpy(c.indices.astype(np.int64)),
            torch.from_numpy(c.data.astype(np.float32)))


def _reference_appnp_cpu(csr, alpha, topk, num_iterations, batch_size, iter_topk, source_start=None,
                         source_end=None, edge_index=None):
    from core.ppr_backends import appnp_backend as ab

    ab.csr_spgemm = _cpu_spgemm
    device = torch.device("cpu")
    if csr is not None:
        graph_rowptr, graph_col, degree, num_nodes = ab._load_csr_graph(csr, device=device)
    else:
        graph_rowptr, graph_col, degree, num_nodes = ab._build_csr_from_edge_index(edge_index, device=device)
    values = ab._build_transition_csr_values(graph_rowptr, graph_col, degree)
    batch_size = max(1, int(batch_size))
    num_iterations = max(1, int(num_iterations))
    source_start = 0 if source_start is None else max(0, min(int(source_start), num_nodes))
    source_end = num_nodes if source_end is None else max(source_start, min(int(source_end), num_nodes))
    topk = min(int(topk), num_nodes)
    iter_topk = topk if iter_topk is None else int(iter_topk)
    iter_topk = None if iter_topk <= 0 else min(iter_topk, num_nodes)
    out_idx, out_val = [], []
    for start in range(source_start, source_end, batch_size):
        end = min(start + batch_size, source_end)
        seeds = torch.arange(start, end, dtype=torch.long)
        rows = seeds.numel()
        st_rowptr = torch.arange(0, rows + 1, dtype=torch.long)
        st_col = seeds.clone()
        st_val = torch.ones(rows, dtype=torch.float32)
        tp_rows = torch.arange(rows, dtype=torch.long)
        tp_cols = seeds
        tp_vals = torch.full((rows,), alpha, dtype=torch.float32)
        for _ in range(num_iterations):
            st_rowptr, st_col, st_val = ab._cusparse_spgemm_iteration(
                st_rowptr, st_col, st_val, graph_rowptr, graph_col, values,
                tp_rows, tp_cols, tp_vals, rows, num_nodes, alpha, iter_topk)
        final_keep = topk if iter_topk is None else min(topk, iter_topk)
        st_rowptr, st_col, st_val = ab._segment_topk_from_csr(st_rowptr, st_col, st_val, final_keep)
        lengths = st_rowptr[1:] - st_rowptr[:-1]
        out_idx.append(torch.stack([seeds.repeat_interleave(lengths), st_col]))
        out_val.append(st_val)
    return torch.cat(out_idx, dim=1), torch.cat(out_val)


def make_appnp():
    rowptr, col = synthetic.chung_lu_graph(300, 900, seed=11)
    csr = {"rowptr": rowptr, "col": col}
    cases = {
        "cfg1": dict(alpha=0.15, topk=8, num_iterations=20, batch_size=64, iter_topk=8),
        "scripts": dict(alpha=0.85, topk=5, num_iterations=10, batch_size=8192, iter_topk=5),
        "unpruned": dict(alpha=0.15, topk=8, num_iterations=20, batch_size=100, iter_topk=0),
        "narrow_iter": dict(alpha=0.3, topk=8, num_iterations=6, batch_size=7, iter_topk=3),
        "shard": dict(alpha=0.15, topk=8, num_iterations=12, batch_size=16, iter_topk=8,
                      source_start=100, source_end=177),
    }
    out = {"rowptr": rowptr, "col": col, "cases": {}}
    for name, kw in cases.items():
        idx, val = _reference_appnp_cpu(csr, **kw)
        out["cases"][name] = {"params": kw, "edge_index": idx, "values": val}
    # a denser, nearly degree-uniform graph: few structural ties at the top-k
    # boundary, so most seeds pin the pruned mode exactly
    rp2, col2 = synthetic.chung_lu_graph(200, 1300, exponent=12.0, seed=13)
    out["dense"] = {"rowptr": rp2, "col": col2, "cases": {}}
    for name, kw in {"cfg1": cases["cfg1"], "scripts": cases["scripts"]}.items():
        idx, val = _reference_appnp_cpu({"rowptr": rp2, "col": col2}, **kw)
        out["dense"]["cases"][name] = {"params": kw, "edge_index": idx, "values": val}
    # the edge_index entry point (`_build_csr_from_edge_index`) on an unsorted,
    # non-symmetric edge list with a repeated edge
    g = torch.Generator().manual_seed(12)
    ei = torch.randint(0, 60, (2, 240), generator=g)
    ei[:, 5] = ei[:, 4]
    idx, val = _reference_appnp_cpu(None, 0.2, 6, 8, 16, 6, edge_index=ei)
    out["edge_index_case"] = {"edge_index_in": ei, "params": dict(alpha=0.2, topk=6, num_iterations=8,
                                                                   batch_size=16, iter_topk=6),
                              "edge_index": idx, "values": val}
    _save("appnp.pt", out)


# --------------------------------------------------------------------------------------
# model training step (loss parity)
# --------------------------------------------------------------------------------------

def _model_step(kind):
    import gt_sp.initialize as ini
    ini._SEQUENCE_PARALLEL_GROUP = object()
    ini._SEQUENCE_PARALLEL_WORLD_SIZE = 1
    import torch.nn.functional as F
    from models.graphormer_dist_node_level import Graphormer
    from models.gt_dist_node_level_single_window import GT_SW

    torch.manual_seed(21)
    args = SimpleNamespace(struct_enc="False")
    common = dict(n_layers=2, num_heads=4, input_dim=16, hidden_dim=32, output_dim=5, attn_bias_dim=1,
                  dropout_rate=0.0, input_dropout_rate=0.0, attention_dropout_rate=0.0, ffn_dim=48,
                  num_global_node=1, args=args, num_in_degree=0, num_out_degree=0, num_spatial=7,
                  num_edges=512, max_dist=5, edge_dim=64)
    model = (GT_SW if kind == "gt_sw" else Graphormer)(**common)
    # init_params draws tiny weights (std 0.02/sqrt(L)); give the projections a
    # larger spread so the attention path carries signal into the loss.
    with torch.no_grad():
        for name, p in model.named_parameters():
            if p.dim() == 2:
                p.normal_(0.0, 0.3)
    state = {k: v.clone() for k, v in model.state_dict().items()}
    g = torch.Generator().manual_seed(22)
    n = 80
    x = torch.randn(n, 16, generator=g)
    y = torch.randint(0, 5, (n,), generator=g)
    rowptr, col = synthetic.chung_lu_graph(n, 300, seed=23)
    edge_index = synthetic.edge_index_from_src_csr(rowptr, col)
    train_mask = torch.rand(n, generator=g) < 0.6
    model.train()
    out, _, score_spe, _ = model(x, None, edge_index, None, None, None, None, attn_type="sparse")
    loss = F.nll_loss(out, y, reduction="none")[train_mask].mean()
    loss.backward()
    grads = {k: p.grad.clone() for k, p in model.named_parameters() if p.grad is not None}
    _save(f"{kind}_step.pt", {"state_dict": state, "x": x, "y": y, "edge_index": edge_index,
                              "train_mask": train_mask, "out": out.detach(), "loss": float(loss.detach()),
                              "scores": [s.clone() for s in score_spe], "grads": grads,
                              "config": {k: v for k, v in common.items() if k != "args"}})


# --------------------------------------------------------------------------------------
# window construction: PPR adjacency, halo merge, duplicate-first order
# --------------------------------------------------------------------------------------

def _ppr_like(n, k, seed):
    """k neighbours per seed with PPR-like values: a few large, many tiny (weight 1 after the
    x1000 truncation, so the halo ranking has ties), and some pairs listed in both directions."""
    g = torch.Generator().manual_seed(seed)
    src = torch.arange(n).repeat_interleave(k)
    dst = torch.randint(0, n, (n * k,), generator=g)
    vals = torch.rand(n * k, generator=g) ** 6 * 0.3
    mirror = torch.randperm(n * k, generator=g)[: n * k // 5]
    src = torch.cat([src, dst[mirror]])
    dst = torch.cat([dst, src[mirror]])
    vals = torch.cat([vals, torch.rand(mirror.numel(), generator=g) * 0.05]).to(torch.float32)
    return torch.stack([src, dst]), vals


def make_window_build():
    from core.metisPartition import weightMetis_keepParent
    from core.ppr_preprocess import build_adj_fromat

    n = 600
    ppr_ei, ppr_val = _ppr_like(n, 6, seed=21)
    csr, eweights, _ = build_adj_fromat((ppr_ei, ppr_val))
    g = torch.Generator().manual_seed(22)
    perm = torch.randperm(n, generator=g)
    windows = [torch.sort(c).values for c in torch.tensor_split(perm, 6)]
    fake = SimpleNamespace(csr_adjacency=csr, eweights=eweights)
    halos = {}
    for pct in (0, 7, 30, 100):
        halos[pct] = [weightMetis_keepParent._merge_related_nodes(fake, w, pct) for w in windows]
    # duplicate-first order over the halo-grown windows (they overlap), grouped 3 + 3 by parent
    child = [halos[30][:3], halos[30][3:]]
    fake2 = SimpleNamespace(child_partitions=[list(grp) for grp in child])
    dups = weightMetis_keepParent._find_duplicate_nodes_and_rerange(fake2)
    _save("window_build.pt", {
        "ppr_edge_index": ppr_ei, "ppr_val": ppr_val,
        "xadj": torch.tensor(csr.adj_starts, dtype=torch.int32),
        "adjncy": torch.tensor(csr.adjacent, dtype=torch.int32),
        "eweights": torch.tensor(eweights, dtype=torch.int32),
        "windows": windows, "halos": halos,
        "child_partitions": child, "reranged": fake2.child_partitions, "dup_nodes": dups,
    })


if __name__ == "__main__":
    # python tests/golden/make_golden.py [section ...]   (default: every section)
    torch.set_num_threads(1)
    sections = {
        "attention": make_attention,
        "dense": make_dense,
        "window": make_window,
        "appnp": make_appnp,
        "gt_sw": lambda: _model_step("gt_sw"),
        "graphormer": lambda: _model_step("graphormer"),
        "window_build": make_window_build,
    }
    for name in (sys.argv[1:] or list(sections)):
        sections[name]()
