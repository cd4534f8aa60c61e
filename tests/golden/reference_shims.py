"""Import shims that let the reference's own Python run on a CPU-only host.

Used only by `make_golden.py` (the fixture generator), in the build container
where the reference checkout exists.  The reference imports several packages
that are absent here (`torch_scatter`, `torch_geometric`, `dgl`, `pymetis`);
this module installs small stand-ins into `sys.modules` before the reference is
imported.  The stand-ins restate the documented behaviour of the functions the
hot path calls:

* `torch_scatter.scatter(src, index, dim, out, dim_size, reduce='sum'|'add')`
  (torch_scatter 2.1.1): sum of `src` rows into `out` along `dim`; when `out` is
  None the output length is `dim_size` or `index.max() + 1` (0 for an empty
  index).  Implemented with `index_add_`, which on CPU adds in index order.
* `torch_geometric.utils.subgraph(subset, edge_index, relabel_nodes=True,
  num_nodes)` (PyG 2.4.0): keep edges with both ends in `subset`, in their
  original order, relabelled to the position of each node in `subset`.
* `pymetis.CSRAdjacency(adj_starts, adjacent)`: the record pymetis builds from the
  two CSR lists (`build_adj_fromat` constructs one); it keeps both lists as given.
* `dgl`, the rest of `pymetis` (`part_graph`), `torch_geometric.utils.ppr` are inert
  placeholders; nothing on the paths exercised by the fixtures calls them.
"""
from __future__ import annotations

import os
import sys
import types

import torch

# The reference checkout's NeutronGT/ directory (the one holding models/, core/, gt_sp/), named by
# the NEUTRONGT_REFERENCE environment variable.
REFERENCE_ROOT = os.environ.get("NEUTRONGT_REFERENCE", "")


def _scatter(src, index, dim=-1, out=None, dim_size=None, reduce="sum"):
    if reduce not in ("sum", "add"):
        raise NotImplementedError(f"scatter reduce={reduce!r} is not needed by the hot path")
    dim = dim if dim >= 0 else src.dim() + dim
    index = index.to(torch.long)
    if out is None:
        if dim_size is None:
            dim_size = int(index.max()) + 1 if index.numel() > 0 else 0
        shape = list(src.shape)
        shape[dim] = dim_size
        out = src.new_zeros(shape)
    return out.index_add_(dim, index, src)


def _subgraph(subset, edge_index, edge_attr=None, relabel_nodes=False, num_nodes=None,
              return_edge_mask=False):
    device = edge_index.device
    subset = torch.as_tensor(subset, dtype=torch.long, device=device)
    if num_nodes is None:
        num_nodes = int(edge_index.max()) + 1 if edge_index.numel() else 0
        if subset.numel():
            num_nodes = max(num_nodes, int(subset.max()) + 1)
    node_mask = torch.zeros(num_nodes, dtype=torch.bool, device=device)
    node_mask[subset] = True
    edge_mask = node_mask[edge_index[0]] & node_mask[edge_index[1]]
    out = edge_index[:, edge_mask]
    if relabel_nodes:
        mapping = torch.full((num_nodes,), -1, dtype=torch.long, device=device)
        mapping[subset] = torch.arange(subset.numel(), device=device)
        out = mapping[out]
    attr = edge_attr[edge_mask] if edge_attr is not None else None
    if return_edge_mask:
        return out, attr, edge_mask
    return out, attr


class _CSRAdjacency:
    def __init__(self, adj_starts, adjacent):
        self.adj_starts = adj_starts
        self.adjacent = adjacent


def _inert(name):
    mod = types.ModuleType(name)

    def __getattr__(attr):
        def _unavailable(*a, **k):
            raise RuntimeError(f"{name}.{attr} is not available in the fixture environment")
        return _unavailable

    mod.__getattr__ = __getattr__
    return mod


def install():
    """Install the stand-ins and put the reference tree on sys.path (idempotent)."""
    if "torch_scatter" not in sys.modules:
        ts = types.ModuleType("torch_scatter")
        ts.scatter = _scatter
        sys.modules["torch_scatter"] = ts
    if "torch_geometric" not in sys.modules:
        tg = types.ModuleType("torch_geometric")
        tgu = types.ModuleType("torch_geometric.utils")
        tgu.subgraph = _subgraph
        for name in ("to_undirected", "remove_self_loops", "add_self_loops", "degree"):
            setattr(tgu, name, getattr(_inert("torch_geometric.utils"), name))
        tgu.ppr = _inert("torch_geometric.utils.ppr")
        tg.utils = tgu
        sys.modules["torch_geometric"] = tg
        sys.modules["torch_geometric.utils"] = tgu
        sys.modules["torch_geometric.utils.ppr"] = tgu.ppr
    for name in ("dgl", "pymetis"):
        if name not in sys.modules:
            sys.modules[name] = _inert(name)
    pm = sys.modules["pymetis"]
    if not isinstance(getattr(pm, "__dict__", {}).get("CSRAdjacency"), type):
        pm.CSRAdjacency = _CSRAdjacency
    if not REFERENCE_ROOT or not os.path.isdir(REFERENCE_ROOT):
        raise RuntimeError("set NEUTRONGT_REFERENCE to the reference checkout's NeutronGT directory")
    if REFERENCE_ROOT not in sys.path:
        sys.path.insert(0, REFERENCE_ROOT)
    import utils.logger as ref_logger  # noqa: E402  (reference module)
    ref_logger.IS_LOGGING = False
