"""neutrongt_b200 — B200-native kernels for NeutronGT's data-parallel hot path.

Host-side mirrors of the reference interfaces, each backed by hand-written sm_100a CUDA
kernels in `csrc/` reached through the C ABI of `include/neutrongt_b200.h`:

* `attention.sparse_attention_bias` / `attention.CoreAttention` — graph-sparse window
  attention (`NeutronGT/models/gt_dist_node_level_single_window.py:112-227`)
* `ppr.personal_pagerank_appnp` / `ppr.personal_pagerank_torch_geometric` / `ppr.personal_pagerank` —
  APPNP PPR + top-k, push PPR + top-k, and the backend dispatcher
  (`NeutronGT/core/ppr_backends/appnp_backend.py:203-310`)
* `window.subgraph_from_csr` — window edge lists
  (`NeutronGT/core/node_level_pipeline/window_state.py:92-119`)
"""
from .attention import CoreAttention, sparse_attention_bias  # noqa: F401
from .ppr import personal_pagerank, personal_pagerank_appnp, personal_pagerank_torch_geometric  # noqa: F401
from .window import compute_local_duplicate_nodes, subgraph_from_csr  # noqa: F401

__all__ = [
    "CoreAttention",
    "sparse_attention_bias",
    "personal_pagerank",
    "personal_pagerank_appnp",
    "personal_pagerank_torch_geometric",
    "subgraph_from_csr",
    "compute_local_duplicate_nodes",
]
