"""CPU oracle for the NeutronGT hot path — TEST INFRASTRUCTURE ONLY.

This package restates, on the CPU, the reference algorithms that the CUDA
library in `neutrongt_b200` replaces.  It is the checker, never the product:
only `tests/`, `__graft_entry__.smoke()` and `bench.py`'s CPU-baseline /
reference arm may import it.  Nothing in `neutrongt_b200` imports it, and the
product path raises if its CUDA library is missing rather than falling back
to anything here.

Modules
-------
attention : graph-sparse window attention forward/backward
            (`models/gt_dist_node_level_single_window.py:112-179`)
window    : window subgraph construction and duplicate-first ordering
            (`core/node_level_pipeline/window_state.py:52-140`)
ppr       : APPNP personalised PageRank with per-iteration top-k, in a canonical
            fp64 order (`core/ppr_backends/appnp_backend.py:17-310`); the arithmetic
            runs in the C file `appnp_oracle.c` built by `oracle/Makefile`.

Pinning: every module is checked against fixtures produced by running the
reference's own code (`tests/golden/make_golden.py`), see tests/test_oracle.py.
"""
