"""Seeded synthetic inputs that stand in for the datasets the reference trains on.

The reference reads ogbn-arxiv / products / Reddit / AmazonProducts from disk
(`NeutronGT/core/node_level_pipeline/graph_data.py:6-26` for the CSR file, the
`x.pt / y.pt / edge_index.pt` triple for the rest).  Those datasets are not
available here, so every benchmark and test builds graphs of the same shape from
a seed instead:

* `chung_lu_graph` – undirected power-law graph (Chung-Lu model), symmetrised and
  stored as an int64 CSR `{rowptr, col}` with each row's columns ascending, the
  layout `utils/trans2csr.py:24-37` writes.
* `chung_lu_graph_device` – the same model sampled on the GPU (torch's CUDA generator), for the
  graphs with 10^7..10^8 edges; same degree distribution, different draws than the host version.
* `poisson_window_csr` – one attention window whose in-degree per destination row
  is Poisson distributed with uniform random sources (the isolated-kernel case).
* `random_partitions` – contiguous chunks of a seeded permutation, each sorted,
  the stand-in for METIS windows.

Everything here is plain numpy / torch on the host and deterministic for a seed.
"""
from __future__ import annotations

import numpy as np
import torch


def chung_lu_graph(num_nodes: int, num_undirected_edges: int, exponent: float = 2.5,
                   seed: int = 0) -> tuple[torch.Tensor, torch.Tensor]:
    """Power-law graph with exactly `num_undirected_edges` distinct undirected edges.

    Node i gets weight (i + 1) ** (-1 / (exponent - 1)); both ends of a candidate
    edge are drawn independently with probability proportional to weight.
    Self loops and repeats are dropped; the first `num_undirected_edges`
    distinct pairs in draw order are kept.  Returns (rowptr, col), int64, with
    both directions of every edge present and each row sorted ascending.
    """
    n = int(num_nodes)
    m = int(num_undirected_edges)
    if n <= 1 or m <= 0:
        return torch.zeros(n + 1, dtype=torch.long), torch.empty(0, dtype=torch.long)
    max_edges = n * (n - 1) // 2
    if m > max_edges:
        raise ValueError(f"{m} undirected edges do not fit in a simple graph on {n} nodes")
    rng = np.random.default_rng(seed)
    w = (np.arange(1, n + 1, dtype=np.float64)) ** (-1.0 / (exponent - 1.0))
    cdf = np.cumsum(w)
    cdf /= cdf[-1]
    keys_parts: list[np.ndarray] = []
    have = 0
    while have < m:
        batch = int((m - have) * 1.3) + 1024
        u = np.searchsorted(cdf, rng.random(batch), side="right")
        v = np.searchsorted(cdf, rng.random(batch), side="right")
        np.minimum(u, n - 1, out=u)
        np.minimum(v, n - 1, out=v)
        keep = u != v
        lo = np.minimum(u[keep], v[keep]).astype(np.int64)
        hi = np.maximum(u[keep], v[keep]).astype(np.int64)
        keys_parts.append(lo * n + hi)
        allk = np.concatenate(keys_parts)
        _, first = np.unique(allk, return_index=True)
        have = first.size
        keys_parts = [allk[np.sort(first)]]
    keys = keys_parts[0][:m]
    lo = keys // n
    hi = keys % n
    src = np.concatenate([lo, hi])
    dst = np.concatenate([hi, lo])
    order = np.lexsort((dst, src))
    src = src[order]
    dst = dst[order]
    counts = np.bincount(src, minlength=n)
    rowptr = np.zeros(n + 1, dtype=np.int64)
    np.cumsum(counts, out=rowptr[1:])
    return torch.from_numpy(rowptr), torch.from_numpy(dst.astype(np.int64))


def chung_lu_graph_device(num_nodes: int, num_undirected_edges: int, exponent: float = 2.5, seed: int = 0,
                          device="cuda") -> tuple[torch.Tensor, torch.Tensor]:
    """`chung_lu_graph` sampled on the device: candidate pairs drawn with torch's seeded CUDA
    generator, self loops dropped, the distinct pairs deduplicated, `num_undirected_edges` of them
    kept by a seeded permutation.  Returns (rowptr int64, col int64) on `device`, both directions,
    rows ascending."""
    n, m = int(num_nodes), int(num_undirected_edges)
    dev = torch.device(device)
    if n <= 1 or m <= 0:
        return torch.zeros(n + 1, dtype=torch.long, device=dev), torch.empty(0, dtype=torch.long, device=dev)
    if m > n * (n - 1) // 2:
        raise ValueError(f"{m} undirected edges do not fit in a simple graph on {n} nodes")
    g = torch.Generator(device=dev).manual_seed(seed)
    w = torch.arange(1, n + 1, dtype=torch.float64, device=dev) ** (-1.0 / (exponent - 1.0))
    cdf = torch.cumsum(w, 0)
    cdf /= cdf[-1].clone()
    keys = torch.empty(0, dtype=torch.long, device=dev)
    draw = int(m * 1.25) + 4096
    for _ in range(256):
        if keys.numel() >= m:
            break
        u = torch.searchsorted(cdf, torch.rand(draw, generator=g, device=dev, dtype=torch.float64), right=True)
        v = torch.searchsorted(cdf, torch.rand(draw, generator=g, device=dev, dtype=torch.float64), right=True)
        u.clamp_(max=n - 1)
        v.clamp_(max=n - 1)
        keep = u != v
        lo, hi = torch.minimum(u[keep], v[keep]), torch.maximum(u[keep], v[keep])
        keys = torch.unique(torch.cat([keys, lo * n + hi]))
        draw = int((m - keys.numel()) * 2.0) + 4096
    if keys.numel() < m:
        raise RuntimeError(f"could not draw {m} distinct edges (the weights concentrate on too few pairs)")
    keys = keys[torch.randperm(keys.numel(), generator=g, device=dev)[:m]]
    lo, hi = keys // n, keys % n
    src = torch.cat([lo, hi])
    dst = torch.cat([hi, lo])
    del keys, lo, hi
    order = torch.argsort(src * n + dst)
    src, dst = src[order], dst[order]
    rowptr = torch.zeros(n + 1, dtype=torch.long, device=dev)
    rowptr[1:] = torch.cumsum(torch.bincount(src, minlength=n), 0)
    return rowptr, dst


def poisson_window_csr(num_tokens: int, mean_degree: float, seed: int = 0) -> tuple[torch.Tensor, torch.Tensor]:
    """Destination-major CSR of one window: row d lists the sources attending into d.

    In-degree of each row ~ Poisson(mean_degree); sources uniform in [0, num_tokens).
    """
    rng = np.random.default_rng(seed)
    n = int(num_tokens)
    deg = rng.poisson(mean_degree, size=n).astype(np.int64)
    rowptr = np.zeros(n + 1, dtype=np.int64)
    np.cumsum(deg, out=rowptr[1:])
    col = rng.integers(0, n, size=int(rowptr[-1]), dtype=np.int64)
    return torch.from_numpy(rowptr), torch.from_numpy(col)


def edge_index_from_dst_csr(rowptr: torch.Tensor, col: torch.Tensor) -> torch.Tensor:
    """[2, E] edge_index with row 0 = source (K/V row) and row 1 = destination (Q row)."""
    lengths = rowptr[1:] - rowptr[:-1]
    dst = torch.arange(lengths.numel(), dtype=torch.long).repeat_interleave(lengths)
    return torch.stack([col.to(torch.long), dst], dim=0)


def edge_index_from_src_csr(rowptr: torch.Tensor, col: torch.Tensor) -> torch.Tensor:
    """[2, E] edge_index of a source-major CSR (row 0 = row id, row 1 = column)."""
    lengths = rowptr[1:] - rowptr[:-1]
    src = torch.arange(lengths.numel(), dtype=torch.long).repeat_interleave(lengths)
    return torch.stack([src, col.to(torch.long)], dim=0)


def random_partitions(num_nodes: int, n_parts: int, seed: int = 0) -> list[torch.Tensor]:
    """`n_parts` contiguous chunks of a seeded permutation, each sorted ascending."""
    g = torch.Generator().manual_seed(seed)
    perm = torch.randperm(int(num_nodes), generator=g)
    return [torch.sort(p).values for p in torch.tensor_split(perm, int(n_parts))]


def node_features(num_nodes: int, dim: int, seed: int = 0, dtype=torch.float32) -> torch.Tensor:
    g = torch.Generator().manual_seed(seed)
    return torch.randn(int(num_nodes), int(dim), generator=g, dtype=torch.float32).to(dtype)


def node_labels(num_nodes: int, num_classes: int, seed: int = 0) -> torch.Tensor:
    g = torch.Generator().manual_seed(seed)
    return torch.randint(0, int(num_classes), (int(num_nodes),), generator=g, dtype=torch.long)


def split_idx(num_nodes: int, seed: int = 0, train: float = 0.6, valid: float = 0.2) -> dict:
    """Random train/valid/test split of node ids."""
    g = torch.Generator().manual_seed(seed)
    perm = torch.randperm(int(num_nodes), generator=g)
    a = int(num_nodes * train)
    b = int(num_nodes * (train + valid))
    return {"train": torch.sort(perm[:a]).values, "valid": torch.sort(perm[a:b]).values,
            "test": torch.sort(perm[b:]).values}
