"""Window-parallel training loop: the caller of the sparse attention.

`train_epoch` keeps the signature and semantics of the reference's
`NeutronGT/core/node_level_pipeline/train_eval.py:197-343`: every rank walks its own
windows; a rank with fewer windows takes zero-gradient steps so all ranks take the same
number of all-reduces (`:211-217, 284-285`); per window: gather features, forward,
masked NLL on the window's train nodes, backward, gradients averaged over ranks
(`:289-295`), optimizer step; the scheduler steps once per epoch.  It returns
`(loss_mean, scores_by_pid, kv_cache_per_partition, time_stats)`.

Changes of mechanism (not of results):
* window edge lists stay on the device (built once by `window.subgraph_from_csr`), so
  the per-step host->device copy of `edge_index` (`:244`) disappears, and the window's
  CSR views are built once and reused by every layer and epoch;
* features are gathered on the device when the feature matrix lives there; a host feature
  matrix is gathered on the host and copied through a pinned staging buffer;
* gradients live in one flat buffer (each parameter's .grad is a view of it), so the
  average over ranks is a few NCCL all-reduces per step instead of one per parameter; in the
  eager loop the buffer is cut into 4 MiB buckets that are all-reduced from post-accumulate
  hooks while backward still runs (the graph-replayed loop keeps one all-reduce per step);
* the window losses stay on the device and are read once per epoch, and the per-stage
  `torch.cuda.synchronize()` calls used for wall-clock timing are replaced by CUDA events.

`build_window_state` produces the per-rank fields the loop reads from the reference's
`StructInfo` (`struct_info.py:16-36`): round-robin window assignment (`window_state.py:210`),
duplicate-first ordering and the duplicate-feature cache (`window_state.py:52-73, 181-205`),
and window edge lists (`window_state.py:122-140`).
"""
from __future__ import annotations

import time
from dataclasses import dataclass, field

import torch
import torch.distributed as dist
import torch.nn.functional as F

from .layers import overlap_weight_grads
from .window import compute_local_duplicate_nodes, subgraph_from_csr


@dataclass
class WindowState:
    local_partition_ids: list
    local_partitions: list
    local_sub_edge_index_for_partition_results: list
    local_dup_indices: list
    local_dup_nodes_per_partition_feature: torch.Tensor
    local_train_masks: list = field(default_factory=list)
    graph_in_degree: torch.Tensor | None = None
    graph_out_degree: torch.Tensor | None = None
    local_spatial_pos_by_pid: list = field(default_factory=list)


def broadcast_partitions(partitions, src: int = 0, group=None, device=None) -> list:
    """The window node lists of rank `src` on every rank, by collective instead of files.

    The reference's rank 0 writes one bundle file per rank (`window_state.py:296-311`:
    `torch.save` of each rank's windows, a barrier, every rank `torch.load`s its own, a barrier,
    rank 0 deletes the files).  Here the node lists travel in three broadcasts (window count,
    lengths, the concatenated ids as int64) over the process group's backend, NCCL between GPUs
    (`device` then a CUDA device) or gloo on the host; every rank then takes its own windows
    (pid mod world_size) in `build_window_state`.  `partitions` is only read on `src`.
    Returns CPU int64 tensors, in the source's order."""
    import torch.distributed as dist
    dev = torch.device("cpu") if device is None else torch.device(device)
    rank = dist.get_rank(group)
    count = torch.zeros(1, dtype=torch.long, device=dev)
    if rank == src:
        count.fill_(len(partitions))
    dist.broadcast(count, src=src, group=group)
    n = int(count.item())
    lengths = torch.zeros(n, dtype=torch.long, device=dev)
    if rank == src and n:
        lengths.copy_(torch.tensor([int(p.numel()) for p in partitions], dtype=torch.long))
    if n:
        dist.broadcast(lengths, src=src, group=group)
    sizes = lengths.cpu().tolist()
    total = sum(sizes)
    flat = torch.empty(total, dtype=torch.long, device=dev)
    if rank == src and total:
        flat.copy_(torch.cat([p.reshape(-1).to(torch.long).cpu() for p in partitions]))
    if total:
        dist.broadcast(flat, src=src, group=group)
    return list(torch.split(flat.cpu(), sizes)) if n else []


def build_window_state(rowptr, col, partitions, rank, world_size, feature, device, split_idx=None,
                       use_cache=True) -> WindowState:
    ids = list(range(rank, len(partitions), world_size))
    parts = [partitions[p].to(torch.long).cpu() for p in ids]
    dups = [torch.empty(0, dtype=torch.long) for _ in parts]
    if use_cache:
        parts, dups = compute_local_duplicate_nodes(parts)
    nonempty = [d for d in dups if d.numel() > 0]
    if nonempty:
        dup_sorted = torch.unique(torch.cat(nonempty), sorted=True)
        dup_idx = [torch.searchsorted(dup_sorted, d).to(device) for d in dups]
        dup_feat = feature[dup_sorted.to(feature.device)].to(device)
    else:
        dup_idx = [torch.empty(0, dtype=torch.long, device=device) for _ in dups]
        dup_feat = feature.new_empty((0, feature.shape[1]), device=device)
    rp, cl = rowptr.to(device), col.to(device)
    edges = [subgraph_from_csr(p, rp, cl, device=device) for p in parts]
    masks = []
    if split_idx is not None:
        train = split_idx["train"].to(device)
        masks = [torch.isin(p.to(device), train) for p in parts]
    return WindowState(ids, parts, edges, dup_idx, dup_feat, masks)


class FlatGradients:
    """All parameters' gradients as views of one flat buffer (one all-reduce per step).

    `zero(set_to_none=True)` is the single-process form of the reference loop
    (`optimizer.zero_grad(set_to_none=True)`, train_eval.py:287): gradients start as None, a
    parameter without a gradient in the window is skipped by the optimizer, and backward hands
    each fresh gradient to its parameter without an accumulate kernel.  With more than one rank
    the reference gives every parameter a gradient (zeros where none was produced) and
    all-reduces them (train_eval.py:289-295): `zero()` keeps the flat views for that."""

    def __init__(self, model: torch.nn.Module, bucket_bytes: int | None = None, group=None):
        self.params = [p for p in model.parameters() if p.requires_grad]
        total = sum(p.numel() for p in self.params)
        dev = self.params[0].device
        self.flat = torch.zeros(total, dtype=self.params[0].dtype, device=dev)
        self._bind()
        self.group = group
        self.buckets = None
        if bucket_bytes is not None and dist.is_available() and dist.is_initialized() \
                and dist.get_world_size(group) > 1:
            self._make_buckets(int(bucket_bytes))

    # ---- all-reduce overlapped with backward -------------------------------------------------
    # With `bucket_bytes`, the flat buffer is cut into buckets of whole parameters, last parameter
    # first (backward produces the last layers' gradients first).  A post-accumulate hook on each
    # parameter counts its bucket down; a bucket whose gradients are all in is all-reduced at once,
    # asynchronously on NCCL's stream, while backward continues with the layers below.  Buckets go
    # out strictly in bucket order (a ready bucket waits for the ones before it), so every rank
    # issues the same collectives in the same order; `average()` sends the rest and waits.
    def _make_buckets(self, bucket_bytes):
        offs, off = [], 0
        for p in self.params:
            offs.append(off)
            off += p.numel()
        esize = self.flat.element_size()
        buckets, cur, cur_bytes = [], [], 0
        for i in reversed(range(len(self.params))):
            cur.append(i)
            cur_bytes += self.params[i].numel() * esize
            if cur_bytes >= bucket_bytes:
                buckets.append(cur)
                cur, cur_bytes = [], 0
        if cur:
            buckets.append(cur)
        self.buckets = []
        self.bucket_of = {}
        for b, idx in enumerate(buckets):
            lo = min(offs[i] for i in idx)
            hi = max(offs[i] + self.params[i].numel() for i in idx)
            self.buckets.append((lo, hi, len(idx)))
            for i in idx:
                self.bucket_of[i] = b
        self._reset_buckets()
        for i, p in enumerate(self.params):
            p.register_post_accumulate_grad_hook(lambda _p, i=i: self._grad_ready(i))

    def _reset_buckets(self):
        self.pending = [n for _, _, n in self.buckets]
        self.handles = []
        self.next_bucket = 0

    def _launch_ready(self, force=False):
        while self.next_bucket < len(self.buckets) and (force or self.pending[self.next_bucket] == 0):
            lo, hi, _ = self.buckets[self.next_bucket]
            self.handles.append(dist.all_reduce(self.flat[lo:hi], op=dist.ReduceOp.SUM, group=self.group,
                                                async_op=True))
            self.next_bucket += 1

    def _grad_ready(self, i):
        if not self.bound:
            return
        b = self.bucket_of[i]
        self.pending[b] -= 1
        if self.pending[b] == 0:
            self._launch_ready()

    def _bind(self):
        off = 0
        for p in self.params:
            p.grad = self.flat[off:off + p.numel()].view_as(p)
            off += p.numel()
        self.bound = True

    def zero(self, set_to_none: bool = False):
        if set_to_none:
            for p in self.params:
                p.grad = None
            self.bound = False
            return
        if not self.bound:
            self._bind()
        self.flat.zero_()
        if self.buckets is not None:
            self._reset_buckets()

    def average(self, world_size: int, group=None):
        if world_size <= 1:
            return
        if self.buckets is not None and self.bound:
            self._launch_ready(force=True)     # buckets with unused parameters go now, in order
            for h in self.handles:
                h.wait()
            self.flat.div_(world_size)
            self._reset_buckets()
            return
        self.flat.div_(world_size)
        dist.all_reduce(self.flat, op=dist.ReduceOp.SUM, group=group)


def _window_features(feature, idx_i, dup_index_i, dup_cache, device, staging=None):
    n_dup = int(dup_index_i.numel())
    rest = idx_i[n_dup:]
    if feature.device == torch.device(device) or feature.is_cuda:
        x = feature[rest.to(feature.device)].to(device)
    else:
        host = feature[rest]
        if staging is not None:
            buf = staging(host.shape, host.dtype)
            buf.copy_(host)
            x = buf.to(device, non_blocking=True)
        else:
            x = host.to(device)
    if n_dup > 0:
        x = torch.cat([dup_cache[dup_index_i], x], dim=0)
    return x


def train_epoch(args, model, local_partition_ids, local_partitions, feature, y, optimizer, lr_scheduler,
                world_size, split_idx, device, epoch, structInfo, grads: FlatGradients | None = None,
                group=None):
    model.train()
    edges = structInfo.local_sub_edge_index_for_partition_results
    dup_idx = structInfo.local_dup_indices
    dup_cache = structInfo.local_dup_nodes_per_partition_feature
    masks = getattr(structInfo, "local_train_masks", None) or []
    use_cache = bool(getattr(args, "use_cache", 1))
    if grads is None:
        # with several ranks, 4 MiB buckets are all-reduced while backward is still running
        grads = FlatGradients(model, bucket_bytes=4 << 20 if world_size > 1 else None, group=group)
    local_count = len(local_partitions)
    max_steps = local_count
    if world_size > 1:
        t = torch.tensor([local_count], device=device, dtype=torch.long)
        dist.all_reduce(t, op=dist.ReduceOp.MAX, group=group)
        max_steps = int(t.item())
    device = torch.device(device)
    y_dev = y.to(device)
    on_gpu = device.type == "cuda"
    staging = _PinnedStaging() if (on_gpu and not feature.is_cuda) else None
    if on_gpu:
        ev_start = torch.cuda.Event(enable_timing=True)
        ev_end = torch.cuda.Event(enable_timing=True)
        ev_start.record()
    else:
        t0 = time.perf_counter()
    losses, scores_by_pid = [], {}
    for i in range(max_steps):
        grads.zero(set_to_none=world_size == 1)
        if i < local_count:
            pid = local_partition_ids[i]
            idx_i = local_partitions[i]
            di = dup_idx[i] if use_cache and dup_idx else idx_i.new_empty(0)
            x_i = _window_features(feature, idx_i, di, dup_cache, device, staging)
            out_i, _, score_spe, _ = model(x_i, None, edges[i], None, None, None, None,
                                           attn_type=getattr(args, "attn_type", "sparse"))
            scores_by_pid[pid] = score_spe[-1]
            idx_dev = idx_i.to(device)
            mask = masks[i] if masks else torch.isin(idx_dev, split_idx["train"].to(device))
            loss_all = F.nll_loss(out_i, y_dev[idx_dev].long(), reduction="none")
            # mean over the window's train nodes (0 when it has none, as `build_zero_loss` gives),
            # written without boolean indexing so no step waits on the host
            m = mask.to(loss_all.dtype)
            loss = (loss_all * m).sum() / m.sum().clamp_min(1.0)
            losses.append(loss.detach())
            with overlap_weight_grads(world_size == 1):   # gradients are handed over, not added (set_to_none)
                loss.backward()
        grads.average(world_size, group)
        optimizer.step()
    lr_scheduler.step()
    if on_gpu:
        ev_end.record()
        ev_end.synchronize()
        elapsed = ev_start.elapsed_time(ev_end) / 1e3
    else:
        elapsed = time.perf_counter() - t0
    loss_mean = float(torch.stack(losses).mean()) if losses else 0.0
    stats = {"epoch_train_total_time": elapsed, "num_processed_windows": local_count,
             "max_window_steps": max_steps}
    return loss_mean, scores_by_pid, None, stats


class _PinnedStaging:
    """Reusable pinned host buffers for host-resident feature matrices."""

    def __init__(self):
        self._bufs = {}

    def __call__(self, shape, dtype):
        key = (tuple(shape), dtype)
        if key not in self._bufs:
            self._bufs[key] = torch.empty(shape, dtype=dtype, pin_memory=True)
        return self._bufs[key]


class GraphedWindowTrainer:
    """An epoch of `train_epoch` as replays of captured CUDA graphs, one per local window.

    Each graph holds the whole window step: feature gather, forward, masked NLL, backward into
    the flat gradient buffer, the gradient average over ranks (NCCL all-reduce) and the
    optimizer step.  A rank with fewer windows replays a zero-gradient step graph, so every
    rank issues the same all-reduces in the same order (`train_eval.py:211-217`).  Shapes and
    edge lists of the windows are fixed (`use_cache == 1`), which is what makes one capture per
    window reusable for every epoch; the launch overhead of the eager loop (hundreds of small
    kernels per window) collapses into one graph launch per window.

    Requirements: device-resident features and labels, an optimizer built with
    `capturable=True`, and a learning rate that changes (if at all) as a tensor in place.
    """

    def __init__(self, args, model, structInfo, feature, y, optimizer, world_size, device, group=None,
                 split_idx=None):
        device = torch.device(device)
        if not feature.is_cuda or not y.is_cuda:
            raise ValueError("graph replay needs device-resident features and labels")
        for g in optimizer.param_groups:
            if not g.get("capturable", False):
                raise ValueError("graph replay needs an optimizer created with capturable=True")
        self.model, self.opt, self.world, self.group, self.dev = model, optimizer, world_size, group, device
        self.attn_type = getattr(args, "attn_type", "sparse")
        self.grads = FlatGradients(model)
        self.edges = structInfo.local_sub_edge_index_for_partition_results
        self.ids = structInfo.local_partition_ids
        parts = structInfo.local_partitions
        masks = getattr(structInfo, "local_train_masks", None) or []
        dups = structInfo.local_dup_indices or [None] * len(parts)
        dup_cache = structInfo.local_dup_nodes_per_partition_feature
        self.windows = []
        for i, idx in enumerate(parts):
            idx_dev = idx.to(device)
            n_dup = int(dups[i].numel()) if dups[i] is not None else 0
            mask = masks[i] if masks else torch.isin(idx_dev, split_idx["train"].to(device))
            self.windows.append(dict(rest=idx_dev[n_dup:], dup=dups[i] if n_dup else None, y=y[idx_dev].long(),
                                     m=mask.to(torch.float32)))
        self.feature, self.dup_cache = feature, dup_cache
        self.max_steps = len(parts)
        if world_size > 1:
            t = torch.tensor([len(parts)], device=device, dtype=torch.long)
            dist.all_reduce(t, op=dist.ReduceOp.MAX, group=group)
            self.max_steps = int(t.item())
        self._capture()

    def _step(self, i):
        self.grads.zero(set_to_none=self.world == 1)
        loss = None
        scores = None
        if i is not None:
            w = self.windows[i]
            x = self.feature[w["rest"]]
            if w["dup"] is not None:
                x = torch.cat([self.dup_cache[w["dup"]], x], dim=0)
            out, _, score_spe, _ = self.model(x, None, self.edges[i], None, None, None, None, attn_type=self.attn_type)
            loss_all = F.nll_loss(out, w["y"], reduction="none")
            loss = (loss_all * w["m"]).sum() / w["m"].sum().clamp_min(1.0)
            with overlap_weight_grads(self.world == 1):
                loss.backward()
            scores = score_spe[-1]
        self.grads.average(self.world, self.group)
        self.opt.step()
        return loss, scores

    def _capture(self):
        self.model.train()
        side = torch.cuda.Stream(self.dev)
        side.wait_stream(torch.cuda.current_stream(self.dev))
        with torch.cuda.stream(side):        # warm-up: CSR caches, allocator, NCCL, optimizer state
            for i in range(len(self.windows)):
                self._step(i)
            if self.max_steps > len(self.windows):
                self._step(None)
        torch.cuda.current_stream(self.dev).wait_stream(side)
        torch.cuda.synchronize(self.dev)
        self.pool = torch.cuda.graph_pool_handle()
        self.graphs, self.outputs = [], []
        for i in range(len(self.windows)):
            g = torch.cuda.CUDAGraph()
            with torch.cuda.graph(g, pool=self.pool):
                out = self._step(i)
            self.graphs.append(g)
            self.outputs.append(out)
        self.dummy = None
        if self.max_steps > len(self.windows):
            self.dummy = torch.cuda.CUDAGraph()
            with torch.cuda.graph(self.dummy, pool=self.pool):
                self._step(None)
        torch.cuda.synchronize(self.dev)

    def run_epoch(self, lr_scheduler=None):
        """Returns (loss_mean, scores_by_pid, elapsed seconds by CUDA events)."""
        start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        start.record()
        for i in range(self.max_steps):
            if i < len(self.graphs):
                self.graphs[i].replay()
            else:
                self.dummy.replay()
        if lr_scheduler is not None:
            lr_scheduler.step()
        end.record()
        end.synchronize()
        losses = [o[0] for o in self.outputs]
        loss_mean = float(torch.stack(losses).mean()) if losses else 0.0
        scores = {pid: o[1] for pid, o in zip(self.ids, self.outputs)}
        return loss_mean, scores, start.elapsed_time(end) / 1e3
