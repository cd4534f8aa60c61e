#!/usr/bin/env python
"""Benchmark of the NeutronGT hot path on B200.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]

Headline (`value`): graph-sparse window attention, forward + backward, in edges/s, on the
isolated-kernel workload: one 65,536-token window per GPU, in-degree ~ Poisson(32) with uniform
sources (E ~ 2.09M), 8 heads x head_dim 16, bf16, inputs resident in HBM, L2 flushed (256 MiB
write) between steps.  A step is one fwd+bwd of the rank's window; with N GPUs each rank owns its
own window (weak scaling) and value = all ranks' edges x K / the slowest rank's device time.

The same JSON line carries:
  e2e          the same metric through the public API (`sparse_attention_bias` + autograd)
               with pinned host buffers: inputs copied in and outputs/grads copied out
               every step, CSR build included;
  roofline     the dominant kernel (backward) against the measured HBM copy bandwidth, plus an
               `l2` object against an L2 copy bandwidth measured in this run;
  cpu_baseline the reference algorithm on the host cores (CPU restatement), bounded sample;
  gt_epoch     GT (4 layers, hidden 128, 8 heads, fp32) epochs on the 169,343-node graph, windows
               built by the preprocessing pipeline (PPR, adjacency, 5 % halo merge, duplicate-first
               order); the seeded random windows without halos as a second figure;
  dense        GPH_Large dense windows (32,768 tokens, head_dim 24, bf16): the per-rank attention
               share, and one whole GPH_Large encoder layer (bf16 projections on the tensor cores,
               dense attention over 32 heads, FFN) forward + backward;
  ppr          APPNP PPR + top-k over every seed of the 169,343-node graph (seed ranges balanced
               by degree across ranks), push PPR (eps 1e-4, top-10) on the 232,965-node graph with
               114.6 M directed edges, APPNP top-4 on the 2,449,029-node graph with 123.7 M
               directed edges, and `csr_spgemm` on the APPNP product (PPR state x D^-1 A);
  clocks       nvidia-smi samples taken during the timed region.

`--impl reference` times the reference's CPU algorithm for the same metric instead
(rank 0 only).
"""
from __future__ import annotations

import argparse
import datetime
import json
import math
import os
import statistics
import subprocess
import sys
import tempfile
import time
from types import SimpleNamespace

import torch

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, ROOT)

N_TOKENS = 65536
MEAN_DEG = 32.0
HEADS = 8
HEAD_DIM = 16
L2_FLUSH_BYTES = 256 << 20
FALLBACK_HBM_GBS = 6650.0


def parse_args():
    p = argparse.ArgumentParser()
    p.add_argument("--gpus", type=int, default=1)
    p.add_argument("--steps", type=int, default=20)
    p.add_argument("--warmup", type=int, default=5)
    p.add_argument("--impl", choices=["ours", "reference"], default="ours")
    p.add_argument("--skip-ppr", action="store_true")
    p.add_argument("--skip-epoch", action="store_true")
    p.add_argument("--skip-dense", action="store_true")
    p.add_argument("--skip-cpu", action="store_true")
    p.add_argument("--skip-layer", action="store_true")
    p.add_argument("--skip-large-ppr", action="store_true",
                   help="skip the PPR runs on the 232,965- and 2,449,029-node graphs")
    p.add_argument("--profile-case", choices=["spattn", "gemm", "push", "dense"], default=None,
                   help="run one small workload for an ncu capture (no JSON line): the 65,536-token window "
                        "fwd+bwd x3 with L2 flushes, the bf16 Linear 32768x768->768 fwd+bwd x3, or push PPR "
                        "(eps 1e-5) on a 40,000-node graph x2")
    p.add_argument("--linear-calls", action="store_true",
                   help="print the per-call device time of the fp32 Linear entry points at the config-2 "
                        "window shape (14,252 rows; CUDA-graph replay of 20 back-to-back calls) instead "
                        "of the JSON line")
    p.add_argument("--epoch-kernels", action="store_true",
                   help="print the per-kernel device time of one graph-replayed config-2 GT epoch "
                        "(torch.profiler over CUPTI) instead of the JSON line")
    return p.parse_args()


# ------------------------------------------------------------------------------------
# distributed plumbing
# ------------------------------------------------------------------------------------
def dist_setup():
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    if world > 1:
        import torch.distributed as dist
        torch.cuda.set_device(local)
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=300),
                                device_id=torch.device("cuda", local))
    elif torch.cuda.is_available():
        torch.cuda.set_device(local)
    return rank, world, local


def barrier(world):
    if world > 1:
        import torch.distributed as dist
        dist.barrier()
    torch.cuda.synchronize()


def allreduce_max(x: float, world: int) -> float:
    if world == 1:
        return x
    import torch.distributed as dist
    t = torch.tensor([x], dtype=torch.float64, device="cuda")
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return float(t.item())


def allreduce_sum(x: float, world: int) -> float:
    if world == 1:
        return x
    import torch.distributed as dist
    t = torch.tensor([x], dtype=torch.float64, device="cuda")
    dist.all_reduce(t, op=dist.ReduceOp.SUM)
    return float(t.item())


# ------------------------------------------------------------------------------------
# clocks during the timed region
# ------------------------------------------------------------------------------------
class ClockSampler:
    FIELDS = ("clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,clocks_event_reasons.hw_slowdown,"
              "clocks_event_reasons.hw_thermal_slowdown,clocks_event_reasons.sw_thermal_slowdown,"
              "clocks_event_reasons.sw_power_cap")

    def __init__(self, device_index: int):
        self.proc = None
        self.path = None
        try:
            uuid = str(torch.cuda.get_device_properties(device_index).uuid)
            self.target = uuid if uuid.startswith("GPU-") else f"GPU-{uuid}"
        except Exception:
            self.target = str(device_index)

    def start(self):
        fd, self.path = tempfile.mkstemp(suffix=".csv")
        os.close(fd)
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", "-i", self.target, f"--query-gpu={self.FIELDS}", "--format=csv,noheader,nounits",
                 "-lms", "100"], stdout=open(self.path, "w"), stderr=subprocess.DEVNULL)
        except Exception:
            self.proc = None
        time.sleep(0.3)

    def stop(self):
        if self.proc is None:
            return None
        self.proc.terminate()
        try:
            self.proc.wait(timeout=5)
        except Exception:
            self.proc.kill()
        rows = []
        for line in open(self.path):
            parts = [x.strip() for x in line.split(",")]
            if len(parts) < 8:
                continue
            try:
                rows.append((float(parts[0]), float(parts[1]), parts[4:8]))
            except ValueError:
                continue
        os.unlink(self.path)
        if not rows:
            return None
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        reasons = sorted({names[i] for _, _, r in rows for i, v in enumerate(r) if v.lower().startswith("active")})
        return {"sm_mhz": statistics.median(r[0] for r in rows), "sm_max_mhz": max(r[1] for r in rows),
                "reasons": reasons, "samples": len(rows)}


def measured_hbm_peak():
    path = os.path.join(ROOT, "MEASURED_PEAKS.json")
    try:
        with open(path) as f:
            return float(json.load(f)["hbm_gbs"]), "measured"
    except Exception:
        return FALLBACK_HBM_GBS, "fallback"


def ncu_traffic():
    """Per-launch DRAM bytes from the committed ncu summary (null when absent)."""
    path = os.path.join(ROOT, "profiles", "ncu_traffic.json")
    try:
        with open(path) as f:
            return json.load(f)
    except Exception:
        return {}


# ------------------------------------------------------------------------------------
# workload: the isolated-kernel window
# ------------------------------------------------------------------------------------
def make_window(seed: int):
    from neutrongt_b200 import synthetic
    rowptr, col = synthetic.poisson_window_csr(N_TOKENS, MEAN_DEG, seed=seed)
    ei = synthetic.edge_index_from_dst_csr(rowptr, col)
    g = torch.Generator().manual_seed(1000 + seed)
    shape = (N_TOKENS, HEADS, HEAD_DIM)
    q, k, v, dout = (torch.randn(shape, generator=g).to(torch.bfloat16) for _ in range(4))
    return q, k, v, dout, ei


def algorithmic_bytes(n, e, heads=HEADS, dim=HEAD_DIM, elt=2, idx=4):
    row = heads * dim * elt
    fwd = e * (2 * row + idx) + n * (2 * row + 4 + 4 * heads + 4)
    bwd = e * (4 * row + 2 * 4 * heads + 2 * idx) + n * (8 * row + 8 + 8 * heads)
    return fwd, bwd


def cpu_baseline_sample(q, k, v, dout, ei, rows=16384, repeats=3):
    """The reference algorithm (torch gathers + index_add scatters, fp32) on the host cores."""
    from oracle import attention as oatt
    threads = os.cpu_count() or 1
    torch.set_num_threads(threads)
    keep = ei[1] < rows
    sub = ei[:, keep]
    qf, kf, vf, gf = (t.float() for t in (q, k, v, dout))
    times = []
    for _ in range(repeats):
        t0 = time.perf_counter()
        oatt.sparse_attention_forward(qf, kf, vf, sub)
        oatt.sparse_attention_backward(qf, kf, vf, sub, gf)
        times.append(time.perf_counter() - t0)
    t = statistics.median(times)
    return {"value": sub.shape[1] / t, "unit": "edges/s", "cores": threads, "kind": "port",
            "sample": f"fwd+bwd of the {rows} lowest destination rows of the window ({sub.shape[1]} edges), "
                      f"fp32, median of {repeats}; oracle/attention.py restates "
                      "models/gt_dist_node_level_single_window.py:112-179 with the same torch ops"}


# ------------------------------------------------------------------------------------
# our implementation
# ------------------------------------------------------------------------------------
def bench_attention(args, rank, world, dev):
    from neutrongt_b200 import sparse_attention_bias
    from neutrongt_b200.attention import WindowAttentionBuffers
    from neutrongt_b200.edge_csr import build_edge_csr

    q_h, k_h, v_h, g_h, ei_h = make_window(seed=rank)
    n, e = N_TOKENS, ei_h.shape[1]
    q, k, v, dout, ei = (t.to(dev) for t in (q_h, k_h, v_h, g_h, ei_h))
    csr = build_edge_csr(ei, n)
    buf = WindowAttentionBuffers(q, k, v, csr)
    flush = torch.empty(L2_FLUSH_BYTES, dtype=torch.uint8, device=dev)
    st = torch.cuda.current_stream(dev)

    for _ in range(args.warmup):
        buf.forward()
        buf.backward(dout)
        flush.fill_(1)
    barrier(world)
    ev = [[torch.cuda.Event(enable_timing=True) for _ in range(3)] for _ in range(args.steps)]
    sampler = ClockSampler(dev.index)
    sampler.start()
    barrier(world)
    for i in range(args.steps):
        flush.fill_(i & 255)
        ev[i][0].record(st)
        buf.forward()
        ev[i][1].record(st)
        buf.backward(dout)
        ev[i][2].record(st)
    barrier(world)
    clocks = sampler.stop()
    t_fwd = sum(a.elapsed_time(b) for a, b, _ in ev) / 1e3
    t_bwd = sum(b.elapsed_time(c) for _, b, c in ev) / 1e3
    t_rank = t_fwd + t_bwd
    t_max = allreduce_max(t_rank, world)
    edges_all = allreduce_sum(float(e), world)
    value = edges_all * args.steps / t_max

    fwd_bytes, bwd_bytes = algorithmic_bytes(n, e)
    peak, peak_kind = measured_hbm_peak()
    avg_fwd, avg_bwd = t_fwd / args.steps, t_bwd / args.steps
    traffic = ncu_traffic()
    dom = "bwd" if avg_bwd >= avg_fwd else "fwd"
    achieved = (bwd_bytes / avg_bwd if dom == "bwd" else fwd_bytes / avg_fwd) / 1e9
    roofline = {"bound": "hbm", "kernel": "spattn_delta_vec+spattn_bwd_r128" if dom == "bwd" else "spattn_fwd_r128",
                "achieved": achieved, "peak": peak, "peak_kind": f"{peak_kind} hbm_gbs (burst)", "unit": "GB/s",
                "frac": achieved / peak, "traffic": traffic.get(dom),
                "algorithmic_bytes_per_launch": bwd_bytes if dom == "bwd" else fwd_bytes,
                "fwd": {"ms": avg_fwd * 1e3, "achieved": fwd_bytes / avg_fwd / 1e9, "frac": fwd_bytes / avg_fwd / 1e9 / peak,
                        "traffic": traffic.get("fwd")},
                "bwd": {"ms": avg_bwd * 1e3, "achieved": bwd_bytes / avg_bwd / 1e9, "frac": bwd_bytes / avg_bwd / 1e9 / peak,
                        "traffic": traffic.get("bwd")},
                "l2": None,
                "compulsory_bytes": {"fwd": 4 * n * HEADS * HEAD_DIM * 2 + 4 * (n + 1 + e) + 4 * n * HEADS + 4 * n,
                                     "note": "Q,K,V,O once + CSR + Z + node scores; K/V (33.5 MB) can stay in L2, "
                                             "so the no-reuse algorithmic bytes and these bracket the DRAM traffic"}}

    # L2-side rooflines, from the committed one-kernel ncu captures of these launches
    # (profiles/ncu_traffic.json): each launch's L2 traffic (lts__t_sectors x 32 B) over the time
    # measured here, against the L2 sustained peak the capture implies (its sectors over its
    # duration, divided by its lts__throughput percentage)
    def l2_roofline(key, avg):
        lts, pct, ncu_us = traffic.get(f"{key}_lts"), traffic.get(f"{key}_lts_pct"), traffic.get(f"{key}_ncu_us")
        achieved = lts / avg / 1e9 if lts else None
        l2_peak = lts / (ncu_us * 1e-6) / (pct / 100.0) / 1e9 if (lts and pct and ncu_us) else None
        return {"traffic": lts, "achieved": achieved, "unit": "GB/s", "peak": l2_peak,
                "frac": achieved / l2_peak if l2_peak else None,
                "peak_kind": "L2 sustained peak implied by the committed capture (profiles/spattn_r128_config3.md)"}

    roofline["l2"] = l2_roofline(dom, avg_bwd if dom == "bwd" else avg_fwd)
    roofline["fwd"]["l2"] = l2_roofline("fwd", avg_fwd)
    roofline["bwd"]["l2"] = l2_roofline("bwd", avg_bwd)

    # e2e through the public API with pinned host buffers.  Every step copies its own inputs in and
    # its results out.  Pipelined: one stream per engine — host-to-device copies, the API call, and
    # device-to-host copies — joined by events, with the inputs of steps i + 1 and i + 2 in flight
    # while step i runs, so the two copy directions (full duplex) and the kernels overlap and the
    # host's wait inside the call (the edge-list validation) never holds back the next input copy.
    # The same steps one after another on one stream are reported beside it.
    pins = [t.pin_memory() for t in (q_h, k_h, v_h, g_h, ei_h)]
    outs = [[torch.empty((n, HEADS, HEAD_DIM), dtype=torch.bfloat16).pin_memory() for _ in range(4)]
            for _ in range(2)]
    ns_h = [torch.empty(n, dtype=torch.float32).pin_memory() for _ in range(2)]
    s_in, s_comp, s_out = torch.cuda.Stream(dev), torch.cuda.Stream(dev), torch.cuda.Stream(dev)
    staged = {}

    def e2e_copy_in(i, s):
        with torch.cuda.stream(s):
            staged[i] = ([t.to(dev, non_blocking=True) for t in pins], torch.cuda.Event())
            staged[i][1].record(s)

    def e2e_compute(i, s, s_copy_out):
        tensors, ready = staged.pop(i)
        with torch.cuda.stream(s):
            s.wait_event(ready)
            for t in tensors:
                t.record_stream(s)
            qd, kd, vd, gd, eid = tensors
            qd.requires_grad_(True)
            kd.requires_grad_(True)
            vd.requires_grad_(True)
            x, ns = sparse_attention_bias(qd, kd, vd, eid, None)
            x.backward(gd)
            results = (x.detach(), qd.grad, kd.grad, vd.grad, ns)
            done = torch.cuda.Event()
            done.record(s)
        with torch.cuda.stream(s_copy_out):
            s_copy_out.wait_event(done)
            for d in results:
                d.record_stream(s_copy_out)
            for h, d in zip(outs[i % 2], results[:4]):
                h.copy_(d, non_blocking=True)
            ns_h[i % 2][:ns.numel()].copy_(ns, non_blocking=True)

    def run_steps(count, streams):
        if len(streams) == 1:                       # one stream: copy in, call, copy out, in turn
            for i in range(count):
                e2e_copy_in(i, streams[0])
                e2e_compute(i, streams[0], streams[0])
            return
        s_i, s_c, s_o = streams
        for i in range(min(2, count)):
            e2e_copy_in(i, s_i)
        for i in range(count):
            e2e_compute(i, s_c, s_o)
            if i + 2 < count:
                e2e_copy_in(i + 2, s_i)

    def timed(streams):
        run_steps(max(2, args.warmup), streams)
        for s in streams:
            st.wait_stream(s)
        barrier(world)
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record(st)
        for s in streams:
            s.wait_stream(st)
        run_steps(args.steps, streams)
        for s in streams:
            st.wait_stream(s)
        e1.record(st)
        barrier(world)
        return allreduce_max(e0.elapsed_time(e1) / 1e3, world)

    t_serial = timed([st])
    t_e2e = timed([s_in, s_comp, s_out])
    h2d = sum(t.numel() * t.element_size() for t in pins)
    d2h = sum(t.numel() * t.element_size() for t in outs[0]) + 4 * (csr.node_scores_len)
    e2e = {"value": edges_all * args.steps / t_e2e, "unit": "edges/s", "h2d_bytes_per_step": h2d,
           "d2h_bytes_per_step": d2h, "ms_per_step": t_e2e / args.steps * 1e3,
           "serial_ms_per_step": t_serial / args.steps * 1e3,
           "serial_value": edges_all * args.steps / t_serial,
           "path": "neutrongt_b200.sparse_attention_bias + autograd backward, pinned host buffers, CSR built "
                   "from the copied edge_index every step; value: input copies, calls and output copies on "
                   "three streams joined by events, two steps' inputs in flight; serial_*: the same steps on "
                   "one stream"}
    return {"value": value, "ms_per_step": t_max / args.steps * 1e3, "edges": e, "roofline": roofline,
            "e2e": e2e, "clocks": clocks, "gpu_launches": 3 * args.steps,
            "host": (q_h, k_h, v_h, g_h, ei_h)}


_GRAPH = {}


def config2_graph():
    """The 169,343-node graph: Chung-Lu, 1,166,243 undirected edges (seed 0)."""
    if "g" not in _GRAPH:
        from neutrongt_b200 import synthetic
        _GRAPH["g"] = synthetic.chung_lu_graph(169343, 1166243, seed=0)
    return _GRAPH["g"]


PPR2 = dict(alpha=0.15, topk=8, num_iterations=20, iter_topk=8)


def config2_windows(dev, pct=5):
    """Windows as the reference's preprocessing builds them (rank 0 in the reference, every rank
    here): APPNP PPR top-8 of every node, the weighted PPR adjacency (build_adj_fromat), 16 seeded
    random parts (METIS is absent) each grown by its top 5 % PPR neighbours (the scripts'
    --related_nodes_topk_rate 5).  Cached per process."""
    if "windows" not in _GRAPH:
        from neutrongt_b200 import personal_pagerank_appnp, synthetic
        from neutrongt_b200.window import build_adj_format, merge_related_nodes
        rowptr, col = config2_graph()
        csr = {"rowptr": rowptr.to(dev), "col": col.to(dev)}
        ei, val = personal_pagerank_appnp(None, csr_data=csr, device=dev, **PPR2)
        adj, ew, _ = build_adj_format((ei, val), device=dev)
        parts = synthetic.random_partitions(169343, 16, seed=0)
        _GRAPH["windows"] = [merge_related_nodes(p, adj, ew, pct, device=dev).cpu() for p in parts]
    return _GRAPH["windows"]


def gt_model(dev):
    from neutrongt_b200.models import GT_SW
    torch.manual_seed(0)
    return GT_SW(n_layers=4, num_heads=8, input_dim=128, hidden_dim=128, output_dim=40, attn_bias_dim=1,
                 dropout_rate=0.3, input_dropout_rate=0.1, attention_dropout_rate=0.5, ffn_dim=128, num_global_node=1,
                 args=SimpleNamespace(struct_enc="False"), num_in_degree=0, num_out_degree=0, num_spatial=7,
                 num_edges=512, max_dist=5, edge_dim=64).to(dev)


def attention_time_per_epoch(ws, dev, heads=8, dim=16, layers=4, reps=3):
    """Device time of the sparse-attention kernels one epoch runs (every local window, every layer,
    forward + backward), timed on their own with the epoch's window shapes (fp32)."""
    from neutrongt_b200.attention import WindowAttentionBuffers
    from neutrongt_b200.edge_csr import edge_csr_for
    bufs = []
    for p, ei in zip(ws.local_partitions, ws.local_sub_edge_index_for_partition_results):
        n = int(p.numel())
        q, k, v, g = (torch.randn(n, heads, dim, device=dev) for _ in range(4))
        bufs.append((WindowAttentionBuffers(q, k, v, edge_csr_for(ei, n)), g))
    for b, g in bufs:
        b.forward()
        b.backward(g)
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record()
    for _ in range(reps):
        for b, g in bufs:
            for _ in range(layers):
                b.forward()
                b.backward(g)
    e1.record()
    e1.synchronize()
    return e0.elapsed_time(e1) / 1e3 / reps


def bench_gt_epoch(args, rank, world, dev, windows, label, warm=2, epochs=5, with_cpu=True):
    """GT (4 layers, hidden 128, 8 heads, fp32) training epochs over the given 16 windows."""
    from neutrongt_b200 import synthetic
    from neutrongt_b200.train import FlatGradients, build_window_state, train_epoch
    n = 169343
    rowptr, col = config2_graph()
    feature = synthetic.node_features(n, 128, seed=1)
    y = synthetic.node_labels(n, 40, seed=2)
    split = synthetic.split_idx(n, seed=3)
    model = gt_model(dev)
    grads = FlatGradients(model)
    opt = torch.optim.AdamW(model.parameters(), lr=1e-4, weight_decay=0.01, fused=True)
    sched = torch.optim.lr_scheduler.LambdaLR(opt, lambda e: 1.0)
    a = SimpleNamespace(use_cache=1, attn_type="sparse")
    feat_dev = feature.to(dev)
    ws = build_window_state(rowptr, col, windows, rank, world, feat_dev, dev, split)

    def run(feat, k):
        out = []
        for _ in range(k):
            barrier(world)
            loss, _, _, st = train_epoch(a, model, ws.local_partition_ids, ws.local_partitions, feat, y, opt, sched,
                                         world, split, dev, 0, ws, grads=grads)
            out.append((st["epoch_train_total_time"], loss))
        return out

    run(feat_dev, warm)
    timed = run(feat_dev, epochs)
    t_dev = allreduce_max(statistics.mean(t for t, _ in timed), world)
    # the same epochs replayed from one captured CUDA graph per window
    from neutrongt_b200.train import GraphedWindowTrainer
    gmodel = gt_model(dev)
    gopt = torch.optim.AdamW(gmodel.parameters(), lr=1e-4, weight_decay=0.01, fused=True, capturable=True)
    trainer = GraphedWindowTrainer(a, gmodel, ws, feat_dev, y.to(dev), gopt, world, dev, split_idx=split)
    for _ in range(warm):
        trainer.run_epoch()
    gt = []
    for _ in range(epochs):
        barrier(world)
        gt.append(trainer.run_epoch())
    t_graph = allreduce_max(statistics.mean(t for _, _, t in gt), world)
    trainer.graphs.clear()          # the graphs hold NCCL calls: release them before teardown
    trainer.dummy = None
    del trainer
    torch.cuda.synchronize()
    t_attn = allreduce_max(attention_time_per_epoch(ws, dev), world)
    e_local = sum(int(e.shape[1]) for e in ws.local_sub_edge_index_for_partition_results)
    n_local = sum(int(p.numel()) for p in ws.local_partitions)
    edges_epoch = allreduce_sum(float(e_local), world)
    out = {"workload": f"GT 4L/128/8H fp32 on the Chung-Lu 169,343-node / 1,166,243-edge graph, {label}; "
                       "features N(0,1) dim 128, 40 classes",
           "epoch_time_s": t_graph, "unit": "s", "higher_is_better": False,
           "epoch_time_eager_s": t_dev,
           "loss_graph_last_epoch": gt[-1][0],
           "scaling": "strong (16 windows split round-robin over ranks)",
           "loss_last_epoch": timed[-1][1], "windows": len(windows),
           "window_nodes_mean": n_local / max(1, len(ws.local_partitions)),
           "attention_edges_per_epoch": edges_epoch,
           "attention_kernels_s_per_epoch": t_attn,
           "attention_share": t_attn / t_graph if t_graph > 0 else None,
           # graph-sparse attention throughput on the 170K-node graph's windows: every layer's
           # forward + backward over the window edges, fp32, on the ranks' own windows
           "attention_edges_per_s": 4 * edges_epoch / t_attn if t_attn > 0 else None,
           "note": "epoch_time_s: one captured CUDA graph per window (gather, forward, loss, backward, gradient "
                   "all-reduce, AdamW) replayed per epoch; epoch_time_eager_s: the same loop eagerly; "
                   "attention_kernels_s_per_epoch: the epoch's sparse-attention launches (4 layers x windows, "
                   "fwd+bwd) timed alone; attention_edges_per_s: 4 layers x attention_edges_per_epoch over that "
                   "time (fp32 fwd+bwd)"}
    if with_cpu:
        run(feature, 1)
        timed_h = run(feature, epochs)
        out["epoch_time_host_features_s"] = allreduce_max(statistics.mean(t for t, _ in timed_h), world)
    if with_cpu and rank == 0 and not args.skip_cpu:
        out["cpu_baseline"] = gt_epoch_cpu_baseline(model, ws, feature, y, split, len(windows))
    return out


def gt_epoch_cpu_baseline(model_gpu, ws, feature, y, split, n_windows, sample=2):
    """The same GT model and loop on the host cores, attention = the reference algorithm restated
    on the CPU (oracle/attention.py, differentiable torch ops); epoch time from a window sample."""
    import copy
    import torch.nn.functional as F
    from oracle import attention as oatt
    threads = os.cpu_count() or 1
    torch.set_num_threads(threads)
    model = copy.deepcopy(model_gpu).cpu()

    def attn(q, k, v, ei, bias):
        x, ns, _, _ = oatt.sparse_attention_forward(q, k, v, ei, bias)
        return x, ns

    for layer in model.layers:
        layer.self_attention.local_attn.sparse_attention_bias = attn
    opt = torch.optim.AdamW(model.parameters(), lr=1e-4, weight_decay=0.01)
    train = split["train"]
    times = []
    for i in range(min(sample, len(ws.local_partitions))):
        idx = ws.local_partitions[i]
        ei = ws.local_sub_edge_index_for_partition_results[i].cpu()
        t0 = time.perf_counter()
        out, _, _, _ = model(feature[idx], None, ei, None, None, None, None, attn_type="sparse")
        mask = torch.isin(idx, train)
        loss = F.nll_loss(out, y[idx], reduction="none")[mask].mean()
        opt.zero_grad(set_to_none=True)
        loss.backward()
        opt.step()
        times.append(time.perf_counter() - t0)
    per_window = statistics.mean(times)
    return {"value": per_window * n_windows, "unit": "s per epoch (window sample x windows)", "cores": threads,
            "kind": "port", "sample": f"{len(times)} windows fwd+bwd+AdamW on the host, scaled to {n_windows} windows"}


def measured_bf16_peak(sustained=False):
    path = os.path.join(ROOT, "MEASURED_PEAKS.json")
    try:
        with open(path) as f:
            return float(json.load(f)["bf16_tflops_sustained" if sustained else "bf16_tflops"]), "measured"
    except Exception:
        return (1400.0 if sustained else 1590.0), "fallback"


def bench_dense(args, rank, world, dev, steps=5, warm=2):
    """GPH_Large dense attention windows, per-rank share: S = 32,768 tokens of one window,
    the rank's 4 of 32 heads after the Ulysses exchange (head_dim 24), bf16, fwd + bwd.  With N > 1
    the step is the reference's `DistributedAttentionNodeLevel` layer: the exchange (NCCL
    all_to_all_single) of q, k, v and the output is inside the timed step.  It is timed as the
    reference runs it (one exchange per tensor) and pipelined in two head chunks (NCCL overlapping
    the kernels); both times are reported and `ms_per_step` is the faster."""
    import math as _m
    from neutrongt_b200.dense_attention import dense_attention
    S, H_total, D = 32768, 32, 24
    H_local = 4
    g = torch.Generator(device=dev).manual_seed(rank)
    if world == 1:
        q, k, v, dy = (torch.randn(S, H_local, D, generator=g, device=dev).to(torch.bfloat16) * 0.5 for _ in range(4))
    else:
        # per-rank sequence shard of the heads the exchange distributes: world * 4 heads in total
        q, k, v, dy = (torch.randn(1, S // world, H_local * world, D, generator=g, device=dev).to(torch.bfloat16) * 0.5
                       for _ in range(4))
    qd, kd, vd = (t.requires_grad_(True) for t in (q, k, v))
    grp = None
    import torch.distributed as _dist
    if world > 1:
        grp = _dist.group.WORLD

    layers = {}
    if world > 1:   # the reference's layer; also with the head exchange pipelined in two chunks
        from neutrongt_b200 import CoreAttention
        from neutrongt_b200.ulysses import DistributedAttentionNodeLevel
        for chunks in (1, 2):
            layers[chunks] = DistributedAttentionNodeLevel(CoreAttention(H_total * D, 0.0, H_total), grp,
                                                           head_chunks=chunks).train()

    def step(chunks):
        if world == 1:
            x, _ = dense_attention(qd, kd, vd, _m.sqrt(D), score_heads=H_total, check_status=False)
            x.backward(dy)
        else:
            y, _ = layers[chunks](qd, kd, vd, None, None, "full")
            y.backward(dy.reshape(y.shape))

    def timed(chunks):
        for _ in range(warm):
            step(chunks)
        barrier(world)
        ev = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)) for _ in range(steps)]
        for a, b in ev:
            a.record()
            step(chunks)
            b.record()
        barrier(world)
        return allreduce_max(sum(a.elapsed_time(b) for a, b in ev) / steps / 1e3, world)

    per_chunks = {c: timed(c) for c in ((1, 2) if world > 1 else (1,))}
    best = min(per_chunks, key=per_chunks.get)
    t = per_chunks[best]
    fwd_flops = 4.0 * S * S * H_local * D
    flops = fwd_flops * 3.5            # forward + backward (recompute S, dP, dV, dK, dQ)
    peak, kind = measured_bf16_peak()
    achieved = flops / t / 1e12
    return {"workload": "GPH_Large dense window, per-rank share: one window of 32,768 tokens, 4 heads of 32 "
                        "(after the Ulysses exchange), head_dim 24, bf16, dense attention fwd+bwd",
            "ms_per_step": t * 1e3, "tflops_algorithmic": achieved,
            "roofline": {"bound": "tensor", "achieved": achieved, "peak": peak,
                         "peak_kind": f"{kind} bf16_tflops (burst)", "unit": "TFLOP/s", "frac": achieved / peak,
                         "note": "algorithmic flops 3.5 x 4 S^2 H D; head_dim 24 runs padded to 32 in the MMAs, "
                                 "and the S^2 exponentials (MUFU) bound this shape before the tensor pipe"},
            "n_gpus": world, "ulysses": world > 1,
            "ulysses_head_chunks": best if world > 1 else None,
            "ms_per_step_by_head_chunks": {str(c): v * 1e3 for c, v in per_chunks.items()} if world > 1 else None}


def balanced_ranges(weights, world):
    """Contiguous seed ranges [s_r, s_{r+1}) cut at equal prefix sums of a per-seed cost, so ranks get
    equal work while the concatenation in rank order keeps the seeds ascending (the gathered output
    is the single-rank output, bit for bit)."""
    c = torch.cumsum(weights.double(), 0)
    total = float(c[-1])
    cuts = [0] + [int(torch.searchsorted(c, total * r / world).item()) for r in range(1, world)] + [weights.numel()]
    return [(cuts[r], max(cuts[r], cuts[r + 1])) for r in range(world)]


def _timed_call(fn, world):
    barrier(world)
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record()
    out = fn()
    e1.record()
    barrier(world)
    return out, allreduce_max(e0.elapsed_time(e1) / 1e3, world)


def bench_ppr(args, rank, world, dev):
    """APPNP PPR + top-8 over every seed of the 169,343-node graph (seeds sharded over ranks in
    degree-balanced contiguous ranges)."""
    from neutrongt_b200 import personal_pagerank_appnp
    rowptr, col = config2_graph()
    n = 169343
    deg = (rowptr[1:] - rowptr[:-1]).to(torch.float64)
    s0, s1 = balanced_ranges(deg + 8.0, world)[rank]
    csr = {"rowptr": rowptr.to(dev), "col": col.to(dev)}
    personal_pagerank_appnp(None, csr_data=csr, device=dev, source_start=s0, source_end=min(s1, s0 + 2000), **PPR2)
    (ei, val), t = _timed_call(lambda: personal_pagerank_appnp(None, csr_data=csr, device=dev, source_start=s0,
                                                                source_end=s1, **PPR2), world)
    out = {"workload": "169,343-node Chung-Lu graph (2,332,486 directed edges), every node a seed, "
                       "alpha 0.15, 20 iterations, top-k 8 per iteration and at the end",
           "seeds_per_s": n / t, "seconds": t, "entries": int(allreduce_sum(float(ei.shape[1]), world)),
           "scaling": "strong (seeds split into contiguous ranges of equal degree + 8 sums per rank)"}
    if rank == 0 and world == 1:
        out["window_build"] = bench_window_build(args, dev, ei, val)
    if rank == 0 and not args.skip_cpu:
        from oracle import ppr as oppr
        threads = os.cpu_count() or 1
        sample = 3000
        st = {}
        t0 = time.perf_counter()
        oppr.personal_pagerank_appnp(None, csr_data={"rowptr": rowptr, "col": col}, source_start=0,
                                     source_end=sample, nthreads=threads, stats=st, **PPR2)
        tc = time.perf_counter() - t0
        out["cpu_baseline"] = {"value": sample / tc, "unit": "seeds/s", "cores": threads, "kind": "port",
                               "sample": f"seeds 0..{sample - 1}, canonical fp64 restatement in C (oracle/appnp_oracle.c)"}
        touched = st["edges_touched"] / sample
        out["adjacency_entries_per_seed"] = touched
        out["achieved_gbs_adjacency_model"] = touched * n * 4 / t / 1e9
    out["spgemm"] = bench_spgemm(args, rank, world, dev, rowptr, col, ei, val, s0, s1)
    return out


def bench_spgemm(args, rank, world, dev, rowptr, col, ei, val, s0, s1):
    """`csr_spgemm` (the cuSPARSE extension's drop-in) on the product the APPNP step forms: C = S P,
    S = this rank's PPR state (the rows of seeds s0..s1 with their top-8 entries, from the APPNP run
    above), P = D^-1 A of the 169,343-node graph (fp32 values 1 / deg(row))."""
    from neutrongt_b200.spgemm import csr_spgemm
    peak, peak_kind = measured_hbm_peak()
    rp_b, col_b = rowptr.to(dev), col.to(dev)
    deg = rp_b[1:] - rp_b[:-1]
    val_b = (1.0 / deg.clamp_min(1).to(torch.float32)).repeat_interleave(deg)
    m = s1 - s0
    rows = ei[0] - s0
    order = torch.argsort(rows, stable=True)
    rows, col_a, val_a = rows[order], ei[1][order].contiguous(), val[order].to(torch.float32).contiguous()
    rp_a = torch.zeros(m + 1, dtype=torch.long, device=dev)
    rp_a[1:] = torch.cumsum(torch.bincount(rows, minlength=m), 0)
    call = lambda: csr_spgemm(rp_a, col_a, val_a, rp_b, col_b, val_b)
    call()
    (c_rp, c_col, c_val), t = _timed_call(call, world)
    nnz_a, nnz_c = col_a.numel(), c_col.numel()
    gathered = int(deg[col_a].sum())   # B entries read: the rows of B that A's entries select
    # algorithmic bytes: A (rowptr 8, col 8 + val 4 per entry, int64 inputs), B's two row pointers per
    # A entry (16) and its selected entries (col 8 + val 4), C written (rowptr 8, col 8 + val 4)
    nbytes = 8 * (m + 1) + 12 * nnz_a + 16 * nnz_a + 12 * gathered + 8 * (m + 1) + 12 * nnz_c
    achieved = allreduce_sum(float(nbytes), world) / t / 1e9
    out = {"workload": "C = S P: S = the APPNP PPR state of every seed of the 169,343-node graph (top-8 "
                       "entries per row), P = D^-1 A (2,332,486 entries); fp32 values, int64 CSR in and out",
           "seconds": t, "rows_per_s": allreduce_sum(float(m), world) / t,
           "a_entries": int(allreduce_sum(float(nnz_a), world)), "b_entries_gathered":
               int(allreduce_sum(float(gathered), world)), "c_entries": int(allreduce_sum(float(nnz_c), world)),
           "scaling": "strong (rows of S split with the PPR seed ranges)",
           "roofline": {"bound": "hbm", "achieved": achieved, "peak": peak, "unit": "GB/s",
                        "frac": achieved / peak if peak else None, "peak_kind": peak_kind,
                        "note": "no-reuse algorithmic bytes (A, B's selected rows, C); B (28 MB) is L2-resident"}}
    if rank == 0 and not args.skip_cpu:
        from oracle import spgemm as ospgemm
        sample = 300   # ~6 s of pure-Python row products
        ra = rp_a[:sample + 1].cpu()
        ca, va = col_a[:int(ra[-1])].cpu(), val_a[:int(ra[-1])].cpu()
        rb, cb, vb = rp_b.cpu(), col_b.cpu(), val_b.cpu()
        t0 = time.perf_counter()
        ospgemm.csr_spgemm(ra, ca, va, rb, cb, vb)
        tc = time.perf_counter() - t0
        out["cpu_baseline"] = {"value": sample / tc, "unit": "rows/s", "cores": 1, "kind": "port",
                               "sample": f"rows 0..{sample - 1} of S (the hub seeds), the row-wise product "
                                         "restated in Python (oracle/spgemm.py)"}
    return out


def bench_ppr_large(args, rank, world, dev):
    """PPR on the two large graphs, seeds sharded over ranks in degree-balanced ranges:
    push PPR (the reference's default backend) with eps 1e-4, alpha 0.15, top-10 on 232,965 nodes /
    57,307,946 undirected edges (mean degree ~492), and APPNP (alpha 0.15, 20 iterations, top-4) on
    2,449,029 nodes / 61,859,140 undirected edges.  Graphs are sampled on the device."""
    from neutrongt_b200 import personal_pagerank_appnp, personal_pagerank_torch_geometric, synthetic
    peak, peak_kind = measured_hbm_peak()
    res = {}
    # ---- push PPR, 232,965 nodes ----
    n5 = 232965
    rp, col = synthetic.chung_lu_graph_device(n5, 114615892 // 2, seed=5, device=dev)
    deg = (rp[1:] - rp[:-1]).double()
    s0, s1 = balanced_ranges(deg.cpu() + 64.0, world)[rank]
    csr = {"rowptr": rp, "col": col}
    # warm-up on the timed range itself, so the per-slot workspace (GBs) is already a cached block
    # when the timed call runs (after a 500-seed warm-up a 2-GPU run timed this call at 0.087 s;
    # repeated full-range calls take 0.011 s on the slower rank)
    personal_pagerank_torch_geometric(None, 0.15, topk=10, eps=1e-4, device=dev, csr_data=csr, source_start=s0,
                                      source_end=s1)
    st = {}
    (ei, _), t = _timed_call(lambda: personal_pagerank_torch_geometric(None, 0.15, topk=10, eps=1e-4, device=dev,
                                                                      csr_data=csr, source_start=s0, source_end=s1,
                                                                      stats=st), world)
    reads = allreduce_sum(float(st["edges_touched"]), world)
    pushes = allreduce_sum(float(st["pushes"]), world)
    # bytes per adjacency entry read in a push: column index 4, residual read + write 16, flags 2,
    # the neighbour's degree (two row pointers) 16
    gbs = reads * 38 / t / 1e9
    push = {"workload": "push PPR (torch_geometric backend), alpha 0.15, eps 1e-4, top-10, every node a seed; "
                        "232,965-node Chung-Lu graph with 114,615,892 directed edges",
            "seconds": t, "seeds_per_s": n5 / t, "pushes": pushes, "adjacency_entries_read": reads,
            "entries": int(allreduce_sum(float(ei.shape[1]), world)),
            "roofline": {"bound": "hbm", "achieved": gbs, "peak": peak, "unit": "GB/s", "frac": gbs / peak,
                         "peak_kind": f"{peak_kind} hbm_gbs",
                         "note": "38 algorithmic bytes per adjacency entry read (column 4, residual 8+8, flags 2, "
                                 "neighbour degree 16); random 8-byte residual accesses"}}
    if rank == 0 and not args.skip_cpu:
        from oracle import ppr as oppr
        threads = os.cpu_count() or 1
        cpu_csr = {"rowptr": rp.cpu(), "col": col.cpu()}
        sample = 1000
        t0 = time.perf_counter()
        oppr.personal_pagerank_push(None, 0.15, topk=10, eps=1e-4, csr_data=cpu_csr, source_start=0,
                                    source_end=sample, nthreads=threads)
        tc = time.perf_counter() - t0
        push["cpu_baseline"] = {"value": sample / tc, "unit": "seeds/s", "cores": threads, "kind": "port",
                                "sample": f"seeds 0..{sample - 1} (the hubs), the push method restated in C "
                                          "(oracle/push_oracle.c)"}
    res["push_232965"] = push
    del rp, col, csr, deg, ei
    torch.cuda.empty_cache()
    # ---- APPNP top-4, 2,449,029 nodes ----
    n4 = 2449029
    rp, col = synthetic.chung_lu_graph_device(n4, 61859140, seed=4, device=dev)
    deg = (rp[1:] - rp[:-1]).double()
    s0, s1 = balanced_ranges(deg.cpu() + 8.0, world)[rank]
    csr = {"rowptr": rp, "col": col}
    prm = dict(alpha=0.15, topk=4, num_iterations=20, iter_topk=4)
    personal_pagerank_appnp(None, csr_data=csr, device=dev, source_start=s0, source_end=min(s1, s0 + 2000), **prm)
    (ei, _), t = _timed_call(lambda: personal_pagerank_appnp(None, csr_data=csr, device=dev, source_start=s0,
                                                              source_end=s1, **prm), world)
    appnp = {"workload": "APPNP PPR, alpha 0.15, 20 iterations, top-4 per iteration and at the end, every node a "
                         "seed; 2,449,029-node Chung-Lu graph with 123,718,280 directed edges",
             "seconds": t, "seeds_per_s": n4 / t, "entries": int(allreduce_sum(float(ei.shape[1]), world))}
    if rank == 0 and not args.skip_cpu:
        from oracle import ppr as oppr
        threads = os.cpu_count() or 1
        sample = 2000
        t0 = time.perf_counter()
        oppr.personal_pagerank_appnp(None, csr_data={"rowptr": rp.cpu(), "col": col.cpu()}, source_start=0,
                                     source_end=sample, nthreads=threads, **prm)
        tc = time.perf_counter() - t0
        appnp["cpu_baseline"] = {"value": sample / tc, "unit": "seeds/s", "cores": threads, "kind": "port",
                                 "sample": f"seeds 0..{sample - 1} (the hubs), canonical fp64 restatement in C "
                                           "(oracle/appnp_oracle.c)"}
    res["appnp_2449029"] = appnp
    return res


def bench_gph_large_layer(args, dev, steps=3, warm=2):
    """One GPH_Large (Graphormer) encoder layer, bf16: 32,768 tokens, hidden 768, ffn 768, 32 heads of
    24, full attention; forward + backward.  The projections run on the bf16 tcgen05 GEMMs, the
    attention on the dense tcgen05 kernels."""
    from neutrongt_b200.models import GraphormerEncoderLayer
    S, hid, heads = 32768, 768, 32
    torch.manual_seed(0)
    layer = GraphormerEncoderLayer(hid, hid, 0.0, 0.0, heads).to(dev).to(torch.bfloat16).train()
    g = torch.Generator(device=dev).manual_seed(0)
    x = torch.randn(1, S, hid, generator=g, device=dev).to(torch.bfloat16).requires_grad_(True)
    dy = torch.randn(1, S, hid, generator=g, device=dev).to(torch.bfloat16)

    def step():
        layer.zero_grad(set_to_none=True)
        x.grad = None
        y, _, _ = layer(x, attn_type="full")
        y.backward(dy)

    for _ in range(warm):
        step()
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record()
    for _ in range(steps):
        step()
    e1.record()
    e1.synchronize()
    t = e0.elapsed_time(e1) / 1e3 / steps
    proj = 2.0 * S * 6 * hid * hid * 3          # QKV, output, FFN in and out: forward + two backward GEMMs
    attn = 4.0 * S * S * hid * 3.5              # 4 S^2 H D forward, 2.5x that backward
    peak, kind = measured_bf16_peak(sustained=True)
    achieved = (proj + attn) / t / 1e12
    return {"workload": "one GPH_Large (Graphormer) encoder layer, bf16, 32,768 tokens, hidden 768, ffn 768, "
                        "32 heads of 24, full attention, forward + backward, one GPU",
            "ms_per_step": t * 1e3, "tflops_algorithmic": achieved,
            "flops": {"projections": proj, "attention": attn},
            "roofline": {"bound": "tensor", "achieved": achieved, "peak": peak, "unit": "TFLOP/s",
                         "peak_kind": f"{kind} bf16_tflops_sustained", "frac": achieved / peak}}


def bench_window_build(args, dev, ppr_ei, ppr_val, pct=5):
    """Window construction on the 169,343-node graph's PPR output: the weighted PPR adjacency
    (build_adj_fromat), the halo merge of each of the 16 windows at the reference scripts'
    --related_nodes_topk_rate 5, and the duplicate-first order of the grown windows (two parents
    of 8).  Windows are the seeded random partitions (pymetis is absent).  Rank-0 preprocessing in
    the reference; measured at N = 1."""
    from neutrongt_b200 import synthetic
    from neutrongt_b200.window import build_adj_format, find_duplicate_nodes_and_rerange, merge_related_nodes
    n = 169343
    parts = synthetic.random_partitions(n, 16, seed=0)

    def run():
        csr, ew, _ = build_adj_format((ppr_ei, ppr_val), device=dev)
        halos = [merge_related_nodes(p, csr, ew, pct, device=dev) for p in parts]
        groups, dups = find_duplicate_nodes_and_rerange([halos[:8], halos[8:]])
        return csr, ew, halos, dups

    run()
    torch.cuda.synchronize()
    e0, e1, e2 = (torch.cuda.Event(enable_timing=True) for _ in range(3))
    e0.record()
    csr, ew, _ = build_adj_format((ppr_ei, ppr_val), device=dev)
    e1.record()
    halos = [merge_related_nodes(p, csr, ew, pct, device=dev) for p in parts]
    _, dups = find_duplicate_nodes_and_rerange([halos[:8], halos[8:]])
    e2.record()
    e2.synchronize()
    t_adj, t_win = e0.elapsed_time(e1) / 1e3, e1.elapsed_time(e2) / 1e3
    out = {"ppr_entries": int(ppr_ei.shape[1]), "undirected_pairs": int(csr.adjacent.numel()) // 2,
           "adjacency_s": t_adj, "halo_and_dup_order_s": t_win, "topk_percent": pct,
           "window_nodes_after_halo_mean": sum(int(h.numel()) for h in halos) / len(halos),
           "duplicated_nodes": sum(int(d.numel()) for d in dups),
           "note": "host reads of output sizes included; CUDA events on the launching stream"}
    if not args.skip_cpu:
        from oracle import window as ow
        m_s = min(200000, int(ppr_ei.shape[1]))
        ei_c, v_c = ppr_ei[:, :m_s].cpu().numpy(), ppr_val[:m_s].cpu().numpy()
        t0 = time.perf_counter()
        ow.ppr_adjacency(ei_c, v_c)
        t_a = (time.perf_counter() - t0) * int(ppr_ei.shape[1]) / m_s
        x, a, e = (t.cpu().numpy() for t in (csr.adj_starts, csr.adjacent, ew))
        t0 = time.perf_counter()
        ow.merge_related_nodes(parts[0], x, a, e, pct)
        t_h = (time.perf_counter() - t0) * len(parts)
        out["cpu_baseline"] = {"value": t_a + t_h, "unit": "s (adjacency + 16 halo merges)", "cores": 1,
                               "kind": "port", "sample": f"adjacency over the first {m_s} PPR entries scaled to all, "
                                                         "one window's halo merge x 16 (oracle/window.py)"}
    return out


def run_ours(args):
    rank, world, local = dist_setup()
    dev = torch.device("cuda", local)
    res = bench_attention(args, rank, world, dev)
    ppr = None if args.skip_ppr else bench_ppr(args, rank, world, dev)
    if ppr is not None and not args.skip_large_ppr:
        ppr.update(bench_ppr_large(args, rank, world, dev))
    epoch = None
    if not args.skip_epoch:
        epoch = bench_gt_epoch(args, rank, world, dev, config2_windows(dev),
                               "16 windows from the preprocessing pipeline (APPNP PPR top-8, PPR adjacency, seeded "
                               "random parts as METIS stand-in, 5 % halo merge, duplicate-first order)")
        from neutrongt_b200 import synthetic
        epoch["random_windows"] = bench_gt_epoch(args, rank, world, dev, synthetic.random_partitions(169343, 16, seed=0),
                                                 "16 seeded random windows without halo growth", epochs=3,
                                                 with_cpu=False)
    dense = None if args.skip_dense else bench_dense(args, rank, world, dev)
    if dense is not None and world == 1 and not args.skip_layer:
        dense["gph_large_layer"] = bench_gph_large_layer(args, dev)
    cpu = None
    if rank == 0 and not args.skip_cpu:
        q, k, v, g, ei = res["host"]
        cpu = cpu_baseline_sample(q, k, v, g, ei)
    if rank == 0:
        line = {
            "metric": "sparse-attn edges/s (graph-sparse window attention fwd+bwd; the GT epoch time is reported "
                      "in gt_epoch)",
            "value": res["value"], "unit": "edges/s", "n_gpus": world, "steps": args.steps, "warmup": args.warmup,
            "ms_per_step": res["ms_per_step"], "higher_is_better": True, "scaling": "weak", "vs_baseline": None,
            "dtype": "bf16", "data": "synthetic",
            "config": {"workload": "isolated graph-sparse attention fwd+bwd, one 65,536-token window per GPU, "
                                   "in-degree ~ Poisson(32), uniform sources",
                       "tokens": N_TOKENS, "edges_per_window": res["edges"], "heads": HEADS, "head_dim": HEAD_DIM,
                       "l2": "flushed between steps (256 MiB write outside the timed events)",
                       "parallelism": f"independent windows, dp{world}"},
            "roofline": res["roofline"], "cpu_baseline": cpu, "e2e": res["e2e"], "gpu_launches": res["gpu_launches"],
            "clocks": res["clocks"], "gt_epoch": epoch, "dense": dense, "ppr": ppr,
        }
        print(json.dumps(line), flush=True)
    if world > 1:
        import torch.distributed as dist
        dist.destroy_process_group()


def run_reference(args):
    rank = int(os.environ.get("RANK", "0"))
    if rank != 0:
        return
    torch.set_num_threads(os.cpu_count() or 1)
    from oracle import attention as oatt
    q, k, v, g, ei = make_window(seed=0)
    rows = 8192
    sub = ei[:, ei[1] < rows]
    qf, kf, vf, gf = (t.float() for t in (q, k, v, g))
    for _ in range(max(1, min(args.warmup, 2))):
        oatt.sparse_attention_forward(qf, kf, vf, sub)
    times = []
    for _ in range(args.steps):
        t0 = time.perf_counter()
        oatt.sparse_attention_forward(qf, kf, vf, sub)
        oatt.sparse_attention_backward(qf, kf, vf, sub, gf)
        times.append(time.perf_counter() - t0)
    t = sum(times)
    value = sub.shape[1] * args.steps / t
    threads = os.cpu_count() or 1
    line = {"impl": "reference", "metric": "sparse-attn edges/s (graph-sparse window attention fwd+bwd; the GT epoch "
                                           "time is reported in gt_epoch)",
            "value": value, "unit": "edges/s", "n_gpus": int(os.environ.get("WORLD_SIZE", "1")), "steps": args.steps,
            "warmup": args.warmup, "ms_per_step": t / args.steps * 1e3, "higher_is_better": True, "scaling": "weak",
            "vs_baseline": None, "dtype": "f32", "data": "synthetic",
            "config": {"workload": "isolated-kernel window (65,536 tokens, Poisson(32) in-degrees), bounded sample: the "
                                   "in-edges of the lowest "
                                   f"{rows} destination rows ({sub.shape[1]} edges) per step",
                       "tokens": N_TOKENS, "heads": HEADS, "head_dim": HEAD_DIM},
            "cpu_baseline": {"value": value, "unit": "edges/s", "cores": threads, "kind": "port",
                             "sample": f"{sub.shape[1]} edges per step; the reference's torch gather/scatter "
                                       "algorithm (oracle/attention.py) in fp32 on the host cores"},
            "e2e": {"value": value, "unit": "edges/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}}
    print(json.dumps(line), flush=True)


def epoch_kernel_table(args):
    """Kernel composition of one graph-replayed GT epoch (the 169,343-node graph's pipeline windows, one GPU)."""
    from torch.profiler import ProfilerActivity, profile
    from neutrongt_b200 import synthetic
    from neutrongt_b200.train import GraphedWindowTrainer, build_window_state
    dev = torch.device("cuda:0")
    torch.cuda.set_device(dev)
    n = 169343
    rowptr, col = config2_graph()
    feature = synthetic.node_features(n, 128, seed=1).to(dev)
    y = synthetic.node_labels(n, 40, seed=2).to(dev)
    split = synthetic.split_idx(n, seed=3)
    ws = build_window_state(rowptr, col, config2_windows(dev), 0, 1, feature, dev, split)
    model = gt_model(dev)
    opt = torch.optim.AdamW(model.parameters(), lr=1e-4, weight_decay=0.01, fused=True, capturable=True)
    trainer = GraphedWindowTrainer(SimpleNamespace(use_cache=1, attn_type="sparse"), model, ws, feature, y, opt, 1,
                                   dev, split_idx=split)
    for _ in range(max(3, args.warmup)):
        trainer.run_epoch()
    t = trainer.run_epoch()[2]
    with profile(activities=[ProfilerActivity.CUDA]) as prof:
        trainer.run_epoch()
        torch.cuda.synchronize()
    rows = [(e.key, e.self_device_time_total, e.count) for e in prof.key_averages() if e.self_device_time_total > 0]
    rows.sort(key=lambda r: -r[1])
    total = sum(r[1] for r in rows)
    print(f"graph-replayed epoch: {t * 1e3:.2f} ms (CUDA events); kernels {total / 1e3:.2f} ms")
    print(f"{'us':>10} {'share':>7} {'calls':>6}  kernel")
    for key, us, cnt in rows:
        print(f"{us:10.1f} {100 * us / total:6.2f}% {cnt:6d}  {key[:110]}")
    trainer.graphs.clear()
    trainer.dummy = None


def linear_calls(rows=14252, n=20, reps=5):
    """Per-call device time of ngt_linear_forward / _backward_input / _backward_weight on the GT
    window's shapes, each call repeated `n` times inside one CUDA graph (no host launch cost)."""
    from neutrongt_b200 import _lib
    dev = torch.device("cuda:0")
    torch.cuda.set_device(dev)
    lib, ptr = _lib.lib(), _lib.ptr
    g = torch.Generator(device=dev).manual_seed(0)
    t = {(r, c): torch.randn(r, c, generator=g, device=dev) for r, c in
         [(rows, 128), (rows, 256), (256, 128), (128, 256)]}
    b = torch.randn(256, generator=g, device=dev)
    out = {c: torch.empty(rows, c, device=dev) for c in (128, 256)}
    dw, db = torch.empty(256, 256, device=dev), torch.empty(256, device=dev)
    ws = {io: _lib.workspace(_lib.size_query(lib.ngt_linear_weight_workspace_size, rows, *io), dev)
          for io in [(128, 128), (128, 256), (256, 128)]}
    st = lambda: _lib.stream_of(b)
    x1, x2 = t[(rows, 128)], t[(rows, 256)]
    calls = {
        "forward 128 -> 128": lambda: lib.ngt_linear_forward(rows, 128, 128, ptr(x1), ptr(t[(128, 256)]), ptr(b),
                                                             ptr(out[128]), st()),
        "forward 128 -> 256": lambda: lib.ngt_linear_forward(rows, 128, 256, ptr(x1), ptr(t[(256, 128)]), ptr(b),
                                                             ptr(out[256]), st()),
        "forward 256 -> 128": lambda: lib.ngt_linear_forward(rows, 256, 128, ptr(x2), ptr(t[(128, 256)]), ptr(b),
                                                             ptr(out[128]), st()),
        "input grad 128 <- 128": lambda: lib.ngt_linear_backward_input(rows, 128, 128, ptr(x1), ptr(t[(256, 128)]),
                                                                       ptr(out[128]), st()),
        "input grad 128 <- 256": lambda: lib.ngt_linear_backward_input(rows, 128, 256, ptr(x2), ptr(t[(256, 128)]),
                                                                       ptr(out[128]), st()),
        "input grad 256 <- 128": lambda: lib.ngt_linear_backward_input(rows, 256, 128, ptr(x1), ptr(t[(128, 256)]),
                                                                       ptr(out[256]), st()),
    }
    for i, o in ws:
        xin, gout = (x1 if i == 128 else x2), (x1 if o == 128 else x2)
        calls[f"weight grad {o} x {i}"] = (lambda i=i, o=o, xin=xin, gout=gout: lib.ngt_linear_backward_weight(
            rows, i, o, ptr(xin), ptr(gout), ptr(dw), ptr(db), ptr(ws[(i, o)]), ws[(i, o)].numel(), st()))
    side = torch.cuda.Stream(device=dev)
    for name, f in calls.items():
        side.wait_stream(torch.cuda.current_stream())
        with torch.cuda.stream(side):
            for _ in range(3):
                _lib.check(f(), name)
        torch.cuda.current_stream().wait_stream(side)
        torch.cuda.synchronize()
        graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(graph):
            for _ in range(n):
                f()
        graph.replay()
        torch.cuda.synchronize()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record()
        for _ in range(reps):
            graph.replay()
        e1.record()
        torch.cuda.synchronize()
        print(f"{name:24s} {e0.elapsed_time(e1) * 1000 / (reps * n):8.2f} us")
        del graph


def profile_case(case):
    """Small, fixed workloads for one-kernel ncu captures (profiles/*.md give the commands)."""
    dev = torch.device("cuda:0")
    torch.cuda.set_device(dev)
    if case == "spattn":
        from neutrongt_b200.attention import WindowAttentionBuffers
        from neutrongt_b200.edge_csr import build_edge_csr
        q, k, v, dout, ei = (t.to(dev) for t in make_window(seed=0))
        buf = WindowAttentionBuffers(q, k, v, build_edge_csr(ei, N_TOKENS))
        flush = torch.empty(L2_FLUSH_BYTES, dtype=torch.uint8, device=dev)
        for i in range(3):
            flush.fill_(i)
            buf.forward()
            buf.backward(dout)
    elif case == "dense":
        import math as _m
        from neutrongt_b200.dense_attention import dense_attention
        g = torch.Generator(device=dev).manual_seed(0)
        S, H, D = 32768, 4, 24   # the GPH_Large per-rank dense window (bench_dense at N = 1)
        q, k, v, dy = (torch.randn(S, H, D, generator=g, device=dev).to(torch.bfloat16) * 0.5 for _ in range(4))
        qd, kd, vd = (t.requires_grad_(True) for t in (q, k, v))
        for _ in range(3):
            x, _ = dense_attention(qd, kd, vd, _m.sqrt(D), score_heads=32, check_status=False)
            x.backward(dy)
    elif case == "gemm":
        from neutrongt_b200.layers import Linear
        x = torch.randn(32768, 768, device=dev).to(torch.bfloat16).requires_grad_(True)
        lin = Linear(768, 768).to(dev).to(torch.bfloat16)
        dy = torch.randn(32768, 768, device=dev).to(torch.bfloat16)
        for _ in range(3):
            lin.zero_grad(set_to_none=True)
            lin(x).backward(dy)
    else:
        from neutrongt_b200 import synthetic
        from neutrongt_b200.ppr import personal_pagerank_torch_geometric
        rp, col = synthetic.chung_lu_graph_device(40000, 2000000, seed=5, device=dev)
        for _ in range(2):
            personal_pagerank_torch_geometric(None, 0.15, topk=10, eps=1e-5, device=dev,
                                              csr_data={"rowptr": rp, "col": col}, source_start=10000,
                                              source_end=14000)
    torch.cuda.synchronize()


def main():
    args = parse_args()
    if args.profile_case:
        profile_case(args.profile_case)
        return
    if args.linear_calls:
        linear_calls()
        return
    if args.epoch_kernels:
        epoch_kernel_table(args)
        return
    if args.impl == "reference":
        run_reference(args)
    else:
        run_ours(args)


if __name__ == "__main__":
    main()
