"""The reference's on-disk formats, read (and for checkpoints written) unchanged.

* `load_optional_edge_csr(dataset_dir, dataset_name)` — `edge_index_csr.pt` holding
  {"rowptr", "col"}, with the checks of `NeutronGT/core/node_level_pipeline/graph_data.py:6-26`
  (same exceptions); returns None when the file is absent.
* `window_state_from_preprocess_cache(payload, ...)` — the preprocess cache written by
  `core/node_level_pipeline/preprocess_cache.py:49-65` (`build_preprocess_cache_payload`): its
  graph CSR and windows (`wm.partitioned_results`) become this rank's `WindowState`, built on the
  device as `build_window_state` does.
* `build_checkpoint_payload(...)` / `load_checkpoint(...)` — the training checkpoint of
  `core/node_level_pipeline/checkpoint.py:118-131`: the same keys, so either code base resumes from
  the other's file (model and optimizer state dicts have the reference's parameter names).
"""
from __future__ import annotations

import os
from typing import Any

import torch


def load_optional_edge_csr(dataset_dir: str, dataset_name: str):
    path = os.path.join(dataset_dir, dataset_name, "edge_index_csr.pt")
    if not os.path.exists(path):
        return None
    data = torch.load(path, map_location="cpu")
    if not isinstance(data, dict) or "rowptr" not in data or "col" not in data:
        raise KeyError(f"Invalid CSR data in {path}: expected dict with rowptr and col")
    rowptr, col = data["rowptr"], data["col"]
    if rowptr.dim() != 1 or col.dim() != 1:
        raise ValueError(f"Invalid CSR tensor shapes in {path}: rowptr dim={rowptr.dim()}, col dim={col.dim()}")
    if rowptr.numel() == 0:
        raise ValueError(f"Invalid CSR rowptr in {path}: rowptr must contain at least one element")
    if int(rowptr[0]) != 0:
        raise ValueError(f"Invalid CSR rowptr in {path}: rowptr[0] must be 0")
    if int(rowptr[-1]) != int(col.numel()):
        raise ValueError(f"Invalid CSR tensors in {path}: rowptr[-1]={int(rowptr[-1])} does not match "
                         f"col.numel()={int(col.numel())}")
    return {"rowptr": rowptr, "col": col}


def _payload(payload_or_path):
    if isinstance(payload_or_path, (str, os.PathLike)):
        return torch.load(payload_or_path, map_location="cpu", weights_only=False)
    return payload_or_path


def window_state_from_preprocess_cache(payload_or_path, rank: int, world_size: int, feature: torch.Tensor, device,
                                       split_idx=None, use_cache: bool = True):
    """This rank's windows (pid mod world_size, as `window_state.py:210` assigns them) from a
    reference preprocess cache, with duplicate-first order and edge lists built on the device."""
    from .train import build_window_state
    p = _payload(payload_or_path)
    csr = p.get("graph_csr_data")
    if csr is None or "rowptr" not in csr or "col" not in csr:
        raise KeyError("preprocess cache has no graph_csr_data {rowptr, col}")
    parts = p["wm"]["partitioned_results"]
    return build_window_state(csr["rowptr"], csr["col"], parts, rank, world_size, feature, device, split_idx,
                              use_cache=use_cache)


_CHECKPOINT_KEYS = ("epoch", "start_epoch", "model_state_dict", "optimizer_state_dict", "lr_scheduler_state_dict",
                    "args_snapshot", "loss_mean_list", "window_state_version", "best_val", "best_test")
# run arguments a checkpoint records and a resume must agree with (checkpoint.py:10-20)
CHECKPOINT_COMPAT_KEYS = ("dataset", "model", "n_layers", "hidden_dim", "num_heads", "attn_type", "n_parts",
                          "related_nodes_topk_rate", "ppr_topk")


def checkpoint_args_snapshot(args) -> dict:
    """The `args_snapshot` record of a checkpoint: each compatibility key read from `args`
    (an argparse namespace or any object with those attributes; a dict is read by key), None
    where absent, as `checkpoint.py:126` builds it."""
    if isinstance(args, dict):
        return {key: args.get(key) for key in CHECKPOINT_COMPAT_KEYS}
    return {key: getattr(args, key, None) for key in CHECKPOINT_COMPAT_KEYS}


def validate_checkpoint_compatibility(args, args_snapshot: dict) -> None:
    """Raises ValueError when a run argument differs from the checkpoint's snapshot; keys the
    snapshot does not hold (or holds as None) are skipped (`checkpoint.py:77-90`)."""
    if not args_snapshot:
        return
    current = checkpoint_args_snapshot(args)
    mismatches = [f"{key}: current={current[key]}, checkpoint={args_snapshot.get(key)}"
                  for key in CHECKPOINT_COMPAT_KEYS
                  if args_snapshot.get(key) is not None and current[key] != args_snapshot.get(key)]
    if mismatches:
        raise ValueError("Checkpoint is incompatible with current run arguments: " + "; ".join(mismatches))


def build_checkpoint_payload(args, model, optimizer, lr_scheduler, epoch: int, loss_mean_list,
                             window_state_version: int, best_val: float, best_test: float) -> dict[str, Any]:
    """The reference's checkpoint payload (`checkpoint.py:118-131`), same keys and types; `args`
    is the run's argument namespace (its compatibility keys become `args_snapshot`)."""
    return {
        "epoch": epoch,
        "start_epoch": epoch + 1,
        "model_state_dict": model.state_dict(),
        "optimizer_state_dict": optimizer.state_dict(),
        "lr_scheduler_state_dict": lr_scheduler.state_dict(),
        "args_snapshot": checkpoint_args_snapshot(args),
        "loss_mean_list": list(loss_mean_list),
        "window_state_version": int(window_state_version),
        "best_val": float(best_val),
        "best_test": float(best_test),
    }


def load_checkpoint(path_or_payload, model, optimizer=None, lr_scheduler=None, map_location="cpu", args=None):
    """Restores model (strict), optimizer and scheduler state from a reference-format checkpoint;
    returns the resume fields (start_epoch, loss_mean_list, best_val, best_test, ...).  With
    `args`, the checkpoint's `args_snapshot` is checked against them first and a mismatch raises
    ValueError before any state is loaded (`checkpoint.py:93-103`)."""
    ck = torch.load(path_or_payload, map_location=map_location, weights_only=False) \
        if isinstance(path_or_payload, (str, os.PathLike)) else path_or_payload
    missing = [k for k in ("model_state_dict",) if k not in ck]
    if missing:
        raise KeyError(f"checkpoint lacks {missing}")
    if args is not None:
        validate_checkpoint_compatibility(args, ck.get("args_snapshot", {}))
    model.load_state_dict(ck["model_state_dict"], strict=True)
    if optimizer is not None and "optimizer_state_dict" in ck:
        optimizer.load_state_dict(ck["optimizer_state_dict"])
    if lr_scheduler is not None and "lr_scheduler_state_dict" in ck:
        lr_scheduler.load_state_dict(ck["lr_scheduler_state_dict"])
    return {
        "start_epoch": int(ck.get("start_epoch", int(ck.get("epoch", -1)) + 1)),
        "loss_mean_list": list(ck.get("loss_mean_list", [])),
        "best_val": float(ck.get("best_val", float("-inf"))),
        "best_test": float(ck.get("best_test", float("-inf"))),
        "window_state_version": int(ck.get("window_state_version", 0)),
        "args_snapshot": dict(ck.get("args_snapshot", {})),
    }
