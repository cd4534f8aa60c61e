"""LayerNorm and Linear for the GT / Graphormer mirrors, with their work on our kernels.

`LayerNorm` and `Linear` subclass `nn.LayerNorm` / `nn.Linear`: same constructor, parameter names
(`weight`, `bias`) and state_dict, so reference checkpoints load unchanged.  On CUDA fp32 inputs:

* `LayerNorm` runs `ngt_layernorm_forward` / `ngt_layernorm_backward` (one warp per row, column
  sums of the weight / bias gradients in a fixed order);
* `Linear` runs `ngt_linear_forward` (y = x W^T + b), `ngt_linear_backward_input` (dx = dy W) and
  `ngt_linear_backward_weight` (dW = dy^T x and db = column sums of dy, one pass, fixed-order
  reduction).  With both dimensions <= 256 the forward and input grad run on the tcgen05 tensor
  cores with split TF32 operands (fp32 precision, `csrc/linear_tc.cu`); the weight grad and wider
  outputs are fp32 FFMA GEMMs sized to the SM count for the windows' thin shapes.

On CUDA bf16 inputs with a bf16 weight (the large model trained in bf16), `Linear` runs the bf16
tcgen05 GEMMs of `csrc/gemm_bf16.cu`: `ngt_linear_bf16_forward`, `ngt_linear_bf16_backward_input`
and `ngt_linear_bf16_backward_weight` (fp32 accumulation in TMEM, TMA-fed 128-byte-swizzled
tiles, any size with both feature counts multiples of 8).

torch's kernels for these ops take 15-60 us per call on the models' [~10^4, 32..256] fp32
windows; these take a few.  Other devices, dtypes or shapes (features not a multiple of 4 (fp32)
or 8 (bf16), a LayerNorm wider than 1024, an fp32 Linear inner dimension above 256) use the torch
operators.  Reference
layers: NeutronGT/models/gt_dist_node_level_single_window.py:235-241, 311-325, 360-361, 537, 565;
graphormer_dist_node_level.py:179, 183, 286.
"""
from __future__ import annotations

import contextlib
import threading

import torch
import torch.nn as nn
import torch.nn.functional as F

from . import _lib

# ---- weight gradients on a side stream -------------------------------------------------------
# Inside `overlap_weight_grads()` a Linear layer's weight / bias gradient kernels run on a side
# stream that forks from the backward's stream and joins it again when the backward pass ends
# (an autograd end-of-backward callback), so they overlap the input-gradient chain of the layers
# below.  Only valid when autograd hands the gradient to the parameter without reading it (the
# parameter's .grad is None, as `optimizer.zero_grad(set_to_none=True)` leaves it); the training
# loops enter it only then.
# (Process-wide state: autograd runs CUDA backward functions on its own per-device threads.)
class _State:
    overlap = False
    pending = None


_state = _State()
_side: dict = {}
_lock = threading.Lock()


@contextlib.contextmanager
def overlap_weight_grads(enabled: bool = True):
    with _lock:
        prev = _state.overlap
        _state.overlap = enabled
    try:
        yield
    finally:
        with _lock:
            _state.overlap = prev


def _side_stream(device) -> torch.cuda.Stream:
    key = device.index
    if key not in _side:
        _side[key] = torch.cuda.Stream(device=device)
    return _side[key]


def _join_later(cur: torch.cuda.Stream, side: torch.cuda.Stream):
    if _state.pending is None:
        _state.pending = {}
        torch.autograd.Variable._execution_engine.queue_callback(_join_all)
    _state.pending[(cur, side)] = None


def _join_all():
    pending = _state.pending or {}
    _state.pending = None
    for cur, side in pending:
        cur.wait_stream(side)


def _rows_ok(x: torch.Tensor, cols: int) -> bool:
    return x.is_cuda and x.dtype == torch.float32 and cols % 4 == 0 and 0 < cols <= 1024


_WS_BYTES: dict = {}


def _ws(rows: int, cols: int, device) -> torch.Tensor:
    key = (rows, cols)
    nbytes = _WS_BYTES.get(key)
    if nbytes is None:
        nbytes = _WS_BYTES[key] = _lib.size_query(_lib.lib().ngt_rowops_workspace_size, rows, cols)
    return _lib.workspace(nbytes, device)


def column_sum(g: torch.Tensor) -> torch.Tensor:
    """Sum over the rows of a [rows, cols] fp32 CUDA tensor (fixed-order reduction)."""
    g = g.contiguous()
    rows, cols = g.shape
    out = torch.empty(cols, dtype=torch.float32, device=g.device)
    ws = _ws(rows, cols, g.device)
    _lib.check(_lib.lib().ngt_column_sum(rows, cols, _lib.ptr(g), _lib.ptr(out), _lib.ptr(ws), ws.numel(),
                                         _lib.stream_of(g)), "ngt_column_sum")
    return out


class _LayerNormFn(torch.autograd.Function):
    @staticmethod
    def forward(ctx, x, weight, bias, eps):
        shape = x.shape
        cols = shape[-1]
        x2 = x.reshape(-1, cols).contiguous()
        rows = x2.shape[0]
        y = torch.empty_like(x2)
        mean = torch.empty(rows, dtype=torch.float32, device=x.device)
        rstd = torch.empty_like(mean)
        _lib.check(_lib.lib().ngt_layernorm_forward(rows, cols, _lib.ptr(x2), _lib.ptr(weight), _lib.ptr(bias),
                                                    float(eps), _lib.ptr(y), _lib.ptr(mean), _lib.ptr(rstd),
                                                    _lib.stream_of(x2)), "ngt_layernorm_forward")
        ctx.save_for_backward(x2, weight, mean, rstd)
        ctx.shape = shape
        return y.view(shape)

    @staticmethod
    def backward(ctx, dy):
        x2, weight, mean, rstd = ctx.saved_tensors
        rows, cols = x2.shape
        dy2 = dy.reshape(rows, cols).contiguous().float()
        dx = torch.empty_like(x2)
        dw = torch.empty(cols, dtype=torch.float32, device=x2.device)
        db = torch.empty_like(dw)
        ws = _ws(rows, cols, x2.device)
        _lib.check(_lib.lib().ngt_layernorm_backward(rows, cols, _lib.ptr(x2), _lib.ptr(dy2), _lib.ptr(weight),
                                                     _lib.ptr(mean), _lib.ptr(rstd), _lib.ptr(dx), _lib.ptr(dw),
                                                     _lib.ptr(db), _lib.ptr(ws), ws.numel(), _lib.stream_of(x2)),
                   "ngt_layernorm_backward")
        return dx.view(ctx.shape), dw, db, None


_WSL: dict = {}


def _linear_ws(rows: int, in_f: int, out_f: int, device) -> torch.Tensor:
    key = (rows, in_f, out_f, device.index)
    nbytes = _WSL.get(key)
    if nbytes is None:
        nbytes = _WSL[key] = _lib.size_query(_lib.lib().ngt_linear_weight_workspace_size, rows, in_f, out_f)
    return _lib.workspace(nbytes, device)


_MAX_INNER = 256     # ngt_linear_forward / ngt_linear_backward_input keep W's inner dimension on chip


class _LinearFn(torch.autograd.Function):
    @staticmethod
    def forward(ctx, x, weight, bias):
        shape = x.shape
        out_f, in_f = weight.shape
        x2 = x.reshape(-1, in_f).contiguous()
        rows = x2.shape[0]
        if in_f <= _MAX_INNER:
            y = torch.empty(rows, out_f, dtype=torch.float32, device=x.device)
            _lib.check(_lib.lib().ngt_linear_forward(rows, in_f, out_f, _lib.ptr(x2), _lib.ptr(weight), _lib.ptr(bias),
                                                     _lib.ptr(y), _lib.stream_of(x2)), "ngt_linear_forward")
        else:
            y = torch.addmm(bias, x2, weight.t())
        ctx.save_for_backward(x2, weight)
        ctx.shape = shape
        return y.view(*shape[:-1], out_f)

    @staticmethod
    def backward(ctx, g):
        x2, weight = ctx.saved_tensors
        out_f, in_f = weight.shape
        g2 = g.reshape(-1, out_f).contiguous()
        rows = g2.shape[0]
        dx = dw = db = None
        if ctx.needs_input_grad[0]:
            if out_f <= _MAX_INNER:
                dx = torch.empty(rows, in_f, dtype=torch.float32, device=g2.device)
                _lib.check(_lib.lib().ngt_linear_backward_input(rows, in_f, out_f, _lib.ptr(g2), _lib.ptr(weight),
                                                                _lib.ptr(dx), _lib.stream_of(g2)),
                           "ngt_linear_backward_input")
            else:
                dx = g2.mm(weight)
            dx = dx.view(ctx.shape)
        if ctx.needs_input_grad[1]:
            overlap = _state.overlap
            cur = torch.cuda.current_stream(g2.device)
            side = _side_stream(g2.device) if overlap else cur
            if overlap:
                side.wait_stream(cur)                  # x2 and g2 are ready
            with torch.cuda.stream(side):
                dw = torch.empty(out_f, in_f, dtype=torch.float32, device=g2.device)
                if ctx.needs_input_grad[2]:
                    db = torch.empty(out_f, dtype=torch.float32, device=g2.device)
                ws = _linear_ws(rows, in_f, out_f, g2.device)
                _lib.check(_lib.lib().ngt_linear_backward_weight(rows, in_f, out_f, _lib.ptr(x2), _lib.ptr(g2),
                                                                 _lib.ptr(dw), _lib.ptr(db), _lib.ptr(ws),
                                                                 ws.numel(), _lib.stream_of(g2)),
                           "ngt_linear_backward_weight")
            if overlap:
                x2.record_stream(side)                 # freed on `cur` later: keep until side is done
                g2.record_stream(side)
                _join_later(cur, side)
        elif ctx.needs_input_grad[2]:
            db = column_sum(g2)
        return dx, dw, db


_WSB: dict = {}


def _linear_bf16_ws(rows: int, in_f: int, out_f: int, device) -> torch.Tensor:
    key = (rows, in_f, out_f, device.index)
    nbytes = _WSB.get(key)
    if nbytes is None:
        nbytes = _WSB[key] = _lib.size_query(_lib.lib().ngt_linear_bf16_weight_workspace_size, rows, in_f, out_f)
    return _lib.workspace(nbytes, device)


class _LinearBf16Fn(torch.autograd.Function):
    """bf16 y = x W^T + b on the tcgen05 tensor cores (fp32 accumulation, one bf16 rounding)."""

    @staticmethod
    def forward(ctx, x, weight, bias):
        shape = x.shape
        out_f, in_f = weight.shape
        x2 = x.reshape(-1, in_f).contiguous()
        rows = x2.shape[0]
        y = torch.empty(rows, out_f, dtype=torch.bfloat16, device=x.device)
        _lib.check(_lib.lib().ngt_linear_bf16_forward(rows, in_f, out_f, _lib.ptr(x2), _lib.ptr(weight),
                                                      _lib.ptr(bias), _lib.ptr(y), _lib.stream_of(x2)),
                   "ngt_linear_bf16_forward")
        ctx.save_for_backward(x2, weight)
        ctx.shape = shape
        ctx.has_bias = bias is not None
        return y.view(*shape[:-1], out_f)

    @staticmethod
    def backward(ctx, g):
        x2, weight = ctx.saved_tensors
        out_f, in_f = weight.shape
        g2 = g.reshape(-1, out_f).to(torch.bfloat16).contiguous()
        rows = g2.shape[0]
        dx = dw = db = None
        if ctx.needs_input_grad[0]:
            dx = torch.empty(rows, in_f, dtype=torch.bfloat16, device=g2.device)
            _lib.check(_lib.lib().ngt_linear_bf16_backward_input(rows, in_f, out_f, _lib.ptr(g2), _lib.ptr(weight),
                                                                 _lib.ptr(dx), _lib.stream_of(g2)),
                       "ngt_linear_bf16_backward_input")
            dx = dx.view(ctx.shape)
        want_db = ctx.has_bias and ctx.needs_input_grad[2]
        if ctx.needs_input_grad[1] or want_db:
            overlap = _state.overlap
            cur = torch.cuda.current_stream(g2.device)
            side = _side_stream(g2.device) if overlap else cur
            if overlap:
                side.wait_stream(cur)
            with torch.cuda.stream(side):
                dw = torch.empty(out_f, in_f, dtype=torch.bfloat16, device=g2.device)
                if want_db:
                    db = torch.empty(out_f, dtype=torch.bfloat16, device=g2.device)
                ws = _linear_bf16_ws(rows, in_f, out_f, g2.device)
                _lib.check(_lib.lib().ngt_linear_bf16_backward_weight(rows, in_f, out_f, _lib.ptr(x2), _lib.ptr(g2),
                                                                      _lib.ptr(dw), _lib.ptr(db), _lib.ptr(ws),
                                                                      ws.numel(), _lib.stream_of(g2)),
                           "ngt_linear_bf16_backward_weight")
            if overlap:
                x2.record_stream(side)
                g2.record_stream(side)
                _join_later(cur, side)
            if not ctx.needs_input_grad[1]:
                dw = None
        return dx, dw, db


def _bf16_linear_ok(x: torch.Tensor, weight: torch.Tensor, bias) -> bool:
    return (x.is_cuda and x.dtype == torch.bfloat16 and weight.dtype == torch.bfloat16 and x.numel() > 0
            and (bias is None or bias.dtype == torch.bfloat16)
            and weight.shape[0] % 8 == 0 and weight.shape[1] % 8 == 0)


class LayerNorm(nn.LayerNorm):
    def forward(self, x):
        if (self.elementwise_affine and self.bias is not None and len(self.normalized_shape) == 1
                and _rows_ok(x, self.normalized_shape[0]) and x.numel() > 0):
            return _LayerNormFn.apply(x, self.weight, self.bias, self.eps)
        return super().forward(x)


class Linear(nn.Linear):
    def forward(self, x):
        if (self.bias is not None and _rows_ok(x, 4) and self.weight.dtype == torch.float32 and x.numel() > 0
                and self.in_features % 4 == 0 and self.out_features % 4 == 0):
            return _LinearFn.apply(x, self.weight, self.bias)
        if _bf16_linear_ok(x, self.weight, self.bias):
            return _LinearBf16Fn.apply(x, self.weight, self.bias)
        return F.linear(x, self.weight, self.bias)
