"""Dense full-attention windows on the tcgen05 tensor cores.

`full_attention(k, q, v, attn_bias, mask, pruning_mask, scale, dropout_p)` keeps the contract of
`CoreAttention.full_attention` (`NeutronGT/models/gt_dist_node_level_single_window.py:56-109`,
note the (k, q, v) argument order): q, k, v are [b, s, H, D] with b == 1; it returns
x [b, s, H, D] and node_scores [s] = sum over queries of the head-mean of |S|, where
S = (q * sqrt(D)) k^T — the reference multiplies by sqrt(D), and so does this kernel.
Gradients flow to q, k and v (`csrc/dense_tma.cu` backward for head_dim <= 32,
`csrc/dense_attn.cu` for 33..64); node_scores carries none.

The kernels compute in bfloat16 with fp32 accumulation; float32 inputs are rounded to
bfloat16 on entry and the output is returned in the input dtype.  Attention dropout uses a
counter-based hash of (seed, head, query, key), regenerated in the backward; it matches
torch's dropout in distribution, not bit for bit.

The optional attn_bias and pruning_mask ([b, H or 1, s, s], added to S) and mask ([s, s] bool,
masked_fill(-1e9) over every head, `…single_window.py:78-99`) are combined into one fp32 bias
(attn_bias + pruning_mask, masked entries -inf) that the biased kernels add before the softmax
(`ngt_dense_attn_forward_bias` / `_backward_bias`; gradients flow to attn_bias and pruning_mask
through that combination, zero at masked entries as masked_fill gives).  A query row whose
every key is masked gets the reference's result for it — a uniform softmax over its masked keys
(all at -1e9) — from a small fix-up after the kernel; a row whose keys are all -inf through the
bias alone is NaN in the reference and 0 here.

A kernel whose bounded wait runs out returns early and sets a device status word; the host
learns of it without a stall (`_StatusWord`): the next call on the device raises, and
`check_dense_status()` waits and raises at once.  Nothing in the forward or backward blocks the
host, so the Ulysses layer enqueues its exchanges while the kernels run.
"""
from __future__ import annotations

import math

import torch

from . import _lib


class _StatusWord:
    """Timeout reports of the dense kernels, read without stalling the host.

    Every bounded wait in the forward and backward kernels that runs out sets the int32 status
    word to 1 (no kernel ever clears it).  One persistent word per device collects every launch;
    after a launch with checking on, the word is copied to pinned host memory on the launching
    stream, so the host never waits for the kernel: the timeout is raised by the next dense
    attention call on that device, or by `check_dense_status`, which waits for the copies.  The
    word only goes 0 -> 1, so every value the host reads is a valid snapshot.
    """

    _by_device: dict = {}

    def __init__(self, dev):
        self.word = torch.zeros(1, dtype=torch.int32, device=dev)
        self.host = torch.zeros(1, dtype=torch.int32, pin_memory=True)
        self.event = torch.cuda.Event()

    @classmethod
    def of(cls, dev):
        key = torch.device(dev).index if torch.device(dev).index is not None else torch.cuda.current_device()
        sw = cls._by_device.get(key)
        if sw is None:
            sw = cls._by_device[key] = cls(torch.device("cuda", key))
        return sw

    def raise_if_set(self):
        if int(self.host[0]) != 0:
            self.event.synchronize()       # every copy in flight has landed before the reset
            self.word.zero_()
            torch.cuda.current_stream(self.word.device).synchronize()
            self.host.zero_()
            raise RuntimeError("dense attention kernel timed out waiting for the tensor core")

    def publish(self):
        if torch.cuda.is_current_stream_capturing():
            return                         # a captured launch is checked by the next eager one
        self.host.copy_(self.word, non_blocking=True)
        self.event.record()


def check_dense_status(device=None):
    """Waits for the status copies of the dense kernels on `device` and raises if any wait of
    theirs timed out since the last report."""
    sw = _StatusWord.of(torch.cuda.current_device() if device is None else device)
    sw.event.synchronize()
    sw.raise_if_set()


class _DenseAttention(torch.autograd.Function):
    @staticmethod
    def forward(ctx, q, k, v, scale, dropout_p, seed, score_heads, check):
        s, heads, dim = q.shape
        out = torch.empty_like(q)
        lse = torch.empty(heads, s, dtype=torch.float32, device=q.device)
        ns = torch.zeros(s, dtype=torch.float32, device=q.device)
        sw = _StatusWord.of(q.device)
        if check:
            sw.raise_if_set()
        _lib.check(_lib.lib().ngt_dense_attn_forward(s, heads, dim, float(scale), 1.0 / score_heads,
                                                     float(dropout_p), int(seed), _lib.ptr(q), _lib.ptr(k),
                                                     _lib.ptr(v), _lib.ptr(out), _lib.ptr(lse), _lib.ptr(ns),
                                                     _lib.ptr(sw.word), _lib.stream_of(q)),
                   "ngt_dense_attn_forward")
        if check:
            sw.publish()
        ctx.save_for_backward(q, k, v, out, lse)
        ctx.args = (scale, dropout_p, seed, check)
        ctx.mark_non_differentiable(ns)
        return out, ns

    @staticmethod
    def backward(ctx, dout, _dns):
        q, k, v, out, lse = ctx.saved_tensors
        scale, dropout_p, seed, check = ctx.args
        s, heads, dim = q.shape
        dout = dout.to(torch.bfloat16).contiguous()
        delta = torch.empty(heads, s, dtype=torch.float32, device=q.device)
        dq_acc = torch.empty(s, heads, dim, dtype=torch.float32, device=q.device)
        dq, dk, dv = torch.empty_like(q), torch.empty_like(k), torch.empty_like(v)
        sw = _StatusWord.of(q.device)
        if check:
            sw.raise_if_set()
        _lib.check(_lib.lib().ngt_dense_attn_backward(s, heads, dim, float(scale), float(dropout_p), int(seed),
                                                      _lib.ptr(q), _lib.ptr(k), _lib.ptr(v), _lib.ptr(out),
                                                      _lib.ptr(dout), _lib.ptr(lse), _lib.ptr(delta), _lib.ptr(dq_acc),
                                                      _lib.ptr(dq), _lib.ptr(dk), _lib.ptr(dv), _lib.ptr(sw.word),
                                                      _lib.stream_of(q)),
                   "ngt_dense_attn_backward")
        if check:
            sw.publish()
        return dq, dk, dv, None, None, None, None, None


class _DenseAttentionBias(torch.autograd.Function):
    """Dense attention with an additive fp32 bias [Hb, s, s] (Hb = 1 or H), differentiable in
    q, k, v and the bias."""

    @staticmethod
    def forward(ctx, q, k, v, bias, scale, dropout_p, seed, score_heads, check):
        s, heads, dim = q.shape
        out = torch.empty_like(q)
        lse = torch.empty(heads, s, dtype=torch.float32, device=q.device)
        ns = torch.zeros(s, dtype=torch.float32, device=q.device)
        hs = 0 if bias.shape[0] == 1 else s * s
        sw = _StatusWord.of(q.device)
        if check:
            sw.raise_if_set()
        _lib.check(_lib.lib().ngt_dense_attn_forward_bias(s, heads, dim, float(scale), 1.0 / score_heads,
                                                          float(dropout_p), int(seed), _lib.ptr(q), _lib.ptr(k),
                                                          _lib.ptr(v), _lib.ptr(bias), hs, _lib.ptr(out),
                                                          _lib.ptr(lse), _lib.ptr(ns), _lib.ptr(sw.word),
                                                          _lib.stream_of(q)),
                   "ngt_dense_attn_forward_bias")
        if check:
            sw.publish()
        ctx.save_for_backward(q, k, v, out, lse, bias)
        ctx.args = (scale, dropout_p, seed, check, hs)
        ctx.mark_non_differentiable(ns, lse)
        return out, ns, lse

    @staticmethod
    def backward(ctx, dout, _dns, _dlse):
        q, k, v, out, lse, bias = ctx.saved_tensors
        scale, dropout_p, seed, check, hs = ctx.args
        s, heads, dim = q.shape
        dout = dout.to(torch.bfloat16).contiguous()
        delta = torch.empty(heads, s, dtype=torch.float32, device=q.device)
        dq_acc = torch.empty(s, heads, dim, dtype=torch.float32, device=q.device)
        dq, dk, dv = torch.empty_like(q), torch.empty_like(k), torch.empty_like(v)
        dbias = torch.empty(heads, s, s, dtype=torch.float32, device=q.device) if ctx.needs_input_grad[3] else None
        sw = _StatusWord.of(q.device)
        if check:
            sw.raise_if_set()
        _lib.check(_lib.lib().ngt_dense_attn_backward_bias(s, heads, dim, float(scale), float(dropout_p), int(seed),
                                                           _lib.ptr(q), _lib.ptr(k), _lib.ptr(v), _lib.ptr(out),
                                                           _lib.ptr(dout), _lib.ptr(lse), _lib.ptr(bias), hs,
                                                           _lib.ptr(delta), _lib.ptr(dq_acc), _lib.ptr(dq), _lib.ptr(dk),
                                                           _lib.ptr(dv), _lib.ptr(dbias), _lib.ptr(sw.word),
                                                           _lib.stream_of(q)),
                   "ngt_dense_attn_backward_bias")
        if check:
            sw.publish()
        if dbias is not None and hs == 0:
            dbias = dbias.sum(0, keepdim=True)
        return dq, dk, dv, dbias, None, None, None, None, None


def _masked_rows_fixup(x, lse, v, mask):
    """Rows whose every key is masked: the reference's softmax over all -1e9 scores is uniform over
    the masked keys, so the row is the mean of their v rows (and its gradient reaches only v)."""
    dead = torch.isneginf(lse)                                   # [H, s]
    if mask is None or not bool(dead.any()):
        return x
    x = x.clone()
    m = mask.to(device=x.device, dtype=torch.float32)
    for h in torch.nonzero(dead.any(dim=1)).flatten().tolist():
        rows = torch.nonzero(dead[h]).flatten()
        w = m[rows]
        cnt = w.sum(1, keepdim=True)
        w = torch.where(cnt > 0, w / cnt.clamp_min(1.0), torch.full_like(w, float("nan")))
        x[rows, h] = (w @ v[:, h].float()).to(x.dtype)
    return x


def dense_attention(q, k, v, scale, dropout_p=0.0, seed=0, score_heads=None, check_status=True):
    """q, k, v: bf16 [s, H, D] -> (out [s, H, D], node_scores [s]); differentiable in q, k, v."""
    heads = q.shape[1]
    return _DenseAttention.apply(q, k, v, scale, dropout_p, seed & (2**64 - 1),
                                 heads if score_heads is None else score_heads, check_status)


def _combined_bias(attn_bias, pruning_mask, mask, s, heads, device):
    """attn_bias + pruning_mask as one fp32 [H or 1, s, s] tensor, masked entries -inf."""
    b = None
    for add in (attn_bias, pruning_mask):
        if add is None:
            continue
        a = add.to(device=device, dtype=torch.float32)
        while a.dim() > 3:
            if a.shape[0] != 1:
                raise ValueError("dense windows are one sequence: the bias batch dimension must be 1")
            a = a[0]
        b = a if b is None else b + a
    if b is None:
        b = torch.zeros(1, s, s, dtype=torch.float32, device=device)
    if b.dim() < 3:
        b = b.reshape((1,) * (3 - b.dim()) + tuple(b.shape))
    b = b.expand(1 if b.shape[0] == 1 else heads, s, s)      # one [s, s] shared by all heads, or one per head
    if mask is not None:
        b = b.masked_fill(mask.to(device=device, dtype=torch.bool).reshape(1, s, s), float("-inf"))
    return b.contiguous()


def full_attention(k, q, v, attn_bias=None, mask=None, pruning_mask=None, scale=None, dropout_p=0.0, seed=None,
                   check_status=True):
    _lib.require_cuda(q, k, v)
    b, s, heads, dim = q.shape
    if b != 1:
        raise ValueError("windows are one sequence (batch 1)")
    scale = math.sqrt(dim) if scale is None else scale
    if seed is None:
        seed = int(torch.randint(0, 2**62, (1,)).item()) if dropout_p > 0 else 0
    dt = q.dtype
    q3, k3, v3 = (t.reshape(s, heads, dim).to(torch.bfloat16).contiguous() for t in (q, k, v))
    if attn_bias is None and mask is None and pruning_mask is None:
        out, ns = dense_attention(q3, k3, v3, scale, dropout_p, seed, check_status=check_status)
    else:
        bias = _combined_bias(attn_bias, pruning_mask, mask, s, heads, q.device)
        out, ns, lse = _DenseAttentionBias.apply(q3, k3, v3, bias, scale, dropout_p, seed & (2**64 - 1), heads,
                                                 check_status)
        out = _masked_rows_fixup(out, lse.detach(), v3, mask)
    return out.to(dt).reshape(b, s, heads, dim), ns
