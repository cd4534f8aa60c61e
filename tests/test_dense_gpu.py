"""Dense full-attention window (tcgen05 kernels), forward and backward:

* against the reference's own `CoreAttention.full_attention` outputs (tests/golden/dense_attention.pt,
  fp64 autograd of the reference module on bf16-representable inputs);
* against `oracle/dense.py` (the restatement pinned to those outputs) in fp32 on the GPU, at shapes
  up to the GPH_Large per-rank window (32,768 tokens, 4 heads, head_dim 24), element by element.

bf16 tolerance: 2e-2 relative (max|a-b| / max|b|)."""
import math

import numpy as np
import pytest
import torch

from conftest import golden, rel_err

pytestmark = pytest.mark.gpu
BF16_TOL = 2e-2


def _mix32(x):
    m = np.uint64(0xFFFFFFFF)
    x = x & m
    x ^= x >> np.uint64(16)
    x = (x * np.uint64(0x7FEB352D)) & m
    x ^= x >> np.uint64(15)
    x = (x * np.uint64(0x846CA68B)) & m
    x ^= x >> np.uint64(16)
    return x


def keep_mask(seed, s, heads, p):
    """The kernels' dropout keep decisions, restated in numpy: [H, s, s] bool."""
    sd = np.uint64((seed ^ (seed >> 32)) & 0xFFFFFFFF)
    thr = np.uint64(min(int(p * 2**32), 2**32 - 1))
    m = np.uint64(0xFFFFFFFF)
    i = np.arange(s, dtype=np.uint64)[None, :, None]
    j = np.arange(s, dtype=np.uint64)[None, None, :]
    h = np.arange(heads, dtype=np.uint64)[:, None, None]
    inner = _mix32((i * np.uint64(0x9E3779B1) + h * np.uint64(0x85EBCA77)) & m)
    x = _mix32(sd ^ inner ^ ((j * np.uint64(0xC2B2AE3D)) & m))
    return torch.from_numpy(x >= thr)


def _reference(q, k, v, scale, keep=None, p=0.0):
    """fp32 oracle; returns (x [s, H, D], node_scores) with autograd through q, k, v."""
    from oracle import dense as odense
    return odense.full_attention(k.float(), q.float(), v.float(), scale=scale, keep=keep, dropout_p=p)


@pytest.mark.parametrize("case", ["d24_h4", "d16_h2", "d8_h3", "d64_h2", "d40_h1"])
def test_matches_reference_fixture(cuda, case):
    """The public `full_attention(k, q, v, ...)` against the reference module's own fp64 results."""
    from neutrongt_b200.dense_attention import full_attention
    c = golden("dense_attention.pt")[case]
    q, k, v, g = (c[n].to(cuda) for n in ("q", "k", "v", "dout"))
    qd, kd, vd = (t.clone().requires_grad_(True) for t in (q, k, v))
    x, ns = full_attention(kd, qd, vd, None, None, None)
    x.backward(g)
    assert x.shape == c["x"].shape
    errs = {"x": rel_err(x, c["x"]), "node_scores": rel_err(ns, c["node_scores"]), "dq": rel_err(qd.grad, c["dq"]),
            "dk": rel_err(kd.grad, c["dk"]), "dv": rel_err(vd.grad, c["dv"])}
    assert all(e < BF16_TOL for e in errs.values()), errs


def test_gph_large_window_elementwise(cuda):
    """The GPH_Large per-rank dense window: 32,768 tokens, 4 heads, head_dim 24, dropout 0.  Every
    element of x, node_scores, dq, dk and dv against the chunked fp32 oracle on the GPU."""
    from neutrongt_b200.dense_attention import dense_attention
    from oracle import dense as odense
    s, H, D = 32768, 4, 24
    q, k, v, dout = _inputs(s, H, D, 2024)
    qd, kd, vd = (t.clone().requires_grad_(True) for t in (q, k, v))
    x, ns = dense_attention(qd, kd, vd, math.sqrt(D))
    x.backward(dout)
    rx, rns, rdq, rdk, rdv = odense.full_attention_chunked(q, k, v, dout)
    errs = {"x": rel_err(x, rx), "node_scores": rel_err(ns, rns), "dq": rel_err(qd.grad, rdq),
            "dk": rel_err(kd.grad, rdk), "dv": rel_err(vd.grad, rdv)}
    assert all(e < BF16_TOL for e in errs.values()), errs


def _inputs(s, H, D, seed):
    g = torch.Generator(device="cuda").manual_seed(seed)
    return [torch.randn(s, H, D, generator=g, device="cuda").to(torch.bfloat16) * 0.5 for _ in range(4)]


@pytest.mark.parametrize("s,H,D", [(128, 1, 32), (128, 2, 24), (200, 4, 24), (1000, 2, 16), (300, 1, 64),
                                   (1024, 4, 24), (129, 1, 16), (640, 1, 24), (1500, 3, 8), (4096, 2, 32),
                                   (700, 2, 40)])
def test_forward_and_backward_match_reference(cuda, s, H, D):
    from neutrongt_b200.dense_attention import dense_attention
    q, k, v, dout = _inputs(s, H, D, s + H + D)
    qd, kd, vd = (t.clone().requires_grad_(True) for t in (q, k, v))
    x, ns = dense_attention(qd, kd, vd, math.sqrt(D))
    x.backward(dout)
    qr, kr, vr = (t.float().clone().requires_grad_(True) for t in (q, k, v))
    rx, rns = _reference(qr, kr, vr, math.sqrt(D))
    rx.backward(dout.float())
    assert x.shape == (s, H, D)
    assert rel_err(x, rx) < BF16_TOL
    assert rel_err(ns, rns) < BF16_TOL
    assert rel_err(qd.grad, qr.grad) < BF16_TOL
    assert rel_err(kd.grad, kr.grad) < BF16_TOL
    assert rel_err(vd.grad, vr.grad) < BF16_TOL


def test_dropout_matches_mask_restatement(cuda):
    from neutrongt_b200.dense_attention import dense_attention
    s, H, D, p, seed = 256, 2, 24, 0.5, 123456789
    q, k, v, dout = _inputs(s, H, D, 7)
    qd, kd, vd = (t.clone().requires_grad_(True) for t in (q, k, v))
    x, _ = dense_attention(qd, kd, vd, math.sqrt(D), dropout_p=p, seed=seed)
    x.backward(dout)
    keep = keep_mask(seed, s, H, p)
    assert 0.45 < float(keep.float().mean()) < 0.55
    qr, kr, vr = (t.float().clone().requires_grad_(True) for t in (q, k, v))
    rx, _ = _reference(qr, kr, vr, math.sqrt(D), keep=keep, p=p)
    rx.backward(dout.float())
    assert rel_err(x, rx) < BF16_TOL
    assert rel_err(qd.grad, qr.grad) < BF16_TOL
    assert rel_err(kd.grad, kr.grad) < BF16_TOL
    assert rel_err(vd.grad, vr.grad) < BF16_TOL


def test_full_attention_contract(cuda):
    from neutrongt_b200 import CoreAttention
    s, H, D = 300, 4, 24
    q, k, v, _ = _inputs(s, H, D, 9)
    attn = CoreAttention(H * D, 0.0, H).eval()
    x, score = attn(q.unsqueeze(0), k.unsqueeze(0), v.unsqueeze(0), None, None, "full")
    rx, rns = _reference(q, k, v, math.sqrt(D))
    assert x.shape == (1, s, H * D)
    assert rel_err(x.reshape(s, H, D), rx) < BF16_TOL
    assert rel_err(score, rns) < BF16_TOL


def test_status_word_reports_a_timeout_without_a_host_wait(cuda):
    """A timeout recorded in the device status word (set here from the host: no wait is made
    to run out) is raised by `check_dense_status` once, and cleared after the report."""
    from neutrongt_b200.dense_attention import _StatusWord, check_dense_status, dense_attention
    s, H, D = 256, 2, 24
    q, k, v, dout = _inputs(s, H, D, 11)
    check_dense_status()
    sw = _StatusWord.of(q.device)
    sw.word.fill_(1)
    qd = q.clone().requires_grad_(True)
    x, _ = dense_attention(qd, k, v, math.sqrt(D))     # launches and publishes the word
    with pytest.raises(RuntimeError, match="timed out"):
        check_dense_status()
    check_dense_status()                                  # reported once, then clear
    x, _ = dense_attention(qd, k, v, math.sqrt(D))
    x.backward(dout)
    check_dense_status()
    assert int(sw.word.item()) == 0


# ---------------- attn_bias / pruning_mask / mask (`…single_window.py:78-99`) ----------------

@pytest.mark.parametrize("case", ["bias_d16", "bias_pruning_mask_d24", "mask_d64"])
def test_bias_and_masks_match_reference_fixture(cuda, case):
    """attn_bias and pruning_mask added to the scores, masked entries filled with -1e9 (one query row
    entirely masked): outputs and the gradients of q, k, v, attn_bias and pruning_mask against the
    reference module's own fp64 results."""
    from neutrongt_b200.dense_attention import full_attention
    c = golden("dense_attention.pt")[case]
    q, k, v, g = (c[n].to(cuda) for n in ("q", "k", "v", "dout"))
    qd, kd, vd = (t.clone().requires_grad_(True) for t in (q, k, v))
    b = c["attn_bias"].to(cuda).requires_grad_(True) if c["attn_bias"] is not None else None
    pm = c["pruning_mask"].to(cuda).requires_grad_(True) if c["pruning_mask"] is not None else None
    mask = c["mask"].to(cuda) if c["mask"] is not None else None
    x, ns = full_attention(kd, qd, vd, b, mask=mask, pruning_mask=pm)
    x.backward(g)
    errs = {"x": rel_err(x, c["x"]), "node_scores": rel_err(ns, c["node_scores"]), "dq": rel_err(qd.grad, c["dq"]),
            "dk": rel_err(kd.grad, c["dk"]), "dv": rel_err(vd.grad, c["dv"])}
    if b is not None:
        errs["dbias"] = rel_err(b.grad, c["dbias"])
    if pm is not None:
        errs["dpruning"] = rel_err(pm.grad, c["dpruning"])
    assert all(e < BF16_TOL for e in errs.values()), errs
    assert torch.isfinite(x).all()


@pytest.mark.parametrize("s,H,D,shared", [(1000, 4, 24, False), (777, 2, 64, True), (300, 3, 16, False)])
def test_bias_against_oracle(cuda, s, H, D, shared):
    from neutrongt_b200.dense_attention import full_attention
    from oracle import dense as odense
    q, k, v, dout = _inputs(s, H, D, s + D)
    g = torch.Generator(device="cuda").manual_seed(s)
    bias = torch.randn(1, 1 if shared else H, s, s, generator=g, device="cuda")
    mask = torch.rand(s, s, generator=g, device="cuda") < 0.2
    qd, kd, vd = (t.clone().unsqueeze(0).requires_grad_(True) for t in (q, k, v))
    bd = bias.clone().requires_grad_(True)
    x, ns = full_attention(kd, qd, vd, bd, mask=mask)
    x.backward(dout.unsqueeze(0))
    qr, kr, vr = (t.float().unsqueeze(0).clone().requires_grad_(True) for t in (q, k, v))
    br = bias.clone().requires_grad_(True)
    rx, rns = odense.full_attention(kr, qr, vr, br, mask=mask)
    rx.backward(dout.float().unsqueeze(0))
    errs = {"x": rel_err(x, rx), "ns": rel_err(ns, rns), "dq": rel_err(qd.grad, qr.grad), "dk": rel_err(kd.grad, kr.grad),
            "dv": rel_err(vd.grad, vr.grad), "dbias": rel_err(bd.grad, br.grad)}
    assert all(e < BF16_TOL for e in errs.values()), errs


def test_bias_with_dropout_matches_mask_restatement(cuda):
    from neutrongt_b200.dense_attention import full_attention
    from oracle import dense as odense
    s, H, D, p, seed = 256, 2, 24, 0.3, 987654321
    q, k, v, dout = _inputs(s, H, D, 17)
    bias = torch.randn(1, H, s, s, device="cuda")
    qd, kd, vd = (t.clone().unsqueeze(0).requires_grad_(True) for t in (q, k, v))
    x, _ = full_attention(kd, qd, vd, bias, dropout_p=p, seed=seed)
    x.backward(dout.unsqueeze(0))
    keep = keep_mask(seed, s, H, p)
    qr, kr, vr = (t.float().unsqueeze(0).clone().requires_grad_(True) for t in (q, k, v))
    rx, _ = odense.full_attention(kr, qr, vr, bias, keep=keep, dropout_p=p)
    rx.backward(dout.float().unsqueeze(0))
    assert rel_err(x, rx) < BF16_TOL
    assert rel_err(qd.grad, qr.grad) < BF16_TOL and rel_err(kd.grad, kr.grad) < BF16_TOL
    assert rel_err(vd.grad, vr.grad) < BF16_TOL
