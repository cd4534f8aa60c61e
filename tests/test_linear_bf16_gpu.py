"""bf16 Linear layers of the large model on the tcgen05 tensor cores (`csrc/gemm_bf16.cu`).

The reference's GPH_Large projections (`…single_window.py:235-237, 313-318`; graphormer
`:139, 179, 183`) are torch Linear layers; trained in bf16 they compute with bf16 operands and
fp32 accumulation.  Here the forward, input gradient and weight / bias gradients are checked
against an fp32 product of the same bf16 operands, within the bf16 tolerance 2e-2 (relative,
max|a-b| / max|b|); the only extra error is the final bf16 rounding (~4e-3).
"""
import ctypes

import pytest
import torch

from conftest import rel_err

pytestmark = pytest.mark.gpu
BF16_TOL = 2e-2

# GPH_Large window rows x (768 -> 768), the fused-QKV and FFN widths, a class layer (40 outputs,
# BN = 128 tiles), odd row counts and feature counts that are multiples of 8 but not of 64
SHAPES = [(32768, 768, 768), (10000, 768, 2304), (4099, 768, 3072), (4099, 3072, 768), (1000, 768, 40),
          (300, 256, 128), (5, 8, 16), (129, 136, 264), (70000, 64, 64)]


def _data(rows, fin, fout, seed):
    g = torch.Generator(device="cuda").manual_seed(seed)
    x = torch.randn(rows, fin, generator=g, device="cuda").to(torch.bfloat16)
    w = (torch.randn(fout, fin, generator=g, device="cuda") / fin ** 0.5).to(torch.bfloat16)
    b = torch.randn(fout, generator=g, device="cuda").to(torch.bfloat16)
    dy = torch.randn(rows, fout, generator=g, device="cuda").to(torch.bfloat16)
    return x, w, b, dy


@pytest.mark.parametrize("rows,fin,fout", SHAPES)
def test_bf16_linear_matches_fp32_product(cuda, rows, fin, fout):
    from neutrongt_b200.layers import Linear
    x, w, b, dy = _data(rows, fin, fout, rows + fin + fout)
    lin = Linear(fin, fout).cuda().to(torch.bfloat16)
    with torch.no_grad():
        lin.weight.copy_(w)
        lin.bias.copy_(b)
    xa = x.clone().requires_grad_(True)
    y = lin(xa)
    y.backward(dy)
    assert y.dtype == torch.bfloat16 and lin.weight.grad.dtype == torch.bfloat16
    xf, wf, bf, dyf = (t.float() for t in (x, w, b, dy))
    errs = {"y": rel_err(y, xf @ wf.t() + bf), "dx": rel_err(xa.grad, dyf @ wf),
            "dw": rel_err(lin.weight.grad, dyf.t() @ xf), "db": rel_err(lin.bias.grad, dyf.sum(0))}
    assert all(e < BF16_TOL for e in errs.values()), errs


def test_bf16_linear_without_bias_and_3d_input(cuda):
    from neutrongt_b200.layers import Linear
    x, w, _, dy = _data(2 * 777, 128, 96, 5)
    lin = Linear(128, 96, bias=False).cuda().to(torch.bfloat16)
    with torch.no_grad():
        lin.weight.copy_(w)
    xa = x.view(2, 777, 128).clone().requires_grad_(True)
    y = lin(xa)
    y.backward(dy.view(2, 777, 96))
    assert y.shape == (2, 777, 96)
    assert rel_err(y.reshape(-1, 96), x.float() @ w.float().t()) < BF16_TOL
    assert rel_err(xa.grad.reshape(-1, 128), dy.float() @ w.float()) < BF16_TOL
    assert rel_err(lin.weight.grad, dy.float().t() @ x.float()) < BF16_TOL


def test_bf16_weight_grad_is_bitwise_reproducible(cuda):
    from neutrongt_b200.layers import Linear
    x, w, b, dy = _data(20000, 768, 768, 9)
    lin = Linear(768, 768).cuda().to(torch.bfloat16)
    grads = []
    for _ in range(3):
        lin.zero_grad(set_to_none=True)
        lin(x).backward(dy)
        grads.append((lin.weight.grad.clone(), lin.bias.grad.clone()))
    for gw, gb in grads[1:]:
        assert torch.equal(gw, grads[0][0]) and torch.equal(gb, grads[0][1])


def test_bf16_c_abi_edges(cuda):
    from neutrongt_b200 import _lib
    lib = _lib.lib()
    st = ctypes.c_void_p(torch.cuda.current_stream().cuda_stream)
    x = torch.randn(64, 32, device="cuda").to(torch.bfloat16)
    w = torch.randn(16, 32, device="cuda").to(torch.bfloat16)
    y = torch.empty(64, 16, device="cuda", dtype=torch.bfloat16)
    assert lib.ngt_linear_bf16_forward(64, 30, 16, _lib.ptr(x), _lib.ptr(w), None, _lib.ptr(y), st) == 1
    assert lib.ngt_linear_bf16_forward(0, 32, 16, None, None, None, None, st) == 0
    dw = torch.full((16, 32), 7.0, device="cuda").to(torch.bfloat16)
    db = torch.full((16,), 7.0, device="cuda").to(torch.bfloat16)
    assert lib.ngt_linear_bf16_backward_weight(0, 32, 16, None, None, _lib.ptr(dw), _lib.ptr(db), None, 0, st) == 0
    torch.cuda.synchronize()
    assert not dw.any() and not db.any()
    small = _lib.workspace(16, "cuda")
    assert lib.ngt_linear_bf16_backward_weight(64, 32, 16, _lib.ptr(x), _lib.ptr(y), _lib.ptr(dw), None,
                                               _lib.ptr(small), 16, st) == 3
    n = ctypes.c_int32(-1)
    assert lib.ngt_linear_status(ctypes.byref(n)) == 0 and n.value == 0
