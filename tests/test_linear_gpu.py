"""fp32 Linear layers (forward, input grad, weight + bias grad) against torch.

Shapes with both dimensions <= 256 run the forward and input grad on the tensor cores with split
TF32 operands (csrc/linear_tc.cu), the others on fp32 FFMA (csrc/linear.cu); the weight grad runs
on the same tensor-core kernel when the input width is <= 256 and there are >= 64 rows, else on FFMA.
Tolerance: relative (max|a-b| / max|b|) against an fp64 torch restatement, 1e-5 -- fp32 precision
in a different summation order than cuBLAS; torch's own fp32 result is held to the same bound.
"""
import ctypes

import pytest
import torch

from conftest import rel_err

pytestmark = pytest.mark.gpu

TOL = 1e-5

# (rows, in, out): the GT / Graphormer window shapes, ragged and tiny row counts, the largest
# inner dimension kept on chip (256), several column tiles, many row tiles per CTA
# (30000, 128, 32) and (30000, 64, 40) are the row counts and narrow outputs for which the
# tensor-core Linear picks a 7- and a 6-slice TMA ring (149-296 row tiles, two CTAs per SM).
SHAPES = [(10583, 128, 128), (10583, 128, 256), (10583, 256, 128), (10583, 128, 64), (10583, 64, 32),
          (10583, 32, 40), (1, 4, 4), (5, 8, 12), (100, 64, 64), (1001, 256, 512), (200000, 128, 128),
          (3, 300, 8), (30000, 128, 32), (30000, 64, 40),
          (3000, 40, 24), (1000, 200, 136)]   # padded input widths and a ragged second output tile


def _ref(x, w, b, dy):
    xd, wd, bd, dyd = (t.double() for t in (x, w, b, dy))
    y = xd @ wd.t() + bd
    return y, dyd @ wd, dyd.t() @ xd, dyd.sum(0)


@pytest.mark.parametrize("rows,fin,fout", SHAPES)
def test_linear_matches_fp64(cuda, rows, fin, fout):
    from neutrongt_b200.layers import Linear
    g = torch.Generator(device="cuda").manual_seed(rows * 7 + fin + fout)
    x = torch.randn(1, rows, fin, generator=g, device="cuda")
    dy = torch.randn(1, rows, fout, generator=g, device="cuda")
    lin = Linear(fin, fout).cuda()
    xa = x.clone().requires_grad_(True)
    y = lin(xa)
    y.backward(dy)
    ry, rdx, rdw, rdb = _ref(x[0], lin.weight.detach(), lin.bias.detach(), dy[0])
    assert rel_err(y[0], ry) < TOL
    assert rel_err(xa.grad[0], rdx) < TOL
    assert rel_err(lin.weight.grad, rdw) < TOL
    assert rel_err(lin.bias.grad, rdb) < TOL
    # torch's fp32 Linear meets the same bound (the tolerance is fp32's, not loosened for us)
    ref = torch.nn.Linear(fin, fout).cuda()
    ref.load_state_dict(lin.state_dict())
    assert rel_err(ref(x)[0], ry) < TOL


def test_weight_grad_is_bitwise_reproducible(cuda):
    from neutrongt_b200.layers import Linear
    x = torch.randn(10583, 128, device="cuda")
    dy = torch.randn(10583, 256, device="cuda")
    lin = Linear(128, 256).cuda()
    grads = []
    for _ in range(3):
        lin.zero_grad(set_to_none=True)
        lin(x).backward(dy)
        grads.append((lin.weight.grad.clone(), lin.bias.grad.clone()))
    for w, b in grads[1:]:
        assert torch.equal(w, grads[0][0]) and torch.equal(b, grads[0][1])


def test_c_abi_without_bias_and_empty_rows(cuda):
    from neutrongt_b200 import _lib
    lib = _lib.lib()
    st = ctypes.c_void_p(torch.cuda.current_stream().cuda_stream)
    x = torch.randn(333, 96, device="cuda")
    w = torch.randn(20, 96, device="cuda")
    y = torch.empty(333, 20, device="cuda")
    assert lib.ngt_linear_forward(333, 96, 20, _lib.ptr(x), _lib.ptr(w), None, _lib.ptr(y), st) == 0
    assert rel_err(y, x.double() @ w.double().t()) < TOL
    dy = torch.randn(333, 20, device="cuda")
    dw = torch.full((20, 96), 7.0, device="cuda")
    ws = _lib.workspace(_lib.size_query(lib.ngt_linear_weight_workspace_size, 333, 96, 20), "cuda")
    assert lib.ngt_linear_backward_weight(333, 96, 20, _lib.ptr(x), _lib.ptr(dy), _lib.ptr(dw), None,
                                          _lib.ptr(ws), ws.numel(), st) == 0
    assert rel_err(dw, dy.double().t() @ x.double()) < TOL
    # zero rows: zero gradients; inner dimension above 256 is refused, not computed
    db = torch.full((20,), 3.0, device="cuda")
    assert lib.ngt_linear_backward_weight(0, 96, 20, None, None, _lib.ptr(dw), _lib.ptr(db), None, 0, st) == 0
    torch.cuda.synchronize()
    assert not dw.any() and not db.any()
    assert lib.ngt_linear_forward(4, 260, 8, _lib.ptr(x), _lib.ptr(w), None, _lib.ptr(y), st) == 2
    assert lib.ngt_linear_backward_input(4, 8, 260, _lib.ptr(x), _lib.ptr(w), _lib.ptr(y), st) == 2
    small = _lib.workspace(16, "cuda")
    assert lib.ngt_linear_backward_weight(333, 96, 20, _lib.ptr(x), _lib.ptr(dy), _lib.ptr(dw), None,
                                          _lib.ptr(small), 16, st) == 3


def test_weight_grads_on_side_stream_match(cuda):
    """overlap_weight_grads(): same gradients as the single-stream backward, bit for bit, and they
    are complete when backward() returns (the side stream joined the backward's stream)."""
    from neutrongt_b200.layers import Linear, overlap_weight_grads
    torch.manual_seed(0)
    net = torch.nn.Sequential(Linear(128, 256), torch.nn.ReLU(), Linear(256, 128), torch.nn.ReLU(),
                              Linear(128, 64)).cuda()
    x = torch.randn(10583, 128, device="cuda", requires_grad=True)
    grads = []
    for overlap in (False, True, True):
        net.zero_grad(set_to_none=True)
        x.grad = None
        with overlap_weight_grads(overlap):
            net(x).square().sum().backward()
        g = [p.grad.clone() for p in net.parameters()] + [x.grad.clone()]   # read right away
        grads.append(g)
    for g in grads[1:]:
        for a, b in zip(g, grads[0]):
            assert torch.equal(a, b)


def test_tensor_core_path_reports_no_timeouts(cuda):
    """The split-TF32 tcgen05 kernel (both dimensions <= 256) bounds its waits and counts any that
    run out; a normal forward + backward leaves the count at zero."""
    from neutrongt_b200 import _lib
    from neutrongt_b200.layers import Linear
    lin = Linear(128, 40).cuda()
    x = torch.randn(777, 128, device="cuda", requires_grad=True)
    lin(x).sum().backward()
    torch.cuda.synchronize()
    n = ctypes.c_int32(-1)
    assert _lib.lib().ngt_linear_status(ctypes.byref(n)) == 0
    assert n.value == 0


def test_inputs_near_flt_max_stay_finite(cuda):
    """Operands within 2^-11 of FLT_MAX split without carrying into the exponent, so the tensor-core
    forward stays finite and fp32-accurate where a naive round-up would give inf - inf = NaN."""
    from neutrongt_b200.layers import Linear
    x = torch.randn(300, 64, device="cuda") * 1e-3
    big = torch.tensor([0x7F7FF000, 0x7F7FFFFF, -0x00800800], dtype=torch.int32).view(torch.float32)
    x[:3, 5] = big.to("cuda")
    lin = Linear(64, 16).cuda()
    with torch.no_grad():
        lin.weight.mul_(1e-3)
    y = lin(x.unsqueeze(0))[0]
    ry = x.double() @ lin.weight.detach().double().t() + lin.bias.detach().double()
    assert bool(torch.isfinite(y).all())
    assert rel_err(y, ry) < TOL
