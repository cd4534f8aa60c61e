"""LayerNorm forward/backward and the column sum on csrc/rowops.cu against torch fp32."""
import pytest
import torch

from conftest import rel_err

pytestmark = pytest.mark.gpu

TOL = 1e-5   # fp32, relative (max|a-b| / max|b|); only the summation order differs from torch


@pytest.mark.parametrize("rows,cols", [(1, 4), (127, 40), (129, 64), (10583, 128), (3000, 256), (517, 768),
                                       (300, 1024)])
def test_layernorm_matches_torch(cuda, rows, cols):
    from neutrongt_b200.layers import LayerNorm
    g = torch.Generator(device="cuda").manual_seed(rows + cols)
    x = torch.randn(rows, cols, generator=g, device="cuda") * 3 + 1
    dy = torch.randn(rows, cols, generator=g, device="cuda")
    ours = LayerNorm(cols).cuda()
    ref = torch.nn.LayerNorm(cols).cuda()
    with torch.no_grad():
        for m in (ours, ref):
            m.weight.copy_(torch.linspace(0.5, 1.5, cols))
            m.bias.copy_(torch.linspace(-0.2, 0.2, cols))
    xa, xb = x.clone().requires_grad_(True), x.clone().requires_grad_(True)
    ya, yb = ours(xa), ref(xb)
    ya.backward(dy)
    yb.backward(dy)
    assert rel_err(ya, yb) < TOL
    assert rel_err(xa.grad, xb.grad) < TOL
    assert rel_err(ours.weight.grad, ref.weight.grad) < TOL
    assert rel_err(ours.bias.grad, ref.bias.grad) < TOL


def test_column_sum_is_deterministic_and_handles_empty(cuda):
    from neutrongt_b200.layers import column_sum
    x = torch.randn(20000, 96, device="cuda")
    a, b = column_sum(x), column_sum(x)
    assert torch.equal(a, b)
    assert rel_err(a, x.double().sum(0).float()) < TOL
    assert torch.equal(column_sum(torch.empty(0, 12, device="cuda")), torch.zeros(12, device="cuda"))
