"""The split-TF32 arithmetic of the tensor-core Linear (csrc/linear_tc.cu), restated in numpy.

Each fp32 operand x is split into hi = x rounded to tf32 (10 mantissa bits; the kernel adds 0x1000
to the bit pattern and clears the low 13 bits) and lo = x - hi; a product is hi_a hi_b + hi_a lo_b
+ lo_a hi_b.  The tensor core reads lo as tf32 too; here lo is truncated to tf32 (the worse of
truncation and rounding) and the products are summed in fp64, so this isolates the error of the
split itself (~1e-7 relative here; the kernel's fp32 accumulation adds fp32's own rounding on top,
~1e-6 measured on the GPU, like fp32 FFMA).  It must stay well inside the 1e-5 relative tolerance
the GPU tests hold the kernel and torch's fp32 Linear to, while plain tf32 (hi only, ~3e-4) must
not: the split is what keeps the model fp32.
"""
import numpy as np
import pytest


def _tf32_round(x):
    b = x.astype(np.float32).view(np.uint32)
    finite = (b & 0x7F800000) != 0x7F800000
    r = (b + np.uint32(0x1000)) & np.uint32(0xFFFFE000)
    r = np.where((r & 0x7F800000) == 0x7F800000, b & np.uint32(0xFFFFE000), r)   # no carry into inf
    r = np.where(finite, r, b)
    return r.astype(np.uint32).view(np.float32)


def _tf32_trunc(x):
    return (x.astype(np.float32).view(np.uint32) & np.uint32(0xFFFFE000)).view(np.float32)


def _split(x):
    hi = _tf32_round(x)
    lo = (x - hi).astype(np.float32)          # exact in fp32
    return hi, _tf32_trunc(lo)


def _split_gemm(a, w):
    ah, al = _split(a)
    wh, wl = _split(w)
    d = lambda u, v: u.astype(np.float64) @ v.astype(np.float64).T
    return (d(al, wh) + d(ah, wl) + d(ah, wh)).astype(np.float32)


def _rel(x, ref):
    return float(np.abs(x.astype(np.float64) - ref).max() / np.abs(ref).max())


def test_rounding_matches_the_definition():
    x = np.array([1.0, 1.0 + 2.0 ** -11, 1.0 + 2.0 ** -10, -3.14159265, 1e-30, 0.0], dtype=np.float32)
    hi = _tf32_round(x)
    assert (hi.view(np.uint32) & 0x1FFF == 0).all()                      # 10 mantissa bits left
    assert hi[0] == 1.0 and hi[2] == np.float32(1.0 + 2.0 ** -10)
    assert hi[1] == np.float32(1.0 + 2.0 ** -10)                          # tie rounds away from zero
    assert np.all(np.abs(x - hi) <= np.abs(x) * 2.0 ** -11 + 1e-45)
    inf = np.array([np.inf, -np.inf], dtype=np.float32)
    assert np.array_equal(_tf32_round(inf), inf)                          # non-finite kept


def test_split_near_flt_max_stays_finite():
    """Within 2^-11 of FLT_MAX, rounding up would carry into the exponent (hi = inf, lo = -inf,
    so hi * w + lo * w is NaN); the split truncates there and hi + lo is still exactly x."""
    big = np.array([0x7F7FF000, 0x7F7FFFFF, 0xFF7FF800, 0x7F7FE000], dtype=np.uint32).view(np.float32)
    hi = _tf32_round(big)
    assert np.isfinite(hi).all()
    lo = (big - hi).astype(np.float32)
    assert np.array_equal((hi.astype(np.float64) + lo.astype(np.float64)).astype(np.float32), big)
    w = np.full((1, 4), 1e-3, dtype=np.float32)
    y = _split_gemm(big[None, :], w)
    assert np.isfinite(y).all()
    assert _rel(y, big[None, :].astype(np.float64) @ w.astype(np.float64).T) < 1e-5


@pytest.mark.parametrize("rows,fin,fout", [(2048, 128, 128), (1024, 256, 128), (1024, 128, 256), (777, 100, 40)])
def test_split_tf32_keeps_fp32_accuracy(rows, fin, fout):
    g = np.random.default_rng(rows + fin + fout)
    x = g.standard_normal((rows, fin)).astype(np.float32)
    w = (g.standard_normal((fout, fin)) / np.sqrt(fin)).astype(np.float32)
    ref = x.astype(np.float64) @ w.astype(np.float64).T
    split = _split_gemm(x, w)
    plain = (_tf32_round(x).astype(np.float64) @ _tf32_round(w).astype(np.float64).T).astype(np.float32)
    fp32 = (x @ w.T).astype(np.float32)
    assert _rel(split, ref) < 1e-5
    assert _rel(split, ref) < 4 * max(_rel(fp32, ref), 2.0 ** -24)        # fp32's own error, within a small factor
    assert _rel(plain, ref) > 1e-4                                         # tf32 alone would fail the bar
