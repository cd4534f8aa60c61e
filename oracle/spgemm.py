"""Restatement of the row-wise sparse product C = A B (test oracle only).

Stands for `csr_spgemm` (`NeutronGT/core/ppr_backends/cusparse_ops.py:97-114`, cuSPARSE SpGEMM in
`csrc/cusparse_spgemm.cu:65-267`): fp32 CSR in, C [m x n] with the structural entries of the
product (cuSPARSE keeps entries whose products cancel), columns ascending.  Each value is the sum
of its products a_ij * b_jc taken in A's entry order, the first added to zero, every multiply and
add rounded to fp32 — the order of SciPy's row-wise csr_matmat, which the CPU tests hold this to
bit for bit (SciPy drops entries that sum to exactly zero; this keeps them, as cuSPARSE does).
Pure Python over the entries: for the small matrices of the tests.
"""
from __future__ import annotations

import numpy as np


def csr_spgemm(rowptr_a, col_a, val_a, rowptr_b, col_b, val_b):
    ra, ca, va = (np.asarray(x) for x in (rowptr_a, col_a, val_a))
    rb, cb, vb = (np.asarray(x) for x in (rowptr_b, col_b, val_b))
    va = va.astype(np.float32)
    vb = vb.astype(np.float32)
    m = ra.size - 1
    out_ptr = np.zeros(m + 1, dtype=np.int64)
    cols, vals = [], []
    for i in range(m):
        acc = {}
        for jj in range(ra[i], ra[i + 1]):
            j, a = int(ca[jj]), va[jj]
            for kk in range(rb[j], rb[j + 1]):
                c = int(cb[kk])
                prod = np.float32(a * vb[kk])
                acc[c] = np.float32(acc.get(c, np.float32(0.0)) + prod)
        keys = sorted(acc)
        cols.extend(keys)
        vals.extend(acc[k] for k in keys)
        out_ptr[i + 1] = out_ptr[i] + len(keys)
    return out_ptr, np.asarray(cols, dtype=np.int64), np.asarray(vals, dtype=np.float32)
