"""Shared helpers for the parity tests: seeded inputs and the tolerance rule.

fp32 tolerance (written here once, used by every fp32 parity test):
    |y - y_ref| <= 1e-5 * scale[r] * sum_k |W[r,k] * x[s,k]| + 1e-30
i.e. 1e-5 relative to the condition of each output (plain relative error is
meaningless where the sum cancels to ~0).  int8 modes are compared bit for bit.
"""
from __future__ import annotations

import numpy as np

FP32_RTOL = 1e-5


def ternary_matrix(rng, rows, cols, p_zero=1 / 3):
    p = [(1 - p_zero) / 2, p_zero, (1 - p_zero) / 2]
    return rng.choice(np.array([-1, 0, 1], np.int8), size=rows * cols, p=p).astype(np.int8)


def condition(t, x, rows, cols, seq, scales):
    """scale[r] * sum_k |W[r,k] x[s,k]| as a [seq*rows] vector (float64)."""
    W = np.abs(t.reshape(rows, cols).astype(np.float64))
    X = np.abs(x.reshape(seq, cols).astype(np.float64))
    return (X @ W.T * np.abs(scales.astype(np.float64))[None, :]).ravel()


def assert_fp32_close(y, ref, cond, rtol=FP32_RTOL, what=""):
    y = np.asarray(y, np.float64).ravel()
    ref = np.asarray(ref, np.float64).ravel()
    err = np.abs(y - ref)
    tol = rtol * cond + 1e-30
    bad = np.nonzero(err > tol)[0]
    assert bad.size == 0, (f"{what}: {bad.size} outputs out of tolerance; worst index {bad[0]} "
                           f"y={y[bad[0]]!r} ref={ref[bad[0]]!r} err={err[bad[0]]:.3e} "
                           f"tol={tol[bad[0]]:.3e}")


def assert_bits_equal(y, ref, what=""):
    a = np.ascontiguousarray(y, np.float32).view(np.uint32).ravel()
    b = np.ascontiguousarray(ref, np.float32).view(np.uint32).ravel()
    bad = np.nonzero(a != b)[0]
    assert bad.size == 0, (f"{what}: {bad.size} outputs differ bitwise; first index {bad[0]}: "
                           f"{a[bad[0]]:#010x} vs {b[bad[0]]:#010x}")
