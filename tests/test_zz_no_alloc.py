"""The allocation-free matmul entry point, checked against the regular one.

`ft_ternary_matmul_f32_noalloc` exists for callers that must not let the
library allocate device memory inside a call (a host that owns all device
memory, or a loop that cannot take cudaMalloc's device-wide synchronisation).
It keeps its scratch in a fixed array inside the library image instead of a
context workspace.  This test calls it through the C ABI twice in a row and
compares each result with `ft_ternary_matmul_f32` on the same inputs, under the
fp32 tolerance rule the other parity tests use; it also checks that shapes
beyond its stated limits are refused with FT_ERR_UNSUPPORTED.

The file name makes pytest collect it last, so a run that stops at the first
failure has already run every other test.  It also passes on its own in a
fresh process.
"""
import ctypes as C

import numpy as np
import pytest
import torch

from oracle import oracle as fo
from tests.helpers import assert_fp32_close, condition, ternary_matrix

pytestmark = pytest.mark.gpu


def _ptr(t):
    return C.c_void_p(t.data_ptr())


@pytest.mark.parametrize("rows,cols,seq", [(5632, 2048, 1), (300, 1000, 3), (16384, 512, 4)])
def test_noalloc_matches_regular_entry_point_twice(rows, cols, seq):
    from ferrisres_b200 import _lib, gpu

    L = _lib.lib()
    ctx = gpu.get_context(0)
    stream = C.c_void_p(torch.cuda.current_stream().cuda_stream)
    rng = np.random.default_rng(rows + cols + seq)
    t = ternary_matrix(rng, rows, cols)
    rs = rng.uniform(0.01, 0.1, rows).astype(np.float32)
    w = gpu.DeviceTernaryWeight.from_packed_u8(fo.pack_ternary(t), rows, cols, rs)
    for call in range(2):  # two calls in a row share (and must re-clear) the scratch
        x = rng.standard_normal(seq * cols).astype(np.float32)
        xd = torch.from_numpy(x).cuda()
        y_reg = torch.full((seq, rows), float("nan"), device="cuda")
        y_na = torch.full((seq, rows), float("nan"), device="cuda")
        rc = L.ft_ternary_matmul_f32(ctx.handle, w.handle, seq, _ptr(xd), _ptr(y_reg), stream)
        assert rc == 0, L.ft_last_error_string()
        rc = L.ft_ternary_matmul_f32_noalloc(ctx.handle, w.handle, seq, _ptr(xd), _ptr(y_na),
                                             stream)
        assert rc == 0, L.ft_last_error_string()
        torch.cuda.synchronize()
        assert_fp32_close(y_na.cpu().numpy(), y_reg.cpu().numpy(),
                          condition(t, x, rows, cols, seq, rs), what=f"no-alloc call {call}")
    ctx.check()  # no bounded wait inside a kernel gave up


def test_noalloc_rejects_shapes_beyond_its_limits():
    from ferrisres_b200 import _lib, gpu

    L = _lib.lib()
    ctx = gpu.get_context(0)
    stream = C.c_void_p(torch.cuda.current_stream().cuda_stream)
    w = gpu.DeviceTernaryWeight.from_ternary(np.ones(16 * 64, np.int8), 16, 64, np.ones(16))
    x = torch.zeros(5, 64, device="cuda")
    y = torch.zeros(5, 16, device="cuda")
    rc = L.ft_ternary_matmul_f32_noalloc(ctx.handle, w.handle, 5, _ptr(x), _ptr(y), stream)
    assert rc == 4 and b"no-alloc" in L.ft_last_error_string()
    wide = gpu.DeviceTernaryWeight.from_ternary(np.ones(16400, np.int8), 1, 16400, np.ones(1))
    xw = torch.zeros(1, 16400, device="cuda")
    rc = L.ft_ternary_matmul_f32_noalloc(ctx.handle, wide.handle, 1, _ptr(xw), _ptr(y), stream)
    assert rc == 4
