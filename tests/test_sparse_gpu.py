"""GPU parity of the 2:4 sparse path against the CPU oracle (through the C ABI).

Weights enter in the reference's two sparse layouts (host SparseTernaryMatrix,
src/model/sparse_ternary.rs:52-70, and the WGSL op's 5-bit groups,
src/compute/kernels/sparse_ternary.rs:71-100).  fp32: tolerance rule of
tests/helpers.py; int8: bit-exact.
"""
import numpy as np
import pytest
import torch

from oracle import oracle as fo
from tests.helpers import assert_bits_equal, assert_fp32_close, condition

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def gpu():
    assert torch.cuda.is_available()
    from ferrisres_b200 import gpu as g
    return g


def sparse24(rng, rows, cols):
    """Exactly two +-1 per group of 4 along K, positions uniform (BASELINE cfg3)."""
    ng = rows * cols // 4
    pats = np.array([(0, 1), (0, 2), (0, 3), (1, 2), (1, 3), (2, 3)])
    pos = pats[rng.integers(0, 6, size=ng)]
    t = np.zeros((ng, 4), np.int8)
    vals = rng.choice(np.array([-1, 1], np.int8), size=(ng, 2))
    np.put_along_axis(t, pos, vals, axis=1)
    return t.ravel()


# seq <= 4 runs on the decode GEMV (one or two n8 operand blocks), larger seq on the engine
SHAPES = [(4, 4, 1), (130, 200, 3), (300, 512, 5), (14336, 4096, 1), (256, 1408, 9), (64, 20, 17),
          (2050, 1412, 2), (129, 4100, 4)]


@pytest.mark.parametrize("rows,cols,seq", SHAPES)
def test_sparse_host_layout_f32(gpu, rows, cols, seq):
    rng = np.random.default_rng(rows + 3 * cols + seq)
    t = sparse24(rng, rows, cols)
    rs = rng.uniform(0.01, 0.1, rows).astype(np.float32)
    x = rng.standard_normal(seq * cols).astype(np.float32)
    pat, sg = fo.sparse_from_ternary(t, rows, cols)
    w = gpu.DeviceTernaryWeight.from_sparse_host(pat, sg, rows, cols, rs)
    y = w.matmul_f32(torch.from_numpy(x).cuda().view(seq, cols)).cpu().numpy()
    ref = fo.sparse_ternary_matmul(pat, sg, 0.0, rs, rows, cols, x, seq)
    assert_fp32_close(y, ref, condition(t, x, rows, cols, seq, rs), what=f"{rows}x{cols}x{seq}")


@pytest.mark.parametrize("rows,cols,seq", [(300, 512, 2), (2050, 1412, 12), (129, 4100, 16),
                                           (14336, 4096, 64)])
def test_sparse_i8_bit_exact(gpu, rows, cols, seq):
    rng = np.random.default_rng(rows * 5 + seq)
    t = sparse24(rng, rows, cols)
    rs = rng.uniform(0.01, 0.1, rows).astype(np.float32)
    x = rng.standard_normal(seq * cols).astype(np.float32)
    q, sx = fo.quantize_absmax_i8(x, seq, cols)
    pat, sg = fo.sparse_from_ternary(t, rows, cols)
    w = gpu.DeviceTernaryWeight.from_sparse_host(pat, sg, rows, cols, rs)
    y = w.matmul_i8(torch.from_numpy(q).cuda().view(seq, cols), torch.from_numpy(sx).cuda())
    ref = fo.ternary_matmul_i8(t, q, sx, rs, seq, cols, rows)
    assert_bits_equal(y.cpu().numpy(), ref, what=f"sparse i8 {rows}x{cols}x{seq}")


def test_sparse_cfg3_m64_f32(gpu):
    """BASELINE config 3 at M=64: K=4096, N=14336."""
    rng = np.random.default_rng(64)
    rows, cols, seq = 14336, 4096, 64
    t = sparse24(rng, rows, cols)
    rs = rng.uniform(0.01, 0.1, rows).astype(np.float32)
    x = rng.standard_normal(seq * cols).astype(np.float32)
    pat, sg = fo.sparse_from_ternary(t, rows, cols)
    w = gpu.DeviceTernaryWeight.from_sparse_host(pat, sg, rows, cols, rs)
    y = w.matmul_f32(torch.from_numpy(x).cuda().view(seq, cols)).cpu().numpy()
    ref = fo.sparse_ternary_matmul(pat, sg, 0.0, rs, rows, cols, x, seq)
    assert_fp32_close(y, ref, condition(t, x, rows, cols, seq, rs), what="cfg3 M=64")


def test_sparse_wgsl_layout_and_accelerator(gpu):
    rng = np.random.default_rng(9)
    rows, cols, seq = 200, 96, 3
    t = sparse24(rng, rows, cols)
    rs = rng.uniform(0.01, 0.1, rows).astype(np.float32)
    x = rng.standard_normal(seq * cols).astype(np.float32)
    words = fo.sparse_wgsl_pack(t, rows, cols)
    ref = fo.sparse_wgsl_ref(words, rs, x, seq, cols, rows)
    w = gpu.DeviceTernaryWeight.from_sparse_wgsl(words, rows, cols, rs)
    y = w.matmul_f32(torch.from_numpy(x).cuda().view(seq, cols)).cpu().numpy()
    assert_fp32_close(y, ref, condition(t, x, rows, cols, seq, rs), what="wgsl layout")
    # GpuMatmulAccelerator::gpu_sparse_ternary_matmul: one global scale
    acc = gpu.GpuMatmulAccelerator()
    y2 = acc.gpu_sparse_ternary_matmul(words, 0.5, x, seq, cols, rows)
    ref2 = fo.sparse_wgsl_ref(words, np.full(rows, 0.5, np.float32), x, seq, cols, rows)
    assert_fp32_close(y2, ref2, condition(t, x, rows, cols, seq, np.full(rows, 0.5)), what="accel")


def test_sparse_reference_kats_on_gpu(gpu):
    # src/model/sparse_ternary.rs:419-432: all +1 on positions 0,1, scale 2 -> 16
    t = np.array([1, 1, 0, 0, 1, 1, 0, 0], np.int8)
    pat, sg = fo.sparse_from_ternary(t, 2, 4)
    w = gpu.DeviceTernaryWeight.from_sparse_host(pat, sg, 2, 4, [2.0, 2.0])
    y = w.matmul_f32(torch.tensor([[3.0, 5.0, 7.0, 11.0]], device="cuda")).cpu().numpy()
    assert np.allclose(y, [[16.0, 16.0]], atol=1e-5)
    # src/compute/kernels/sparse_ternary.rs:362-384: identity-ish rows -> 3, 4, 6, 7
    t = np.array([1, 1, 0, 0, 1, 0, 1, 0, 0, 1, 0, 1, 0, 0, 1, 1], np.int8)
    w = gpu.DeviceTernaryWeight.from_sparse_wgsl(fo.sparse_wgsl_pack(t, 4, 4), 4, 4, np.ones(4))
    y = w.matmul_f32(torch.tensor([[1.0, 2.0, 3.0, 4.0]], device="cuda")).cpu().numpy()
    assert np.allclose(y, [[3, 4, 6, 7]], atol=1e-5)


def test_sparse_grouped_and_bytes(gpu):
    rng = np.random.default_rng(12)
    rows, cols = 1408, 2048
    ws, ys, refs, conds = [], [], [], []
    x = rng.standard_normal(cols).astype(np.float32)
    xt = torch.from_numpy(x).cuda().view(1, cols)
    for i in range(3):
        t = sparse24(rng, rows, cols)
        rs = rng.uniform(0.01, 0.1, rows).astype(np.float32)
        pat, sg = fo.sparse_from_ternary(t, rows, cols)
        ws.append(gpu.DeviceTernaryWeight.from_sparse_host(pat, sg, rows, cols, rs))
        ys.append(torch.empty(1, rows, device="cuda"))
        refs.append(fo.sparse_ternary_matmul(pat, sg, 0.0, rs, rows, cols, x, 1))
        conds.append(condition(t, x, rows, cols, 1, rs))
    gpu.GroupCall(ws, [xt] * 3, ys)()
    for y, ref, c in zip(ys, refs, conds):
        assert_fp32_close(y.cpu().numpy(), ref, c, what="sparse grouped")
    # 1.5 bits/weight on the device (metadata nibble + 2 sign bits per group; plus row scales)
    assert ws[0].device_bytes() == (rows // 128 + (rows % 128 > 0)) * (cols // 128) * 3072 + \
        (rows + 127) // 128 * 128 * 4
    gpu.get_context().check()
