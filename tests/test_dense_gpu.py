"""GPU parity of the dense ternary path against the CPU oracle (through the C ABI).

fp32 activations: tolerance rule of tests/helpers.py (1e-5 of each output's
condition).  int8 activations: bit-exact.
"""
import numpy as np
import pytest
import torch

from oracle import oracle as fo
from tests.helpers import assert_bits_equal, assert_fp32_close, condition, ternary_matrix

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def gpu():
    assert torch.cuda.is_available()
    from ferrisres_b200 import gpu as g
    return g


SHAPES = [  # (rows, cols, seq) incl. ragged edges (rows % 128, cols % 128, cols % 16 != 0)
    (1, 4, 1), (7, 6, 2), (128, 128, 1), (130, 200, 3), (300, 512, 5), (5632, 2048, 1),
    (256, 1408, 9), (2048, 1408, 4), (129, 4100, 2), (64, 20, 17)]


@pytest.mark.parametrize("rows,cols,seq", SHAPES)
def test_f32_matches_oracle(gpu, rows, cols, seq):
    rng = np.random.default_rng(rows * 7 + cols + seq)
    t = ternary_matrix(rng, rows, cols)
    rs = rng.uniform(0.01, 0.1, rows).astype(np.float32)
    x = rng.standard_normal(seq * cols).astype(np.float32)
    w = gpu.DeviceTernaryWeight.from_packed_u8(fo.pack_ternary(t), rows, cols, rs)
    y = w.matmul_f32(torch.from_numpy(x).cuda().view(seq, cols)).cpu().numpy()
    if cols % 16 == 0:  # reference GPU-layout mirror (per-row scales)
        ref = fo.gpu_ternary_mm_cpu(fo.pack_ternary_rows_u32(t, rows, cols), rs, x, seq, cols, rows)
    else:
        ref = np.concatenate([fo.ternary_matmul(t, 1.0, x[s * cols:(s + 1) * cols], rows, cols, 1)
                              * rs for s in range(seq)])
    assert_fp32_close(y, ref, condition(t, x, rows, cols, seq, rs), what=f"{rows}x{cols}x{seq}")


def test_cfg1_baseline_seed0(gpu):
    """BASELINE config 1 as specified: seed 0, W [5632, 2048] with P(-1)=P(0)=P(+1)=1/3,
    per-row scales ~ U(0.01, 0.1), x [1, 2048] ~ N(0, 1)."""
    rng = np.random.default_rng(0)
    rows, cols = 5632, 2048
    t = rng.integers(-1, 2, size=rows * cols).astype(np.int8)
    rs = rng.uniform(0.01, 0.1, rows).astype(np.float32)
    x = rng.standard_normal(cols).astype(np.float32)
    w = gpu.DeviceTernaryWeight.from_packed_u8(fo.pack_ternary(t), rows, cols, rs)
    y = w.matmul_f32(torch.from_numpy(x).cuda().view(1, cols)).cpu().numpy()
    ref = fo.gpu_ternary_mm_cpu(fo.pack_ternary_rows_u32(t, rows, cols), rs, x, 1, cols, rows)
    assert_fp32_close(y, ref, condition(t, x, rows, cols, 1, rs), what="cfg1 seed 0")


@pytest.mark.parametrize("rows,cols,seq", SHAPES + [
    (300, 1000, 16), (257, 4096, 12), (64, 4098, 15), (130, 1024, 6), (512, 2052, 8)])
def test_i8_bit_exact(gpu, rows, cols, seq):
    rng = np.random.default_rng(rows + cols * 3 + seq)
    t = ternary_matrix(rng, rows, cols, p_zero=0.5)
    sw = rng.uniform(0.01, 0.1, rows).astype(np.float32)
    x = rng.standard_normal(seq * cols).astype(np.float32)
    q, sx = fo.quantize_absmax_i8(x, seq, cols)
    w = gpu.DeviceTernaryWeight.from_packed_u8(fo.pack_ternary(t), rows, cols, sw)
    y = w.matmul_i8(torch.from_numpy(q).cuda().view(seq, cols), torch.from_numpy(sx).cuda())
    ref = fo.ternary_matmul_i8(t, q, sx, sw, seq, cols, rows)
    assert_bits_equal(y.cpu().numpy(), ref, what=f"{rows}x{cols}x{seq}")


@pytest.mark.parametrize("seq", [1, 4, 5, 64, 65, 300])
def test_bf16_activations(gpu, seq):
    rng = np.random.default_rng(seq)
    rows, cols = 384, 1408
    t = ternary_matrix(rng, rows, cols)
    rs = rng.uniform(0.01, 0.1, rows).astype(np.float32)
    xb = torch.from_numpy(rng.standard_normal((seq, cols)).astype(np.float32)).to(torch.bfloat16)
    x = xb.float().numpy().ravel()
    w = gpu.DeviceTernaryWeight.from_packed_u8(fo.pack_ternary(t), rows, cols, rs)
    y = w.matmul_bf16(xb.cuda()).cpu().numpy()
    ref = np.concatenate([fo.ternary_matmul(t, 1.0, x[s * cols:(s + 1) * cols], rows, cols, 1) * rs
                          for s in range(seq)])
    assert_fp32_close(y, ref, condition(t, x, rows, cols, seq, rs), what=f"bf16 seq={seq}")


@pytest.mark.parametrize("seq", [1, 3])
def test_grouped_f32(gpu, seq):
    """One launch over several weights of different shapes; two share x."""
    rng = np.random.default_rng(40 + seq)
    shapes = [(5632, 2048), (2048, 2048), (300, 2048), (1408, 512), (129, 70)]
    ws, xs, ys, refs, conds = [], [], [], [], []
    x_shared = rng.standard_normal(seq * 2048).astype(np.float32)
    xt_shared = torch.from_numpy(x_shared).cuda().view(seq, 2048)
    for i, (rows, cols) in enumerate(shapes):
        t = ternary_matrix(rng, rows, cols)
        rs = rng.uniform(0.01, 0.1, rows).astype(np.float32)
        if cols == 2048 and i < 3:
            x, xt = x_shared, xt_shared
        else:
            x = rng.standard_normal(seq * cols).astype(np.float32)
            xt = torch.from_numpy(x).cuda().view(seq, cols)
        ws.append(gpu.DeviceTernaryWeight.from_packed_u8(fo.pack_ternary(t), rows, cols, rs))
        xs.append(xt)
        ys.append(torch.full((seq, rows), float("nan"), device="cuda"))
        refs.append(np.concatenate([fo.ternary_matmul(t, 1.0, x[s * cols:(s + 1) * cols], rows,
                                                      cols, 1) * rs for s in range(seq)]))
        conds.append(condition(t, x, rows, cols, seq, rs))
    gpu.GroupCall(ws, xs, ys)()
    for y, ref, cond in zip(ys, refs, conds):
        assert_fp32_close(y.cpu().numpy(), ref, cond, what="grouped")
    # same call again: scratch left clean by the first call
    for y in ys:
        y.fill_(float("nan"))
    gpu.GroupCall(ws, xs, ys)()
    for y, ref, cond in zip(ys, refs, conds):
        assert_fp32_close(y.cpu().numpy(), ref, cond, what="grouped again")


def test_grouped_i8_bit_exact(gpu):
    rng = np.random.default_rng(77)
    seq = 40
    shapes = [(1408, 2048), (1408, 2048), (2048, 1408)]
    ws, qs, sxs, ys, refs = [], [], [], [], []
    for rows, cols in shapes:
        t = ternary_matrix(rng, rows, cols)
        rs = rng.uniform(0.01, 0.1, rows).astype(np.float32)
        x = rng.standard_normal(seq * cols).astype(np.float32)
        q, sx = fo.quantize_absmax_i8(x, seq, cols)
        ws.append(gpu.DeviceTernaryWeight.from_packed_u8(fo.pack_ternary(t), rows, cols, rs))
        qs.append(torch.from_numpy(q).cuda().view(seq, cols))
        sxs.append(torch.from_numpy(sx).cuda())
        ys.append(torch.empty(seq, rows, device="cuda"))
        refs.append(fo.ternary_matmul_i8(t, q, sx, rs, seq, cols, rows))
    gpu.GroupCall(ws, qs, ys, qs_sx=sxs)()
    for y, ref in zip(ys, refs):
        assert_bits_equal(y.cpu().numpy(), ref, what="grouped i8")


@pytest.mark.parametrize("seq,mode", [(1, "f32"), (3, "f32"), (2, "i8"), (9, "i8")])
def test_grouped_large(gpu, seq, mode):
    """A large group in one launch: 44 weights over four activations (four
    segments, CTAs split among them by work), ragged row counts, both operand
    widths, run twice."""
    rng = np.random.default_rng(90 + seq)
    kinds = [(5632, 2048)] * 4 + [(1000, 2048), (2050, 1408), (129, 70)]
    mats = [ternary_matrix(rng, r, c) for r, c in kinds]
    scales = [rng.uniform(0.01, 0.1, r).astype(np.float32) for r, _ in kinds]
    acts = {}
    for key, cols in [(0, 2048), (1, 2048), (2, 1408), (3, 70)]:
        x = rng.standard_normal(seq * cols).astype(np.float32)
        if mode == "i8":
            q, sx = fo.quantize_absmax_i8(x, seq, cols)
            acts[key] = (x, q, sx, torch.from_numpy(q).cuda().view(seq, cols),
                         torch.from_numpy(sx).cuda())
        else:
            acts[key] = (x, None, None, torch.from_numpy(x).cuda().view(seq, cols), None)
    plan = [(i % 4, i % 2) for i in range(32)] + [(4, 0), (4, 1)] * 2 + [(5, 2)] * 6 + [(6, 3)] * 2
    uploaded = [gpu.DeviceTernaryWeight.from_packed_u8(fo.pack_ternary(t), r, c, s)
                for t, (r, c), s in zip(mats, kinds, scales)]
    refs = {}
    ws, xs, sxs, ys, conds = [], [], [], [], []
    for m, a in plan:
        rows, cols = kinds[m]
        x, q, sx, xt, sxt = acts[a]
        if (m, a) not in refs:
            if mode == "i8":
                refs[(m, a)] = fo.ternary_matmul_i8(mats[m], q, sx, scales[m], seq, cols, rows)
            else:
                refs[(m, a)] = np.concatenate(
                    [fo.ternary_matmul(mats[m], 1.0, x[s * cols:(s + 1) * cols], rows, cols, 1)
                     * scales[m] for s in range(seq)])
        ws.append(uploaded[m])
        xs.append(xt)
        sxs.append(sxt)
        ys.append(torch.full((seq, rows), float("nan"), device="cuda"))
        conds.append(None if mode == "i8" else condition(mats[m], x, rows, cols, seq, scales[m]))
    for rep in range(2):
        for y in ys:
            y.fill_(float("nan"))
        if mode == "i8":
            gpu.GroupCall(ws, xs, ys, qs_sx=sxs)()
        else:
            gpu.GroupCall(ws, xs, ys)()
        for i, ((m, a), y) in enumerate(zip(plan, ys)):
            if mode == "i8":
                assert_bits_equal(y.cpu().numpy(), refs[(m, a)], what=f"large i8 #{i} rep {rep}")
            else:
                assert_fp32_close(y.cpu().numpy(), refs[(m, a)], conds[i], what=f"large #{i} rep {rep}")


def test_no_kernel_timeouts(gpu):
    """Run after the others in this module: no bounded wait inside a kernel gave up."""
    gpu.get_context().check()


def test_quantizer_bit_exact(gpu):
    rng = np.random.default_rng(0)
    x = rng.standard_normal((9, 1000)).astype(np.float32)
    x[3] = 0.0              # absmax == 0 row
    x[4, 7] = 1e30          # huge outlier
    x[5] = np.float32(0.5) * np.sign(x[5])  # exact .5 products
    q, sx = gpu.quantize_absmax_i8(torch.from_numpy(x).cuda())
    rq, rsx = fo.quantize_absmax_i8(x, 9, 1000)
    assert (q.cpu().numpy().ravel() == rq).all()
    assert_bits_equal(sx.cpu().numpy(), rsx)


def test_quantizer_bf16_input(gpu):
    rng = np.random.default_rng(1)
    xb = torch.from_numpy(rng.standard_normal((4, 4096)).astype(np.float32)).to(torch.bfloat16)
    q, sx = gpu.quantize_absmax_i8(xb.cuda())
    rq, rsx = fo.quantize_absmax_i8(xb.float().numpy(), 4, 4096)
    assert (q.cpu().numpy().ravel() == rq).all()
    assert_bits_equal(sx.cpu().numpy(), rsx)


def test_cfg2_prefill_bit_exact(gpu):
    """BASELINE config 2 at full size: M=512, K=4096, N=11008, bf16 -> int8."""
    M, K, N = 512, 4096, 11008
    g = torch.Generator().manual_seed(2)
    t = torch.multinomial(torch.tensor([0.25, 0.5, 0.25]), N * K, replacement=True,
                          generator=g).to(torch.int8) - 1
    t = t.numpy().astype(np.int8)
    sw = (torch.rand(N, generator=g) * 0.09 + 0.01).numpy().astype(np.float32)
    xb = torch.randn(M, K, generator=g).to(torch.bfloat16)
    q, sx = gpu.quantize_absmax_i8(xb.cuda())
    rq, rsx = fo.quantize_absmax_i8(xb.float().numpy(), M, K)
    assert (q.cpu().numpy().ravel() == rq).all()
    w = gpu.DeviceTernaryWeight.from_packed_u8(fo.pack_ternary(t), N, K, sw)
    y = w.matmul_i8(q, sx).cpu().numpy()
    ref = fo.ternary_matmul_i8(t, rq, rsx, sw, M, K, N)
    assert_bits_equal(y, ref, what="cfg2")


def test_u32_upload_and_device_upload_agree(gpu):
    rng = np.random.default_rng(5)
    rows, cols = 200, 96
    t = ternary_matrix(rng, rows, cols)
    rs = rng.uniform(0.01, 0.1, rows).astype(np.float32)
    x = torch.from_numpy(rng.standard_normal((3, cols)).astype(np.float32)).cuda()
    words = fo.pack_ternary_rows_u32(t, rows, cols)
    w1 = gpu.DeviceTernaryWeight.from_packed_u8(fo.pack_ternary(t), rows, cols, rs)
    w2 = gpu.DeviceTernaryWeight.from_packed_u32(words, rows, cols, rs)
    y1, y2 = w1.matmul_f32(x), w2.matmul_f32(x)
    assert torch.equal(y1, y2)


def test_op_dispatch_wgsl_layout(gpu):
    """TernaryMatMulOp::dispatch on raw u32 buffers (reference WGSL layout)."""
    rng = np.random.default_rng(6)
    for rows, cols, seq in [(2, 2, 1), (33, 17, 3), (512, 2048, 2)]:
        t = ternary_matrix(rng, rows, cols)
        rs = rng.uniform(0.01, 0.1, rows).astype(np.float32)
        x = rng.standard_normal(seq * cols).astype(np.float32)
        words = fo.pack_ternary_rows_u32(t, rows, cols)
        op = gpu.TernaryMatMulOp.new()
        out = torch.empty(seq * rows, dtype=torch.float32, device="cuda")
        op.dispatch(torch.from_numpy(words.view(np.int32)).cuda(), torch.from_numpy(rs).cuda(),
                    torch.from_numpy(x).cuda(), out, seq, cols, rows)
        ref = fo.gpu_ternary_mm_cpu(words, rs, x, seq, cols, rows)
        assert_fp32_close(out.cpu().numpy(), ref, condition(t, x, rows, cols, seq, rs))


def test_accelerator_host_buffers(gpu):
    """GpuMatmulAccelerator::gpu_ternary_matmul{,_vram} (host slices in/out)."""
    rng = np.random.default_rng(8)
    rows, cols, seq = 300, 256, 2
    t = ternary_matrix(rng, rows, cols)
    rs = rng.uniform(0.01, 0.1, rows).astype(np.float32)
    x = rng.standard_normal(seq * cols).astype(np.float32)
    words = fo.pack_ternary_rows_u32(t, rows, cols)
    acc = gpu.GpuMatmulAccelerator()
    y = acc.gpu_ternary_matmul(words, rs, x, seq, cols, rows)
    ref = fo.gpu_ternary_mm_cpu(words, rs, x, seq, cols, rows)
    assert_fp32_close(y, ref, condition(t, x, rows, cols, seq, rs))
    w = gpu.DeviceTernaryWeight.from_packed_u32(words, rows, cols, rs)
    y2 = acc.gpu_ternary_matmul_vram(w, x, seq, cols, rows)
    assert_fp32_close(y2, ref, condition(t, x, rows, cols, seq, rs))


@pytest.mark.parametrize("rows,cols,seq", [(300, 256, 2), (300, 256, 9), (16384, 512, 5)])
def test_host_buffer_outputs(gpu, rows, cols, seq):
    """ft_gpu_ternary_matmul_vram with a pageable output (staged in pinned
    memory) and a pinned caller output; small outputs are written by the kernel
    through the pinned memory's mapping (decode GEMV and engine shapes), the
    16384-row output is copied back."""
    from ferrisres_b200.gpu import _vram_fn
    rng = np.random.default_rng(rows + seq)
    t = ternary_matrix(rng, rows, cols)
    rs = rng.uniform(0.01, 0.1, rows).astype(np.float32)
    x = rng.standard_normal(seq * cols).astype(np.float32)
    w = gpu.DeviceTernaryWeight.from_packed_u8(fo.pack_ternary(t), rows, cols, rs)
    ref = np.concatenate([fo.ternary_matmul(t, 1.0, x[s * cols:(s + 1) * cols], rows, cols, 1) * rs
                          for s in range(seq)])
    cond = condition(t, x, rows, cols, seq, rs)
    acc = gpu.GpuMatmulAccelerator()
    for _ in range(2):
        assert_fp32_close(acc.gpu_ternary_matmul_vram(w, x, seq, cols, rows), ref, cond,
                          what="pageable output")
    xp = torch.from_numpy(x).pin_memory()
    yp = torch.full((seq * rows,), float("nan"), dtype=torch.float32).pin_memory()
    from ferrisres_b200._lib import check
    check(_vram_fn()(w.ctx.handle, w.handle, xp.data_ptr(), int(seq), cols, rows, yp.data_ptr()))
    assert_fp32_close(yp.numpy(), ref, cond, what="pinned output")


def test_reference_kats_on_gpu(gpu):
    """The reference's own known answers, run through the GPU path."""
    acc = gpu.GpuMatmulAccelerator()
    one = np.ones(2, np.float32)
    # src/compute/kernels/ternary_matmul.rs:293-335
    w = fo.pack_ternary_rows_u32(np.array([1, 0, 0, 1], np.int8), 2, 2)
    assert np.allclose(acc.gpu_ternary_matmul(w, one, [3.0, 5.0], 1, 2, 2), [3, 5], atol=1e-5)
    w = fo.pack_ternary_rows_u32(np.array([1, -1, 1, 1], np.int8), 2, 2)
    assert np.allclose(acc.gpu_ternary_matmul(w, [2.0, 0.5], [1.0, 2.0], 1, 2, 2), [-2, 1.5],
                       atol=1e-5)
    # src/model/ternary.rs:1300-1312: 1,-1,0,1,0,-1 . 1..6 = -3
    dw = gpu.DeviceTernaryWeight.from_ternary(np.array([1, -1, 0, 1, 0, -1], np.int8), 1, 6, [1.0])
    y = dw.matmul_f32(torch.arange(1, 7, dtype=torch.float32, device="cuda").view(1, 6))
    assert abs(float(y[0, 0]) + 3.0) < 1e-5
    # src/model/ternary.rs:1001-1008: negative scale -> -20
    dw = gpu.DeviceTernaryWeight.from_ternary(np.ones(4, np.int8), 1, 4, [-2.0])
    y = dw.matmul_f32(torch.arange(1, 5, dtype=torch.float32, device="cuda").view(1, 4))
    assert abs(float(y[0, 0]) + 20.0) < 1e-6


def test_empty_seq_is_noop(gpu):
    dw = gpu.DeviceTernaryWeight.from_ternary(np.ones(4, np.int8), 1, 4, [1.0])
    y = dw.matmul_f32(torch.empty(0, 4, device="cuda"))
    assert y.shape == (0, 1)


def test_shape_errors(gpu):
    from ferrisres_b200 import ShapeError
    dw = gpu.DeviceTernaryWeight.from_ternary(np.ones(8, np.int8), 2, 4, [1.0, 1.0])
    with pytest.raises(ShapeError):
        dw.matmul_f32(torch.zeros(1, 5, device="cuda"))
    with pytest.raises(ShapeError):
        dw.matmul_i8(torch.zeros(1, 4, dtype=torch.int8, device="cuda"),
                     torch.zeros(2, device="cuda"))
