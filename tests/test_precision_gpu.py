"""Range and non-finite activations on the GPU path, against the CPU oracle.

The oracle is gpu_ternary_mm_cpu (src/model/cpu_block_attn_res.rs:2373-2398),
the reference's CPU mirror of the TernaryMatMulOp shader
(src/compute/kernels/ternary_matmul.rs:54-70): per row, an fp32 sum of x[k]
over the nonzero weights (code -1 subtracts, +1 adds, 0 is skipped), times the
row scale.

* Outliers: one channel per token is 1e4x or 1e7x the others; half of the
  rows have a zero weight on that channel, so their outputs are sums of
  ordinary-sized terms next to a huge token absmax.  Finite outputs must
  satisfy the fp32 rule of tests/helpers.py (1e-5 of each output's condition).
* Non-finite: +inf, -inf and NaN at chosen positions, with weights arranged so
  every combination of {-1, 0, +1} meets them; a token with more non-finite
  elements than the kernels list (the whole-row scan); an all-finite token
  beside them.  NaN placement and the sign of every infinity must equal the
  oracle's exactly; the finite outputs follow the fp32 rule.

seq 1 and 2 run on the decode GEMV (8 digits per token), 5 and 40 on the
tcgen05 engine.  Dense and 2:4 sparse weights; fp32 and bf16 activations.
"""
import numpy as np
import pytest
import torch

from oracle import oracle as fo
from tests.helpers import assert_fp32_close, condition, ternary_matrix

pytestmark = pytest.mark.gpu

ROWS, COLS = 1024, 1024


@pytest.fixture(scope="module")
def gpu():
    assert torch.cuda.is_available()
    from ferrisres_b200 import gpu as g
    return g


def sparse24(rng, rows, cols):
    ng = rows * cols // 4
    pats = np.array([(0, 1), (0, 2), (0, 3), (1, 2), (1, 3), (2, 3)])
    pos = pats[rng.integers(0, 6, size=ng)]
    t = np.zeros((ng, 4), np.int8)
    np.put_along_axis(t, pos, rng.choice(np.array([-1, 1], np.int8), size=(ng, 2)), axis=1)
    return t.ravel()


def upload(gpu, t, rs, sparse):
    if sparse:
        pat, sg = fo.sparse_from_ternary(t, ROWS, COLS)
        return gpu.DeviceTernaryWeight.from_sparse_host(pat, sg, ROWS, COLS, rs)
    return gpu.DeviceTernaryWeight.from_packed_u8(fo.pack_ternary(t), ROWS, COLS, rs)


def run(gpu, w, x, seq, bf16):
    xt = torch.from_numpy(x).view(seq, COLS)
    if bf16:
        return w.matmul_bf16(xt.to(torch.bfloat16).cuda()).cpu().numpy().ravel()
    return w.matmul_f32(xt.cuda()).cpu().numpy().ravel()


def oracle(t, rs, x, seq):
    return fo.gpu_ternary_mm_cpu(fo.pack_ternary_rows_u32(t, ROWS, COLS), rs, x, seq, COLS, ROWS)


@pytest.mark.parametrize("sparse", [False, True])
@pytest.mark.parametrize("bf16", [False, True])
@pytest.mark.parametrize("seq", [1, 2, 5, 40])
@pytest.mark.parametrize("ratio", [1e4, 1e7])
def test_outlier_channel(gpu, ratio, seq, bf16, sparse):
    rng = np.random.default_rng(int(ratio) % 1000 + 10 * seq + 2 * bf16 + sparse)
    t = (sparse24(rng, ROWS, COLS) if sparse else ternary_matrix(rng, ROWS, COLS)).reshape(ROWS, COLS)
    rs = rng.uniform(0.01, 0.1, ROWS).astype(np.float32)
    x = rng.standard_normal((seq, COLS)).astype(np.float32)
    k0 = rng.integers(0, COLS, size=seq)
    for s in range(seq):
        x[s, k0[s]] = ratio * (1 if s % 2 == 0 else -1)
    # the first half of the rows never meets any token's outlier channel (2:4
    # weights: that row's group of 4 gets its two nonzeros elsewhere, so it
    # stays a valid 2:4 group)
    for s in range(seq):
        if sparse:
            g0, e = k0[s] // 4 * 4, k0[s] % 4
            other = [p for p in range(4) if p != e][:2]
            t[: ROWS // 2, g0:g0 + 4] = 0
            for p in other:
                t[: ROWS // 2, g0 + p] = rng.choice(np.array([-1, 1], np.int8), size=ROWS // 2)
        else:
            t[: ROWS // 2, k0[s]] = 0
    t = t.ravel()
    if bf16:
        x = torch.from_numpy(x).to(torch.bfloat16).float().numpy()
    x = x.ravel()
    w = upload(gpu, t, rs, sparse)
    y = run(gpu, w, x, seq, bf16)
    ref = oracle(t, rs, x, seq)
    assert_fp32_close(y, ref, condition(t, x, ROWS, COLS, seq, rs),
                      what=f"ratio {ratio:g} seq {seq} bf16 {bf16} sparse {sparse}")
    w.ctx.check()


def nonfinite_case(rng, seq, sparse):
    t = (sparse24(rng, ROWS, COLS) if sparse else ternary_matrix(rng, ROWS, COLS)).reshape(ROWS, COLS)
    x = rng.standard_normal((seq, COLS)).astype(np.float32)
    # token 0: +inf, -inf, NaN at three positions in three different groups of 4
    ks = [5, 402, 901]
    x[0, ks[0]], x[0, ks[1]], x[0, ks[2]] = np.inf, -np.inf, np.nan
    if not sparse:
        # every (w at k0, w at k1, w at k2) combination over the rows
        r = np.arange(ROWS)
        t[:, ks[0]] = r % 3 - 1
        t[:, ks[1]] = (r // 3) % 3 - 1
        t[:, ks[2]] = (r // 9) % 3 - 1
    if seq > 1:  # token 1: two +inf
        x[1, 77], x[1, 600] = np.inf, np.inf
    if seq > 2:  # token 2: more non-finite elements than the kernels list
        pos = rng.choice(COLS, size=40, replace=False)
        x[2, pos] = rng.choice(np.array([np.inf, -np.inf, np.nan], np.float32), size=40)
    return t.ravel(), x  # tokens 3.. stay finite


@pytest.mark.parametrize("sparse", [False, True])
@pytest.mark.parametrize("bf16", [False, True])
@pytest.mark.parametrize("seq", [1, 2, 5, 40])
def test_nonfinite_inputs(gpu, seq, bf16, sparse):
    rng = np.random.default_rng(100 + 10 * seq + 2 * bf16 + sparse)
    t, x = nonfinite_case(rng, seq, sparse)
    rs = rng.uniform(0.01, 0.1, ROWS).astype(np.float32)
    if bf16:
        x = torch.from_numpy(x).to(torch.bfloat16).float().numpy()
    x = x.ravel()
    w = upload(gpu, t, rs, sparse)
    y = run(gpu, w, x, seq, bf16)
    ref = oracle(t, rs, x, seq)
    assert np.array_equal(np.isnan(y), np.isnan(ref)), "NaN placement differs from the oracle"
    inf = np.isinf(ref)
    assert np.array_equal(np.isinf(y), inf), "infinity placement differs from the oracle"
    assert np.array_equal(np.sign(y[inf]), np.sign(ref[inf])), "an infinity has the wrong sign"
    assert np.isnan(ref).any() and inf.any(), "the case must exercise NaN and inf outputs"
    fin = np.isfinite(ref)
    xf = np.where(np.isfinite(x), x, 0.0).astype(np.float32)
    cond = condition(t, xf, ROWS, COLS, seq, rs)
    assert_fp32_close(y[fin], ref[fin], cond[fin], what=f"finite outputs seq {seq}")
    w.ctx.check()


def test_baseline_cfg1_seed0(gpu):
    """BASELINE config 1 exactly: seed 0, W [5632, 2048] with P = 1/3 each, row scales
    U(0.01, 0.1), x ~ N(0, 1) [1, 2048]."""
    rows, cols = 5632, 2048
    rng = np.random.default_rng(0)
    t = rng.integers(-1, 2, size=rows * cols).astype(np.int8)
    rs = rng.uniform(0.01, 0.1, rows).astype(np.float32)
    x = rng.standard_normal(cols).astype(np.float32)
    w = gpu.DeviceTernaryWeight.from_packed_u8(fo.pack_ternary(t), rows, cols, rs)
    y = w.matmul_f32(torch.from_numpy(x).cuda().view(1, cols)).cpu().numpy().ravel()
    ref = fo.ternary_matmul_packed_parallel_rows(fo.pack_ternary(t), rs, x, rows, cols)
    assert_fp32_close(y, ref, condition(t, x, rows, cols, 1, rs), what="cfg1 seed 0")
    # the reference's single-alpha special case: all scales equal
    ones = np.full(rows, 0.05, np.float32)
    w1 = gpu.DeviceTernaryWeight.from_packed_u8(fo.pack_ternary(t), rows, cols, ones)
    y1 = w1.matmul_f32(torch.from_numpy(x).cuda().view(1, cols)).cpu().numpy().ravel()
    ref1 = fo.ternary_matmul_packed_parallel_rows(fo.pack_ternary(t), ones, x, rows, cols)
    assert_fp32_close(y1, ref1, condition(t, x, rows, cols, 1, ones), what="cfg1 scalar scale")
