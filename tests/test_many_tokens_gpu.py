"""Launches of >= 4096 activation tokens, against the CPU oracle.

From 4096 token slots on, the tensor-core path builds the fp32 / bf16 operand
with one warp per token (prep_b_kernel with W = 1 in csrc/ft_tc.cu); the other
test files' shorter launches spread a token over 2 to 8 warps, whose partial
absmax and non-finite lists meet in shared memory.  Same rules as
tests/test_precision_gpu.py:
NaN placement and every infinity's sign equal the oracle's exactly
(gpu_ternary_mm_cpu, src/model/cpu_block_attn_res.rs:2373-2398), finite outputs
within 1e-5 of each output's condition (tests/helpers.py).  K = 1000 ends inside
a 128-column chunk; the tokens include non-finite elements below and
above the per-token list capacity and a 1e6 outlier channel.  The blocked-scale
form (src/model/ternary.rs:541-579) runs the same kernel with column-block scales.
"""
import numpy as np
import pytest
import torch

from oracle import oracle as fo
from tests.helpers import assert_fp32_close, condition, ternary_matrix

pytestmark = pytest.mark.gpu

ROWS, COLS, SEQ = 256, 1000, 4100


@pytest.fixture(scope="module")
def gpu():
    assert torch.cuda.is_available()
    from ferrisres_b200 import gpu as g
    return g


def case(rng):
    t = ternary_matrix(rng, ROWS, COLS).reshape(ROWS, COLS)
    x = rng.standard_normal((SEQ, COLS)).astype(np.float32)
    ks = [5, 402, 999]
    x[0, ks[0]], x[0, ks[1]], x[0, ks[2]] = np.inf, -np.inf, np.nan
    r = np.arange(ROWS)
    t[:, ks[0]] = r % 3 - 1
    t[:, ks[1]] = (r // 3) % 3 - 1
    t[:, ks[2]] = (r // 9) % 3 - 1
    pos = rng.choice(COLS, size=40, replace=False)  # more than the kernels list
    x[3000, pos] = rng.choice(np.array([np.inf, -np.inf, np.nan], np.float32), size=40)
    x[4099, 77] = 1e6  # outlier channel of the last token
    return t.ravel(), x


def check(y, ref, t, x, rs, what):
    assert np.array_equal(np.isnan(y), np.isnan(ref)), f"{what}: NaN placement differs"
    inf = np.isinf(ref)
    assert np.array_equal(np.isinf(y), inf), f"{what}: infinity placement differs"
    assert np.array_equal(np.sign(y[inf]), np.sign(ref[inf])), f"{what}: infinity sign"
    fin = np.isfinite(ref)
    xf = np.where(np.isfinite(x), x, 0.0).astype(np.float32)
    cond = condition(t, xf.ravel(), ROWS, COLS, SEQ, rs)
    assert_fp32_close(y[fin], ref[fin], cond[fin], what=what)


@pytest.mark.parametrize("bf16", [False, True])
def test_many_tokens_matches_oracle(gpu, bf16):
    rng = np.random.default_rng(41 + bf16)
    t, x = case(rng)
    rs = rng.uniform(0.01, 0.1, ROWS).astype(np.float32)
    xt = torch.from_numpy(x)
    if bf16:
        xb = xt.to(torch.bfloat16)
        x = xb.float().numpy()
    w = gpu.DeviceTernaryWeight.from_packed_u8(fo.pack_ternary(t), ROWS, COLS, rs)
    y = (w.matmul_bf16(xb.cuda()) if bf16 else w.matmul_f32(xt.cuda())).cpu().numpy().ravel()
    ref = fo.gpu_ternary_mm_cpu(fo.pack_ternary_rows_u32(t, ROWS, COLS), rs, x.ravel(), SEQ,
                                COLS, ROWS)
    check(y, ref, t, x, rs, f"{SEQ} tokens bf16={bf16}")
    w.ctx.check()


def test_many_tokens_blocked_scales(gpu):
    rng = np.random.default_rng(43)
    t = ternary_matrix(rng, ROWS, COLS)
    bs = 64
    scales = rng.uniform(0.01, 2.0, -(-COLS // bs)).astype(np.float32)
    x = rng.standard_normal(SEQ * COLS).astype(np.float32)
    w = gpu.DeviceTernaryWeight.from_packed_u8(fo.pack_ternary(t), ROWS, COLS,
                                               np.ones(ROWS, np.float32))
    y = w.matmul_blocked_f32(torch.from_numpy(x).cuda().view(SEQ, COLS),
                             torch.from_numpy(scales).cuda(), bs).cpu().numpy().ravel()
    ref = fo.ternary_matmul_blocked(t, scales, bs, x, ROWS, COLS, SEQ)
    a = np.repeat(np.abs(scales.astype(np.float64)), bs)[:COLS]
    W = np.abs(t.reshape(ROWS, COLS).astype(np.float64)) * a[None, :]
    cond = (np.abs(x.reshape(SEQ, COLS).astype(np.float64)) @ W.T).ravel()
    assert_fp32_close(y, ref, cond, what=f"blocked {SEQ} tokens")
    w.ctx.check()
