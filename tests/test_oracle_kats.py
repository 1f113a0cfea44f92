"""Pin the CPU oracle against the reference crate's own unit-test known answers.

Each test reproduces one reference test (cited as file:line in shift/FerrisRes
v0.2.3) with the same inputs and the same expected values; the oracle restates
the function under test.  CPU only.
"""
import math

import numpy as np
import pytest

from oracle import oracle as fo


def knuth_ternary(n):
    # src/model/ternary.rs:1274, src/model/sparse_ternary.rs:438
    i = np.arange(n, dtype=np.uint64)
    v = ((i * np.uint64(2654435761)) & np.uint64(0xFFFFFFFF)) >> np.uint64(30)
    return np.clip(v.astype(np.int64) - 1, -1, 1).astype(np.int8)


# ----------------------------------------------------- src/model/ternary.rs
def test_pack_unpack_roundtrip():  # ternary.rs:797-803
    v = np.array([-1, 0, 1] * 4, np.int8)
    assert (fo.unpack_ternary(fo.pack_ternary(v), v.size) == v).all()


def test_pack_non_multiple_of_4():  # ternary.rs:806-812
    v = np.array([-1, 0, 1], np.int8)
    p = fo.pack_ternary(v)
    assert p.size == 1
    assert (fo.unpack_ternary(p, 3) == v).all()
    # encoding -1->00, 0->01, +1->10, LSB first (ternary.rs:134-147)
    assert p[0] == (0b00 | (0b01 << 2) | (0b10 << 4))


def test_pack_single_value():  # ternary.rs:815-822
    for v in (-1, 0, 1):
        p = fo.pack_ternary(np.array([v], np.int8))
        assert p.size == 1 and fo.unpack_ternary(p, 1)[0] == v


def test_pack_unpack_large():  # ternary.rs:968-975
    v = (np.arange(1024) % 3 - 1).astype(np.int8)
    p = fo.pack_ternary(v)
    assert p.size == 256
    assert (fo.unpack_ternary(p, 1024) == v).all()


def test_quantize_zero_weights():  # ternary.rs:778-784
    q, s = fo.quantize_ternary(np.zeros(16, np.float32))
    assert (q == 0).all() and s == 1.0


def test_quantize_preserves_sign():  # ternary.rs:787-794
    q, _ = fo.quantize_ternary(np.array([-3.0, -0.5, -0.01, 0.01, 0.5, 3.0], np.float32))
    assert q[0] == -1 and q[5] == 1 and q[2] == q[3]


def test_quantize_roundtrip_cos():  # ternary.rs:753-775
    w = np.array([0.5, -0.3, 1.2, -0.8, 0.0, 0.01, -1.5, 2.0], np.float32)
    q, s = fo.quantize_ternary(w)
    assert s > 0 and set(np.unique(q)) <= {-1, 0, 1}
    r = q.astype(np.float32) * s
    cos = float(w @ r) / (np.linalg.norm(w) * np.linalg.norm(r))
    assert cos > 0.85


def test_ternary_matmul_identity():  # ternary.rs:980-998
    t = np.eye(4, dtype=np.int8).ravel()
    x = np.array([1, 2, 3, 4], np.float32)
    y = fo.ternary_matmul(t, 1.0, x, 4, 4, 1)
    assert np.abs(y - x).max() < 1e-6


def test_ternary_matmul_negative_scale():  # ternary.rs:1001-1008
    y = fo.ternary_matmul(np.ones(4, np.int8), -2.0, np.array([1, 2, 3, 4], np.float32), 1, 4, 1)
    assert abs(y[0] + 20.0) < 1e-6


def test_ternary_matmul_batch():  # ternary.rs:1011-1034
    t = np.array([1, -1, 0, 0, 1, -1], np.int8)
    x = np.array([1, 2, 3, 4, 5, 6], np.float32)
    y = fo.ternary_matmul(t, 1.0, x, 2, 3, 2)
    assert np.abs(y - np.array([-1, -1, -1, -1], np.float32)).max() < 1e-6


def _mod3(n):
    i = np.arange(n)
    return np.where(i % 3 == 0, 1, np.where(i % 3 == 1, -1, 0)).astype(np.int8)


def test_ternary_matmul_vs_fp32():  # ternary.rs:1037-1071
    t = _mod3(8 * 16)
    x = (np.arange(16, dtype=np.float32) * np.float32(0.1)).astype(np.float32)
    y = fo.ternary_matmul(t, 0.5, x, 8, 16, 1)
    deq = t.astype(np.float32) * np.float32(0.5)
    ref = np.array([sum(deq[r * 16 + j] * x[j] for j in range(16)) for r in range(8)], np.float32)
    assert np.abs(y - ref).max() < 1e-5


def test_ternary_matmul_packed_vs_unpacked():  # ternary.rs:1074-1108
    t = _mod3(4 * 16)
    x = np.sin(np.arange(16, dtype=np.float32) * np.float32(0.1)).astype(np.float32)
    a = fo.ternary_matmul(t, 0.7, x, 4, 16, 1)
    b = fo.ternary_matmul_packed(fo.pack_ternary(t), 0.7, x, 4, 16, 1)
    assert np.abs(a - b).max() < 1e-5


def test_ternary_matmul_decode_vs_general():  # ternary.rs:1175-1201
    i = np.arange(8 * 32)
    t = np.where(i % 5 < 2, 1, np.where(i % 5 < 4, -1, 0)).astype(np.int8)
    x = np.tan(np.arange(32, dtype=np.float32) * np.float32(0.05)).astype(np.float32)
    a = fo.ternary_matmul(t, 0.3, x, 8, 32, 1)
    b = fo.ternary_matmul_decode(t, 0.3, x, 8, 32)
    assert np.abs(a - b).max() < 1e-5


def test_ternary_matmul_all_zeros():  # ternary.rs:1256-1262
    y = fo.ternary_matmul(np.zeros(16, np.int8), 1.0, np.ones(16, np.float32), 1, 16, 1)
    assert abs(y[0]) < 1e-10


def test_ternary_matmul_large_layer():  # ternary.rs:1265-1297
    t = knuth_ternary(512 * 256)
    x = np.sin(np.arange(256, dtype=np.float32) * np.float32(0.01)).astype(np.float32)
    d = fo.ternary_matmul_decode(t, 0.1, x, 512, 256)
    g = fo.ternary_matmul(t, 0.1, x, 512, 256, 1)
    assert d.max() > d.min()
    assert np.abs(d - g).max() < 1e-3


def test_packed_matmul_non_multiple_of_4():  # ternary.rs:1300-1312
    t = np.array([1, -1, 0, 1, 0, -1], np.int8)
    x = np.array([1, 2, 3, 4, 5, 6], np.float32)
    a = fo.ternary_matmul(t, 1.0, x, 1, 6, 1)
    b = fo.ternary_matmul_packed(fo.pack_ternary(t), 1.0, x, 1, 6, 1)
    assert abs(a[0] - b[0]) < 1e-5 and abs(b[0] + 3.0) < 1e-5


def test_packed_parallel_equals_packed_for_scalar_scale():
    # ternary.rs:471-529 with all-equal row scales reduces to the reference's
    # own _packed_parallel; its per-byte 4-term grouping stays within 1e-5.
    rng = np.random.default_rng(3)
    t = rng.integers(-1, 2, size=64 * 128).astype(np.int8)
    x = rng.standard_normal(128).astype(np.float32)
    a = fo.ternary_matmul_packed_parallel_rows(fo.pack_ternary(t), np.full(64, 0.25, np.float32),
                                               x, 64, 128)
    b = fo.ternary_matmul(t, 0.25, x, 64, 128, 1)
    assert np.abs(a - b).max() < 1e-5


def test_pack_ternary_u32_matches_wgsl_packer():
    # ternary.rs:1317-1328 (flat u8 -> u32) equals the WGSL per-row packer
    # (kernels/ternary_matmul.rs:267-291) whenever in_cols % 16 == 0.
    t = knuth_ternary(8 * 64)
    flat = fo.pack_ternary_u32(fo.pack_ternary(t), t.size)
    rows = fo.pack_ternary_rows_u32(t, 8, 64)
    assert (flat == rows).all()


# ------------------------------------ src/compute/kernels/ternary_matmul.rs
def test_wgsl_ref_identity():  # ternary_matmul.rs:293-305
    p = fo.pack_ternary_rows_u32(np.array([1, 0, 0, 1], np.int8), 2, 2)
    y = fo.gpu_ternary_mm_cpu(p, np.ones(2, np.float32), np.array([3, 5], np.float32), 1, 2, 2)
    assert abs(y[0] - 3) < 1e-5 and abs(y[1] - 5) < 1e-5


def test_wgsl_ref_negate():  # ternary_matmul.rs:308-319
    p = fo.pack_ternary_rows_u32(np.array([-1, 0, 0, -1], np.int8), 2, 2)
    y = fo.gpu_ternary_mm_cpu(p, np.ones(2, np.float32), np.array([3, 5], np.float32), 1, 2, 2)
    assert abs(y[0] + 3) < 1e-5 and abs(y[1] + 5) < 1e-5


def test_wgsl_ref_scaled():  # ternary_matmul.rs:322-335
    p = fo.pack_ternary_rows_u32(np.array([1, -1, 1, 1], np.int8), 2, 2)
    y = fo.gpu_ternary_mm_cpu(p, np.array([2.0, 0.5], np.float32), np.array([1, 2], np.float32),
                              1, 2, 2)
    assert abs(y[0] + 2.0) < 1e-5 and abs(y[1] - 1.5) < 1e-5


def test_wgsl_ref_batch():  # ternary_matmul.rs:338-360
    p = fo.pack_ternary_rows_u32(np.array([1, 0, 0, -1], np.int8), 2, 2)
    y = fo.gpu_ternary_mm_cpu(p, np.ones(2, np.float32), np.arange(1, 7, dtype=np.float32), 3, 2, 2)
    assert np.abs(y - np.array([1, -2, 3, -4, 5, -6], np.float32)).max() < 1e-5


def test_wgsl_pack_17_values():  # ternary_matmul.rs:363-381
    v = np.array([1, 0, -1, 1, -1, 0, 0, 1, -1, -1, 1, 0, 0, 1, -1, 0, 1], np.int8)
    p = fo.pack_ternary_rows_u32(v, 1, 17)
    assert p.size == 2
    for i, x in enumerate(v):
        code = (int(p[i // 16]) >> ((i % 16) * 2)) & 3
        assert code == {-1: 0, 0: 1, 1: 2}[int(x)]


# --------------------------------------------- src/model/sparse_ternary.rs
def test_sparse_from_ternary_basic():  # sparse_ternary.rs:338-366
    t = np.array([1, -1, 0, 1, -1, 0, 0, -1, 0, 0, 1, 0, 1, -1, 1, -1], np.int8)
    pat, sg = fo.sparse_from_ternary(t, 4, 4)
    d = fo.sparse_to_ternary(pat, sg, 4, 4)
    for g in range(4):
        assert np.count_nonzero(d[g * 4:(g + 1) * 4]) <= 2


def test_sparse_preserves_signs():  # sparse_ternary.rs:369-391
    t = np.array([1, 1, 0, 0, -1, -1, 0, 0, 1, -1, 0, 0], np.int8)
    pat, sg = fo.sparse_from_ternary(t, 3, 4)
    d = fo.sparse_to_ternary(pat, sg, 3, 4)
    assert list(d[0:4]) == [1, 1, 0, 0]
    assert list(d[4:6]) == [-1, -1]
    assert list(d[8:10]) == [1, -1]


def test_sparse_known_output():  # sparse_ternary.rs:419-432
    t = np.array([1, 1, 0, 0, 1, 1, 0, 0], np.int8)
    pat, sg = fo.sparse_from_ternary(t, 2, 4)
    y = fo.sparse_ternary_matmul(pat, sg, 2.0, None, 2, 4, np.array([3, 5, 7, 11], np.float32), 1)
    assert abs(y[0] - 16) < 1e-5 and abs(y[1] - 16) < 1e-5


def test_sparse_identity_nonzero():  # sparse_ternary.rs:394-416
    t = np.eye(4, dtype=np.int8).ravel()
    pat, sg = fo.sparse_from_ternary(t, 4, 4)
    y = fo.sparse_ternary_matmul(pat, sg, 1.0, None, 4, 4, np.array([1, 2, 3, 4], np.float32), 1)
    assert np.abs(y).max() > 0


def test_sparse_prune_equals_from_ternary():  # sparse_ternary.rs:575-582
    t = np.array([1, -1, 0, 1, -1, 0, 1, -1], np.int8)
    a = fo.sparse_to_ternary(*fo.sparse_from_ternary(t, 2, 4), 2, 4)
    assert a.size == 8


def test_sparse_roundtrip_exact_2of4():
    rng = np.random.default_rng(11)
    rows, cols = 16, 64
    t = np.zeros(rows * cols, np.int8)
    for g in range(rows * cols // 4):
        pos = rng.choice(4, 2, replace=False)
        t[g * 4 + pos] = rng.choice([-1, 1], 2)
    pat, sg = fo.sparse_from_ternary(t, rows, cols)
    assert (fo.sparse_to_ternary(pat, sg, rows, cols) == t).all()
    x = rng.standard_normal(cols).astype(np.float32)
    a = fo.sparse_ternary_matmul(pat, sg, 0.5, None, rows, cols, x, 1)
    b = fo.ternary_matmul(t, 0.5, x, rows, cols, 1)
    assert np.abs(a - b).max() < 1e-5


def test_sparse_storage_bits():  # sparse_ternary.rs:445-470 (bits/weight 1.5 < 2)
    t = knuth_ternary(64 * 256)
    pat, sg = fo.sparse_from_ternary(t, 64, 256)
    bpw = (pat.size + sg.size) * 8 / t.size
    assert 0.5 < bpw < 2.0 and abs(bpw - 1.5) < 1e-9


# -------------------------------------- src/compute/kernels/sparse_ternary.rs
def test_wgsl_sparse_identity():  # sparse_ternary.rs:362-384
    t = np.array([1, 1, 0, 0, 1, 0, 1, 0, 0, 1, 0, 1, 0, 0, 1, 1], np.int8)
    p = fo.sparse_wgsl_pack(t, 4, 4)
    y = fo.sparse_wgsl_ref(p, np.ones(4, np.float32), np.array([1, 2, 3, 4], np.float32), 1, 4, 4)
    assert np.abs(y - np.array([3, 4, 6, 7], np.float32)).max() < 1e-5


def test_wgsl_sparse_negate():  # sparse_ternary.rs:387-401
    t = np.array([-1, -1, 0, 0, -1, 0, -1, 0], np.int8)
    p = fo.sparse_wgsl_pack(t, 2, 4)
    y = fo.sparse_wgsl_ref(p, np.ones(2, np.float32), np.array([1, 2, 3, 4], np.float32), 1, 4, 2)
    assert np.abs(y - np.array([-3, -4], np.float32)).max() < 1e-5


def test_wgsl_sparse_all_patterns():  # sparse_ternary.rs:404-419
    t = np.array([1, -1, 0, 0, 0, 0, 1, -1], np.int8)
    p = fo.sparse_wgsl_pack(t, 1, 8)
    y = fo.sparse_wgsl_ref(p, np.ones(1, np.float32), np.arange(1, 9, dtype=np.float32), 1, 8, 1)
    assert abs(y[0] + 2.0) < 1e-5


def test_wgsl_sparse_batch():  # sparse_ternary.rs:422-436
    p = fo.sparse_wgsl_pack(np.array([1, 1, 0, 0], np.int8), 1, 4)
    x = np.array([1, 2, 0, 0, 3, 4, 0, 0], np.float32)
    y = fo.sparse_wgsl_ref(p, np.ones(1, np.float32), x, 2, 4, 1)
    assert abs(y[0] - 3) < 1e-5 and abs(y[1] - 7) < 1e-5


def test_wgsl_sparse_matches_host_layout():
    rng = np.random.default_rng(5)
    rows, cols = 8, 48
    t = np.zeros(rows * cols, np.int8)
    for g in range(rows * cols // 4):
        t[g * 4 + rng.choice(4, 2, replace=False)] = rng.choice([-1, 1], 2)
    rs = rng.uniform(0.01, 0.1, rows).astype(np.float32)
    x = rng.standard_normal(2 * cols).astype(np.float32)
    a = fo.sparse_wgsl_ref(fo.sparse_wgsl_pack(t, rows, cols), rs, x, 2, cols, rows)
    pat, sg = fo.sparse_from_ternary(t, rows, cols)
    b = fo.sparse_ternary_matmul(pat, sg, 0.0, rs, rows, cols, x, 2)
    assert np.abs(a - b).max() < 1e-6


# ------------------------------------------------ src/inference/turboquant_kv.rs
def test_3bit_pack_roundtrip():  # turboquant_kv.rs:417-423
    c = np.array([0, 1, 2, 3, 4, 5, 6, 7, 0, 3, 5, 7, 1, 2, 4, 6], np.uint8)
    assert (fo.unpack_3bit(fo.pack_3bit(c), c.size) == c).all()


def test_3bit_single_group():  # turboquant_kv.rs:426-432
    c = np.array([7, 6, 5, 4, 3, 2, 1, 0], np.uint8)
    p = fo.pack_3bit(c)
    assert p.size == 3 and (fo.unpack_3bit(p, 8) == c).all()
    # LSB-first bit stream: value i occupies bits 3i..3i+2
    bits = int(p[0]) | (int(p[1]) << 8) | (int(p[2]) << 16)
    assert [(bits >> (3 * i)) & 7 for i in range(8)] == list(c)


def test_3bit_non_multiple():  # turboquant_kv.rs:435-440
    c = np.array([1, 2, 3, 4, 5], np.uint8)
    assert (fo.unpack_3bit(fo.pack_3bit(c), 5) == c).all()


def test_3bit_quantize_uniform():  # turboquant_kv.rs:457-464
    codes, mn, mx = fo.quantize_3bit(np.arange(8, dtype=np.float32))
    assert list(codes) == list(range(8)) and abs(mn) < 1e-5 and abs(mx - 7) < 1e-5


def test_3bit_quantize_constant():  # turboquant_kv.rs:467-474
    codes, mn, mx = fo.quantize_3bit(np.full(16, 3.14, np.float32))
    assert (codes == 0).all() and abs(mn - 3.14) < 1e-5 and abs(mx - 3.14) < 1e-5
    assert (fo.dequantize_3bit(codes, mn, mx) == np.float32(3.14)).all()


def test_3bit_quantize_roundtrip_mse():  # turboquant_kv.rs:443-454
    v = np.sin(np.arange(128, dtype=np.float32) * np.float32(0.1) - np.float32(6.4)).astype(np.float32)
    codes, mn, mx = fo.quantize_3bit(v)
    r = fo.dequantize_3bit(codes, mn, mx)
    assert codes.max() <= 7 and float(np.mean((v - r) ** 2)) < 0.1


def test_kv_append_get_mse():  # turboquant_kv.rs:477-497 (kv_dim 16, group 8)
    k = np.array([1.0, -0.5, 0.3, -0.1, 2.0, -1.5, 0.7, -0.3, 1.1, -0.4, 0.2, -0.2, 1.8, -1.3,
                  0.6, -0.4], np.float32)
    packed, mm = fo.kv_quantize_vector(k, 8)
    assert packed.size == 6 and mm.size == 4
    out = fo.kv_dequantize_vector(packed, mm, 16, 8)
    assert float(np.mean((k - out) ** 2)) < 0.5


# ------------------------------------------------------------- MoE routing
def test_moe_gating_top2_known_answer():
    # tests/kernel_tests.rs:285-324: top-2 of logits [0.1,0.5,0.3,0.9,0.2]
    # selects the 0.9 and 0.5 experts.  Build a router with hidden=1, x=1 so
    # that the router scores equal those logits (ternary_moe.rs:153-160), and
    # check the renormalised gates (ternary_moe.rs:180-218).
    logits = np.array([0.1, 0.5, 0.3, 0.9, 0.2], np.float32)
    E, H, F = 5, 1, 1
    one = [np.ones(1, np.int8)] * E
    s = [np.ones(1, np.float32)] * E
    y, route, probs = fo.moe_forward(logits, one, s, one, s, one, s, H, F, 2,
                                     np.ones(1, np.float32), 1)
    assert list(route) == [3, 1]
    e = np.exp(logits - logits.max())
    p = e / e.sum()
    w3, w1 = p[3] / (p[3] + p[1]), p[1] / (p[3] + p[1])
    assert abs(w3 - math.exp(0.9) / (math.exp(0.9) + math.exp(0.5))) < 1e-6
    silu1 = 1.0 / (1.0 + math.exp(-1.0))
    assert abs(y[0] - (w3 + w1) * silu1) < 1e-6


def test_moe_forward_shape_and_nonzero():  # ternary_moe.rs:317-355 (make_test_moe)
    H, F, E = 8, 16, 2
    router = (np.arange(H * E, dtype=np.float32) * np.float32(0.1) - np.float32(0.4)).astype(np.float32)

    def tern(base, n):
        w = np.sin((np.arange(n, dtype=np.float32) + np.float32(base)) * np.float32(0.05)).astype(np.float32)
        return fo.quantize_ternary(w)

    gate, gs, up, us, down, ds = [], [], [], [], [], []
    for e in range(E):
        q, a = tern(e * 0.1, F * H); gate.append(q); gs.append(np.full(F, a, np.float32))
        q, a = tern(e * 0.1 + 0.5, F * H); up.append(q); us.append(np.full(F, a, np.float32))
        q, a = tern(e * 0.1 + 1.0, H * F); down.append(q); ds.append(np.full(H, a, np.float32))
    x = (np.arange(H, dtype=np.float32) * np.float32(0.1)).astype(np.float32)
    y, route, _ = fo.moe_forward(router, gate, gs, up, us, down, ds, H, F, 2, x, 1)
    assert y.shape == (H,) and np.abs(y).max() > 1e-10
    y3, _, _ = fo.moe_forward(router, gate, gs, up, us, down, ds, H, F, 2,
                              np.full(3 * H, 0.1, np.float32), 3)
    assert y3.shape == (3 * H,)


# ---------------------------------------------------------- flash decode
def test_flash_decode_matches_softmax_attention():
    # tests/kernel_tests.rs:1073-1110 inputs (sin/cos sequences), 1 head
    # group, checked against a direct float64 softmax-attention.
    S, Hh, D = 8, 2, 4
    q = np.sin(np.arange(Hh * D) * 0.1).astype(np.float32)
    k = np.cos(np.arange(S * Hh * D) * 0.05).astype(np.float32)
    v = np.sin(np.arange(S * Hh * D) * 0.07).astype(np.float32)
    out = fo.flash_decode_gqa(q, k, v, 1, S, Hh, Hh, D)
    K = k.reshape(S, Hh, D).astype(np.float64)
    V = v.reshape(S, Hh, D).astype(np.float64)
    Q = q.reshape(Hh, D).astype(np.float64)
    ref = np.zeros((Hh, D))
    for h in range(Hh):
        sc = K[:, h] @ Q[h] / math.sqrt(D)
        w = np.exp(sc - sc.max())
        ref[h] = (w / w.sum()) @ V[:, h]
    assert np.abs(out.reshape(Hh, D) - ref).max() < 1e-3


def test_int8_mode_integer_equals_reference_f32():
    # int8 mode: the reference's f32 ternary_matmul on int8 codes-as-f32 is
    # exact (|sum| <= 127*K < 2^24), so it equals the int32 path bit for bit.
    rng = np.random.default_rng(7)
    M, K, N = 3, 512, 40
    t = rng.integers(-1, 2, size=N * K).astype(np.int8)
    x = rng.standard_normal(M * K).astype(np.float32)
    q, sx = fo.quantize_absmax_i8(x, M, K)
    sw = rng.uniform(0.01, 0.1, N).astype(np.float32)
    a = fo.ternary_matmul_i8(t, q, sx, sw, M, K, N)
    b = fo.ternary_matmul_i8(t, q, sx, sw, M, K, N, via_f32=True)
    assert (a.view(np.uint32) == b.view(np.uint32)).all()


def test_quantize_absmax_i8_edges():
    x = np.array([0, 0, 0, 0, 1.0, -2.0, 0.5, 0.0, 127.0, -127.0, 0.5, 1.5], np.float32)
    q, sx = fo.quantize_absmax_i8(x, 3, 4)
    assert list(q[0:4]) == [0, 0, 0, 0] and sx[0] == 1.0
    assert sx[1] == np.float32(2.0) / np.float32(127.0)
    assert list(q[4:8]) == [64, -127, 32, 0]  # 63.5 rounds half away from zero
    assert list(q[8:12]) == [127, -127, 1, 2]


# ------------------------------------ block scales and index lists (A7, (f)4)
def _cosine(a, b):
    a, b = np.asarray(a, np.float64), np.asarray(b, np.float64)
    return float(a @ b / (np.linalg.norm(a) * np.linalg.norm(b)))


def test_blocked_quantize_roundtrip():  # ternary.rs:824-843
    w = np.sin(np.arange(1000, dtype=np.float32) * np.float32(0.01) - np.float32(5.0))
    q, s = fo.quantize_ternary_blocked(w, 128)
    assert s.size == 8
    r = np.repeat(s, 128)[:1000] * q.astype(np.float32)
    assert _cosine(w, r) > 0.90


def test_blocked_vs_per_tensor():  # ternary.rs:846-873
    i = np.arange(512, dtype=np.float32)
    w = np.where(i < 256, i * np.float32(0.001) - np.float32(0.128),
                 i * np.float32(0.01) - np.float32(2.56)).astype(np.float32)
    qt, st = fo.quantize_ternary(w)
    qb, sb = fo.quantize_ternary_blocked(w, 64)
    cos_t = _cosine(w, qt.astype(np.float32) * st)
    cos_b = _cosine(w, np.repeat(sb, 64) * qb.astype(np.float32))
    assert cos_b >= cos_t - 0.01


def blocked_kat_case():
    """The inputs of ternary.rs:1098-1176 (test_ternary_matmul_blocked_vs_scalar)."""
    out_rows, in_cols, bs = 4, 32, 8
    w = (np.sin(np.arange(out_rows * in_cols, dtype=np.float32) * np.float32(1.618))
         * np.float32(0.5)).astype(np.float32).reshape(out_rows, in_cols)
    nb = in_cols // bs
    scales = np.zeros(nb, np.float32)
    norm = np.float32(0.7978845608)
    for b in range(nb):
        s = np.float32(0.0)
        for r in range(out_rows):  # rows outer, columns inner: the reference's loop order
            for j in range(b * bs, (b + 1) * bs):
                s = np.float32(s + abs(w[r, j]))
        scales[b] = np.float32(np.float32(s / np.float32(out_rows * bs)) / norm) if s > 0 else 1
    t = np.zeros((out_rows, in_cols), np.int8)
    for b in range(nb):
        inv = np.float32(np.float32(1.0) / scales[b])
        v = (w[:, b * bs:(b + 1) * bs] * inv).astype(np.float32)
        t[:, b * bs:(b + 1) * bs] = np.clip(np.trunc(v + np.copysign(np.float32(0.5), v)), -1, 1)
    x = np.cos(np.arange(in_cols, dtype=np.float32) * np.float32(0.1)).astype(np.float32)
    ref = np.zeros(out_rows, np.float32)
    for r in range(out_rows):
        for b in range(nb):
            for j in range(b * bs, (b + 1) * bs):
                ref[r] = np.float32(ref[r] + np.float32(scales[b] * np.float32(t[r, j])) * x[j])
    return t.ravel(), scales, bs, x, out_rows, in_cols, ref


def test_ternary_matmul_blocked_vs_scalar():  # ternary.rs:1098-1176
    t, scales, bs, x, rows, cols, ref = blocked_kat_case()
    y = fo.ternary_matmul_blocked(t, scales, bs, x, rows, cols, 1)
    assert np.abs(y - ref).max() < 1e-4


def test_ternary_sparse_decode_vs_general():  # ternary.rs:1208-1235
    rows, cols, scale = 4, 16, 0.5
    i = np.arange(rows * cols)
    t = np.where(i % 3 == 0, 1, np.where(i % 3 == 1, -1, 0)).astype(np.int8)
    x = (np.arange(cols, dtype=np.float32) * np.float32(0.1)).astype(np.float32)
    po, pi, no, ni = fo.ternary_sparse_indices(t, rows, cols)
    y = fo.ternary_matmul_sparse_decode(po, pi, no, ni, scale, x, rows)
    g = fo.ternary_matmul_decode(t, scale, x, rows, cols)
    assert np.abs(y - g).max() < 1e-5


def test_sparse_indices_counts():  # ternary.rs:1238-1253
    t = np.array([1, -1, 0, 1, -1, 0, 0, -1, 0, 0, 0, 0], np.int8)
    po, pi, no, ni = fo.ternary_sparse_indices(t, 3, 4)
    assert list(pi[po[0]:po[1]]) == [0, 3] and list(ni[no[0]:no[1]]) == [1]
    assert list(pi[po[1]:po[2]]) == [] and list(ni[no[1]:no[2]]) == [0, 3]
    assert list(pi[po[2]:po[3]]) == [] and list(ni[no[2]:no[3]]) == []


def test_bitmoe_synchronized_alpha_and_requantize():  # bit_moe.rs:319-386
    # make_test_bit_moe: hidden 4, inter 8, 2 experts, weights sin((i + base) * 0.1);
    # init_shadows_from_ternary then recompute_alpha; requantize with that alpha.
    import torch
    hd, idim, ne = 4, 8, 2
    mats = []
    for e in range(ne):
        for base, size in ((e, idim * hd), (e + 0.5, idim * hd), (e + 1.0, hd * idim)):
            w = np.sin((np.arange(size, dtype=np.float32) + np.float32(base)) * np.float32(0.1))
            q, a = fo.quantize_ternary(w.astype(np.float32))
            shadow = torch.from_numpy(q.astype(np.float32) * a).to(torch.bfloat16)
            mats.append(shadow.view(torch.int16).numpy().view(np.uint16))
    alpha = fo.bitmoe_recompute_alpha(mats)
    assert alpha is not None and alpha > 0
    for m in mats:
        q = fo.bitmoe_requantize(m, alpha)
        assert set(np.unique(q)) <= {-1, 0, 1}
    assert fo.bitmoe_recompute_alpha([]) is None
    assert (fo.bitmoe_requantize(mats[0], 0.0) == 0).all()  # alpha < 1e-10 -> all zero


def test_kvt_known_answers():
    """Mode T of the 3-bit KV cache (own spec): v = D (H e_0) = the signs gives
    D v = 1, H 1 = 128 e_0, norm sqrt(128), rotated y = sqrt(128) e_0: code 7
    at 0 (clamped) and code 4 (the centroid above 0) elsewhere."""
    s = fo.kvt_signs(42)
    assert set(np.unique(s)) == {-1.0, 1.0}
    codes, norm = fo.kvt_quantize(s, s)
    assert norm == np.float32(np.sqrt(np.float32(128)))
    assert codes[0] == 7 and (codes[1:] == 4).all()
    # zero vector: norm 0, every code 4, (min, max) = (-0, 0)
    p, mm = fo.kvt_store_vector(np.zeros(128, np.float32), s)
    assert (fo.unpack_3bit(p, 128) == 4).all() and mm.tolist() == [0.0, 0.0]
    # the rotation is orthonormal: forward then inverse is the identity to fp32 rounding
    rng = np.random.default_rng(0)
    x = rng.standard_normal(128).astype(np.float32)
    y = fo.kvt_rotate(x, s)
    assert abs(np.linalg.norm(y) - np.linalg.norm(x)) < 1e-5 * np.linalg.norm(x)
    assert np.max(np.abs(fo.kvt_rotate(y, s, inverse=True) - x)) < 1e-5
    # Gaussian vectors: relative reconstruction error near the 8-level
    # uniform quantiser's (step 0.625 sigma -> about 0.19)
    v = rng.standard_normal((64, 128)).astype(np.float32)
    err = [np.linalg.norm(fo.kvt_load_vector(*fo.kvt_store_vector(r, s), s) - r) / np.linalg.norm(r)
           for r in v]
    assert 0.12 < np.mean(err) < 0.25, np.mean(err)
