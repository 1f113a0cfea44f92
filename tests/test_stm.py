""".stm expert files: the reference's format tests (src/model/expert_loader.rs:
437-520) restated, the directory loader, and (GPU) a file uploaded straight
into a resident sparse weight, checked against the CPU oracle's 2:4 matmul."""
import os
import struct

import numpy as np
import pytest

from ferrisres_b200 import stm
from oracle import oracle as fo
from tests.helpers import assert_fp32_close, condition


def make_test_sparse(rows, cols, scale=0.5):
    """The reference's test matrix (expert_loader.rs:425-435): value i is
    ((i * 2654435761 mod 2^32) >> 30) - 1 clamped to [-1, 1], packed by
    SparseTernaryMatrix::from_ternary."""
    i = np.arange(rows * cols, dtype=np.uint64)
    v = ((i * np.uint64(2654435761)) & np.uint64(0xFFFFFFFF)) >> np.uint64(30)
    t = np.clip(v.astype(np.int64) - 1, -1, 1).astype(np.int8)
    pat, sg = fo.sparse_from_ternary(t, rows, cols)
    return stm.SparseTernaryMatrix(pat, sg, scale, rows, cols), t


def test_stm_write_read_roundtrip(tmp_path):
    orig, _ = make_test_sparse(8, 16)
    p = tmp_path / "test.stm"
    stm.write_stm(p, orig)
    got = stm.read_stm(p)
    assert (got.rows, got.cols) == (orig.rows, orig.cols)
    assert abs(got.scale - orig.scale) < 1e-6
    assert np.array_equal(got.patterns, orig.patterns)
    assert np.array_equal(got.signs, orig.signs)
    assert np.array_equal(fo.sparse_to_ternary(got.patterns, got.signs, 8, 16),
                          fo.sparse_to_ternary(orig.patterns, orig.signs, 8, 16))
    # the 24-byte header is the reference's little-endian layout
    raw = p.read_bytes()
    assert struct.unpack_from("<IIIfII", raw, 0) == (
        0x53544D31, 8, 16, 0.5, orig.patterns.size, orig.signs.size)
    assert len(raw) == 24 + orig.patterns.size + orig.signs.size


def test_stm_mmap_roundtrip(tmp_path):
    import mmap
    orig, _ = make_test_sparse(4, 8)
    p = tmp_path / "test_mmap.stm"
    stm.write_stm(p, orig)
    with open(p, "rb") as f, mmap.mmap(f.fileno(), 0, access=mmap.ACCESS_READ) as m:
        got = stm.read_stm_mmap(m)
    assert (got.rows, got.cols) == (4, 8)
    assert np.array_equal(got.patterns, orig.patterns)
    assert np.array_equal(got.signs, orig.signs)


def test_stm_invalid_magic(tmp_path):
    p = tmp_path / "bad.stm"
    p.write_bytes(struct.pack("<IIIfII", 0xDEADBEEF, 0, 0, 0.0, 0, 0))
    with pytest.raises(stm.StmFormatError, match="magic"):
        stm.read_stm(p)


def test_stm_truncated_file(tmp_path):
    p = tmp_path / "trunc.stm"
    p.write_bytes(struct.pack("<I", 0x53544D31))  # magic only, no header
    with pytest.raises(stm.StmFormatError):
        stm.read_stm(p)
    orig, _ = make_test_sparse(4, 8)
    q = tmp_path / "short.stm"
    stm.write_stm(q, orig)
    q.write_bytes(q.read_bytes()[:-1])  # one data byte short
    with pytest.raises(stm.StmFormatError, match="truncated"):
        stm.read_stm(q)


def test_loader_naming_and_stats(tmp_path):
    orig, _ = make_test_sparse(8, 16)
    stm.write_stm(tmp_path / "layer_00_expert_1.stm", orig)
    stm.write_stm(tmp_path / "layer_01_expert_0.stm", orig)
    ld = stm.ExpertLoader.open(tmp_path, num_layers=2, num_experts=2, hidden_dim=8, top_k=1)
    try:
        assert ld.cache_hit_rate() == 0.0 and ld.cache_size() == 0
        assert ld._maps[0][0] is None and ld._maps[0][1] is not None
        assert ld._maps[1][0] is not None and ld._maps[1][1] is None
        assert ld.ensure_loaded(0, 0) is False  # missing file: a miss, nothing loaded
        assert ld.stats.cache_misses == 1 and ld.cache_size() == 0
    finally:
        ld.close()


def test_loader_route_matches_reference_order():
    """route(): softmax over router[e*hd + j] . x, top-k by descending
    probability (expert_loader.rs:260-290) -- here against float64."""
    ld = stm.ExpertLoader.open("/nonexistent-dir", 1, 5, 4, 2)
    rng = np.random.default_rng(3)
    r = rng.standard_normal(5 * 4).astype(np.float32)
    x = rng.standard_normal(4).astype(np.float32)
    ld.set_routers([r])
    got = ld.route(0, x)
    ref = np.argsort(-(r.reshape(5, 4).astype(np.float64) @ x.astype(np.float64)),
                     kind="stable")[:2]
    assert got == list(ref)
    ld.close()


@pytest.mark.gpu
def test_stm_upload_matches_oracle(tmp_path):
    import torch
    assert torch.cuda.is_available()
    rows, cols, seq = 300, 512, 3
    orig, t = make_test_sparse(rows, cols, scale=0.07)
    p = tmp_path / "layer_00_expert_0.stm"
    stm.write_stm(p, orig)
    ld = stm.ExpertLoader.open(tmp_path, 1, 1, cols, 1)
    try:
        assert ld.ensure_loaded(0, 0)
        w = ld.get_expert(0, 0)
        assert ld.ensure_loaded(0, 0) and ld.stats.cache_hits == 1
        rng = np.random.default_rng(5)
        x = rng.standard_normal(seq * cols).astype(np.float32)
        y = w.matmul_f32(torch.from_numpy(x).cuda().view(seq, cols)).cpu().numpy()
        dense = fo.sparse_to_ternary(orig.patterns, orig.signs, rows, cols)
        ref = fo.sparse_ternary_matmul(orig.patterns, orig.signs, 0.07,
                                       np.full(rows, 0.07, np.float32), rows, cols, x, seq)
        assert_fp32_close(y, ref, condition(dense, x, rows, cols, seq,
                                            np.full(rows, 0.07, np.float32)), what="stm")
        # the direct upload path gives the same weight
        w2 = stm.upload_stm(p)
        y2 = w2.matmul_f32(torch.from_numpy(x).cuda().view(seq, cols)).cpu().numpy()
        assert np.array_equal(y, y2)
    finally:
        ld.close()
