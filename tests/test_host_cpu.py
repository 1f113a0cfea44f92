"""Host-side mirrors of the reference's ternary helpers (ferrisres_b200.ternary)
against the CPU oracle.  CPU only."""
import numpy as np

from ferrisres_b200 import ternary as T
from oracle import oracle as fo


def test_quantize_ternary_blocked_matches_oracle():
    rng = np.random.default_rng(3)
    for n, bs in ((1000, 128), (515, 64), (7, 8), (4096, 4096)):
        w = rng.standard_normal(n).astype(np.float32) * rng.uniform(0.1, 3)
        q, s = T.quantize_ternary_blocked(w, bs)
        qo, so = fo.quantize_ternary_blocked(w, bs)
        assert (q == qo).all() and (s.view(np.uint32) == so.view(np.uint32)).all()
        r = T.dequantize_ternary_blocked(q, s, bs)
        assert r.shape == w.shape


def test_ternary_sparse_indices_matches_oracle():
    rng = np.random.default_rng(4)
    rows, cols = 37, 101
    t = rng.integers(-1, 2, size=rows * cols).astype(np.int8)
    pos, neg = T.ternary_sparse_indices(t, rows, cols)
    po, pi, no, ni = fo.ternary_sparse_indices(t, rows, cols)
    for r in range(rows):
        assert list(pos[r]) == list(pi[po[r]:po[r + 1]])
        assert list(neg[r]) == list(ni[no[r]:no[r + 1]])
    off, idx = T.index_lists_to_csr(pos)
    assert (off == po).all() and (idx == pi).all()


def test_safetensors_roundtrip(tmp_path):
    from ferrisres_b200 import checkpoint as ck
    rng = np.random.default_rng(5)
    a = rng.standard_normal((3, 5)).astype(np.float32)
    b = rng.standard_normal((7,)).astype(np.float32)
    p = str(tmp_path / "m.safetensors")
    ck.write_safetensors(p, {"layers.0.moe.router": (a, "BF16"), "final_norm": (b, "F32")})
    st = ck.SafeTensors(p)
    assert st.info("layers.0.moe.router") == ("BF16", (3, 5))
    # BF16 is written by truncation and widened back exactly
    want = ((a.view(np.uint32) >> 16) << 16).view(np.float32)
    assert (st.get_f32("layers.0.moe.router").view(np.uint32) == want.view(np.uint32)).all()
    assert (st.get_f32("final_norm") == b).all()
    import pytest
    from ferrisres_b200._lib import ShapeError
    with pytest.raises(ShapeError):
        st.get_f32("missing")
