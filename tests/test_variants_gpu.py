"""GPU parity of the block-scale, index-list and fp32-ingestion entry points.

* ternary_matmul_blocked (src/model/ternary.rs:541-579) against the oracle's
  restatement, under the fp32 rule of tests/helpers.py with the condition
  sum_k |scale_b(k) * W[r,k] * x[k]|; the reference's own known answer
  (ternary.rs:1098-1176) on the GPU; non-finite inputs with the products'
  semantics of that function (0 * inf = NaN).
* Index lists (ternary_sparse_indices / ternary_matmul_sparse_decode,
  ternary.rs:647-707): upload and decode against the oracle; malformed lists
  are refused.
* fp32 ingestion (quantize_ternary, ternary.rs:31-57, via
  TernaryExpert::from_fp32, src/model/cpu_moe.rs:33-37): codes read back
  bit for bit and alpha bit for bit against the oracle.
* STE re-quantization with a layer-shared alpha (src/training/bit_moe.rs:
  210-262): alpha and codes bit for bit against the oracle.
* A MoE layer built from fp32 experts against the oracle's
  TernaryMoELayer::forward on the oracle-quantized experts.
"""
import numpy as np
import pytest
import torch

from oracle import oracle as fo
from tests.helpers import assert_fp32_close, ternary_matrix

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def gpu():
    assert torch.cuda.is_available()
    from ferrisres_b200 import gpu as g
    return g


def blocked_condition(t, scales, bs, x, rows, cols, seq):
    a = np.repeat(np.abs(scales.astype(np.float64)), bs)[:cols]
    W = np.abs(t.reshape(rows, cols).astype(np.float64)) * a[None, :]
    return (np.abs(x.reshape(seq, cols).astype(np.float64)) @ W.T).ravel()


@pytest.mark.parametrize("rows,cols,seq,bs", [(300, 512, 1, 128), (1024, 2048, 2, 64),
                                              (129, 1000, 3, 100), (640, 1408, 40, 8),
                                              (64, 257, 5, 1)])
def test_blocked_matches_oracle(gpu, rows, cols, seq, bs):
    rng = np.random.default_rng(rows + cols + seq + bs)
    t = ternary_matrix(rng, rows, cols)
    nb = -(-cols // bs)
    scales = rng.uniform(0.01, 2.0, nb).astype(np.float32)
    x = rng.standard_normal(seq * cols).astype(np.float32)
    w = gpu.DeviceTernaryWeight.from_packed_u8(fo.pack_ternary(t), rows, cols,
                                               np.ones(rows, np.float32))
    y = w.matmul_blocked_f32(torch.from_numpy(x).cuda().view(seq, cols),
                             torch.from_numpy(scales).cuda(), bs).cpu().numpy().ravel()
    ref = fo.ternary_matmul_blocked(t, scales, bs, x, rows, cols, seq)
    assert_fp32_close(y, ref, blocked_condition(t, scales, bs, x, rows, cols, seq),
                      what=f"blocked {rows}x{cols}x{seq} bs {bs}")


def test_blocked_reference_known_answer(gpu):
    from tests.test_oracle_kats import blocked_kat_case
    t, scales, bs, x, rows, cols, ref = blocked_kat_case()
    w = gpu.DeviceTernaryWeight.from_packed_u8(fo.pack_ternary(t), rows, cols,
                                               np.ones(rows, np.float32))
    y = w.matmul_blocked_f32(torch.from_numpy(x).cuda().view(1, cols),
                             torch.from_numpy(scales).cuda(), bs).cpu().numpy().ravel()
    assert np.abs(y - ref).max() < 1e-4  # the reference test's bound


@pytest.mark.parametrize("seq", [1, 5])
def test_blocked_nonfinite(gpu, seq):
    rows, cols, bs = 512, 512, 64
    rng = np.random.default_rng(seq)
    t = ternary_matrix(rng, rows, cols)
    scales = rng.uniform(0.5, 1.5, cols // bs).astype(np.float32)
    x = rng.standard_normal((seq, cols)).astype(np.float32)
    x[0, 10] = np.inf
    if seq > 1:
        x[1, 300] = np.nan
        x[2, 20], x[2, 21] = np.inf, -np.inf
    x = x.ravel()
    w = gpu.DeviceTernaryWeight.from_packed_u8(fo.pack_ternary(t), rows, cols,
                                               np.ones(rows, np.float32))
    y = w.matmul_blocked_f32(torch.from_numpy(x).cuda().view(seq, cols),
                             torch.from_numpy(scales).cuda(), bs).cpu().numpy().ravel()
    ref = fo.ternary_matmul_blocked(t, scales, bs, x, rows, cols, seq)
    assert np.array_equal(np.isnan(y), np.isnan(ref))
    inf = np.isinf(ref)
    assert np.array_equal(np.isinf(y), inf) and np.array_equal(np.sign(y[inf]), np.sign(ref[inf]))
    fin = np.isfinite(ref)
    xf = np.where(np.isfinite(x), x, 0).astype(np.float32)
    cond = blocked_condition(t, scales, bs, xf, rows, cols, seq)
    assert_fp32_close(y[fin], ref[fin], cond[fin], what="blocked finite outputs")


@pytest.mark.parametrize("rows,cols,p_zero", [(5632, 2048, 1 / 3), (300, 777, 0.9), (7, 16, 0.5)])
def test_index_lists_decode(gpu, rows, cols, p_zero):
    from ferrisres_b200 import ternary as T
    rng = np.random.default_rng(rows + cols)
    t = ternary_matrix(rng, rows, cols, p_zero=p_zero)
    pos, neg = T.ternary_sparse_indices(t, rows, cols)
    x = rng.standard_normal(cols).astype(np.float32)
    scale = np.float32(0.37)
    w = gpu.DeviceTernaryWeight.from_sparse_indices(pos, neg, rows, cols, scale)
    assert (w.export_packed_u8() == fo.pack_ternary(t)).all()
    y = w.matmul_f32(torch.from_numpy(x).cuda().view(1, cols)).cpu().numpy().ravel()
    po, pi, no, ni = fo.ternary_sparse_indices(t, rows, cols)
    ref = fo.ternary_matmul_sparse_decode(po, pi, no, ni, scale, x, rows)
    cond = (np.abs(t.reshape(rows, cols).astype(np.float64)) @ np.abs(x.astype(np.float64))) * scale
    assert_fp32_close(y, ref, cond, what="sparse decode")
    y2 = gpu.ternary_matmul_sparse_decode(pos, neg, scale, x, rows)
    assert_fp32_close(y2, ref, cond, what="sparse decode (host form)")


def test_index_lists_rejected_when_malformed(gpu):
    from ferrisres_b200._lib import ShapeError
    ok = [np.array([0, 3])]
    for pos, neg in (([np.array([3, 0])], [np.array([], np.int64)]),   # out of order
                     ([np.array([0, 9])], [np.array([], np.int64)]),   # out of range
                     (ok, [np.array([3])])):                            # in both lists
        with pytest.raises(ShapeError):
            gpu.DeviceTernaryWeight.from_sparse_indices(pos, neg, 1, 8, 1.0)


@pytest.mark.parametrize("rows,cols", [(300, 512), (1408, 2048), (5, 7)])
def test_fp32_ingestion_bit_exact(gpu, rows, cols):
    rng = np.random.default_rng(rows * cols)
    w = (rng.standard_normal(rows * cols) * 0.02).astype(np.float32)
    w[:3] = [0.0, 1e3, -1e3]  # large magnitudes clamp to +-1
    dw = gpu.DeviceTernaryWeight.from_fp32(w, rows, cols)
    q, a = fo.quantize_ternary(w)
    assert np.float32(dw.alpha).view(np.uint32) == np.float32(a).view(np.uint32)
    assert (dw.export_packed_u8() == fo.pack_ternary(q)).all()
    # and the weight computes with alpha as its row scale
    x = rng.standard_normal(cols).astype(np.float32)
    y = dw.matmul_f32(torch.from_numpy(x).cuda().view(1, cols)).cpu().numpy().ravel()
    ref = fo.gpu_ternary_mm_cpu(fo.pack_ternary_rows_u32(q, rows, cols),
                                np.full(rows, a, np.float32), x, 1, cols, rows) \
        if cols % 16 == 0 else fo.ternary_matmul(q, a, x, rows, cols, 1)
    cond = (np.abs(q.reshape(rows, cols).astype(np.float64)) @ np.abs(x.astype(np.float64))) * a
    assert_fp32_close(y, ref, cond, what="ingested weight")


def test_ste_shared_alpha_requantize(gpu):
    rng = np.random.default_rng(11)
    shapes = [(1408, 2048), (1408, 2048), (2048, 1408), (96, 64)]
    shadows = [torch.from_numpy((rng.standard_normal(r * c) * 0.03).astype(np.float32))
               .to(torch.bfloat16).view(r, c).cuda() for r, c in shapes]
    alpha = gpu.shadow_alpha(shadows)
    bits = [s.view(torch.int16).cpu().numpy().view(np.uint16).ravel() for s in shadows]
    ref_alpha = fo.bitmoe_recompute_alpha(bits)
    assert np.float32(alpha).view(np.uint32) == np.float32(ref_alpha).view(np.uint32)
    for (r, c), s, b in zip(shapes, shadows, bits):
        w = gpu.DeviceTernaryWeight.from_packed_u8(np.full((r * c + 3) // 4, 0x55, np.uint8), r,
                                                   c, np.ones(r, np.float32))
        w.requantize(s, alpha)
        torch.cuda.synchronize()
        assert (w.export_packed_u8() == fo.pack_ternary(fo.bitmoe_requantize(b, alpha))).all()
    # alpha below 1e-10 quantizes everything to zero
    w.requantize(shadows[-1], 1e-12)
    torch.cuda.synchronize()
    assert (w.export_packed_u8() == fo.pack_ternary(np.zeros(96 * 64, np.int8))).all()
    assert gpu.shadow_alpha([]) is None


def test_moe_from_fp32_matches_oracle(gpu):
    from ferrisres_b200 import moe
    rng = np.random.default_rng(12)
    E, H, F, T, K = 8, 256, 128, 48, 2
    router = (rng.standard_normal(E * H) * 0.05).astype(np.float32)
    g = [(rng.standard_normal(F * H) * 0.02).astype(np.float32) for _ in range(E)]
    u = [(rng.standard_normal(F * H) * 0.02).astype(np.float32) for _ in range(E)]
    d = [(rng.standard_normal(H * F) * 0.02).astype(np.float32) for _ in range(E)]
    layer = moe.TernaryMoELayer.from_fp32(router, g, u, d, H, F, K)
    x = rng.standard_normal((T, H)).astype(np.float32)
    y = layer.forward_device(torch.from_numpy(x).cuda()).cpu().numpy()
    qs = [fo.quantize_ternary(m) for m in g], [fo.quantize_ternary(m) for m in u], \
        [fo.quantize_ternary(m) for m in d]
    gq, uq, dq = [[q for q, _ in lst] for lst in qs]
    gs = [np.full(F, a, np.float32) for _, a in qs[0]]
    us = [np.full(F, a, np.float32) for _, a in qs[1]]
    ds = [np.full(H, a, np.float32) for _, a in qs[2]]
    ref, _, probs = fo.moe_forward(router, gq, gs, uq, us, dq, ds, H, F, K, x.ravel(), T)
    ref = ref.reshape(T, H).astype(np.float64)
    p = probs.reshape(T, E)
    srt = -np.sort(-p, axis=1)
    tie = (srt[:, K - 1] - srt[:, K]) < 1e-6
    rms = np.sqrt(np.mean(ref ** 2, axis=1, keepdims=True))
    err = np.abs(y - ref) / (1e-4 * rms + 1e-7)
    assert (err.max(axis=1)[~tie] <= 1.0).all()


def test_fp32_ingestion_edge_values(gpu):
    """NaN (sum |w| is NaN, so alpha = 1, and NaN quantizes to 0 as Rust's `as i32`
    maps it), infinities and huge values saturate to +-1."""
    w = np.array([0.0, np.nan, 1e30, -1e30, np.inf, -np.inf, 0.5, -0.5, 0.49, 2.0, -3.0, 1e-30],
                 np.float32)
    dw = gpu.DeviceTernaryWeight.from_fp32(w, 3, 4)
    q, a = fo.quantize_ternary(w)
    assert np.float32(dw.alpha).view(np.uint32) == np.float32(a).view(np.uint32)
    assert (dw.export_packed_u8() == fo.pack_ternary(q)).all()


def test_checkpoint_moe_layers(gpu, tmp_path):
    """A FerrisRes checkpoint (src/model/checkpoint.rs:1-29 naming, BF16 tensors as
    the reference saves them) loaded into resident MoE layers and checked against
    the oracle on the widened, oracle-quantized experts."""
    import json

    from ferrisres_b200 import checkpoint as ck
    rng = np.random.default_rng(13)
    E, H, F, T = 8, 256, 128, 40
    tensors, layer_cfg, refs = {}, [], {}
    for i in range(3):
        moe_layer = i != 1
        layer_cfg.append({"use_gelu": i == 2, "has_moe": moe_layer, "num_experts": E if moe_layer else 0,
                          "top_k": 2 if moe_layer else 0, "inter_dim": F})
        if not moe_layer:
            tensors[f"layers.{i}.ffn_gate"] = (rng.standard_normal((F, H)).astype(np.float32), "BF16")
            continue
        tensors[f"layers.{i}.moe.router"] = ((rng.standard_normal((E, H)) * 0.05).astype(np.float32),
                                             "BF16")
        for e in range(E):
            for nm, shape in (("gate", (F, H)), ("up", (F, H)), ("down", (H, F))):
                tensors[f"layers.{i}.moe.expert.{e}.{nm}"] = (
                    (rng.standard_normal(shape) * 0.02).astype(np.float32), "BF16")
    base = str(tmp_path / "model")
    ck.write_safetensors(base + ".safetensors", tensors)
    json.dump({"hidden_dim": H, "layer_configs": layer_cfg}, open(base + ".json", "w"))
    layers = ck.load_moe_layers(base)
    assert sorted(layers) == [0, 2]
    st = ck.SafeTensors(base + ".safetensors")
    x = rng.standard_normal((T, H)).astype(np.float32)
    for i, layer in layers.items():
        y = layer.forward_device(torch.from_numpy(x).cuda()).cpu().numpy()
        router = st.get_f32(f"layers.{i}.moe.router").ravel()
        q = {nm: [fo.quantize_ternary(st.get_f32(f"layers.{i}.moe.expert.{e}.{nm}").ravel())
                  for e in range(E)] for nm in ("gate", "up", "down")}
        sc = {nm: [np.full(F if nm != "down" else H, a, np.float32) for _, a in q[nm]] for nm in q}
        ref, _, probs = fo.moe_forward(router, [t for t, _ in q["gate"]], sc["gate"],
                                       [t for t, _ in q["up"]], sc["up"], [t for t, _ in q["down"]],
                                       sc["down"], H, F, 2, x.ravel(), T, use_gelu=i == 2)
        ref = ref.reshape(T, H).astype(np.float64)
        srt = -np.sort(-probs.reshape(T, E), axis=1)
        tie = (srt[:, 1] - srt[:, 2]) < 1e-6
        rms = np.sqrt(np.mean(ref ** 2, axis=1, keepdims=True))
        err = np.abs(y - ref) / (1e-4 * rms + 1e-7)
        assert (err.max(axis=1)[~tie] <= 1.0).all(), f"layer {i}"
    # expert-parallel partial load: rank 1 of 2 holds experts 4..7 only
    part = ck.load_moe_layer(st, 0, rank=1, world=2)
    assert part.n_experts == E
