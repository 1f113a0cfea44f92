"""GPU parity of the 3-bit KV cache and its flash decode.

Stored form (codes and per-vector min/max) and get_range dequantisation are
bit-exact against the oracle's restatement of TurboQuantKVCache
(src/inference/turboquant_kv.rs:83-117, :240-291, :370-410).  The flash
decode is compared with the oracle's flash_decode_ref restatement
(tests/kernel_tests.rs:1073-1110, GQA map src/model/cpu_block_attn_res.rs:471-472)
over the same stored cache, and with a float64 evaluation of the same math:
    |out - exact64| <= 1e-5 * (1 + |exact64|)     (our kernel)
    |out - oracle|  <= 2e-5 * (1 + |exact64|)     (the fp32 oracle itself
                                                     drifts with the length)
"""
import numpy as np
import pytest
import torch

from oracle import oracle as fo

pytestmark = pytest.mark.gpu

D = 128


@pytest.fixture(scope="module")
def kv():
    assert torch.cuda.is_available()
    from ferrisres_b200 import kv as kvmod
    return kvmod


def rand_kv(rng, B, S, Hkv, special=True):
    k = rng.standard_normal((B, S, Hkv, D)).astype(np.float32)
    v = rng.standard_normal((B, S, Hkv, D)).astype(np.float32)
    if special and S > 3:
        k[0, 1, 0, :] = 3.14  # constant vector: range 0, all codes 0
        v[0, 2, -1, :] = -2.0
        k[-1, 3, -1, :] = np.arange(D) % 8  # codes == values
        v[-1, 0, 0, ::2] = 5.0  # ties at the maximum
    return k, v


def oracle_store(k, v):
    """Reference stored form: codes [B, S, Hkv*48], min/max [B, S, Hkv, 2]."""
    B, S, Hkv, _ = k.shape
    kc = np.zeros((B, S, Hkv * 48), np.uint8)
    vc = np.zeros_like(kc)
    km = np.zeros((B, S, Hkv, 2), np.float32)
    vm = np.zeros_like(km)
    for b in range(B):
        for s in range(S):
            p, mm = fo.kv_quantize_vector(k[b, s].reshape(-1), D)
            kc[b, s], km[b, s] = p, mm.reshape(Hkv, 2)
            p, mm = fo.kv_quantize_vector(v[b, s].reshape(-1), D)
            vc[b, s], vm[b, s] = p, mm.reshape(Hkv, 2)
    return kc, km, vc, vm


def oracle_dequant(kc, km, Hkv):
    B, S = kc.shape[:2]
    out = np.zeros((B, S, Hkv, D), np.float32)
    for b in range(B):
        for s in range(S):
            out[b, s] = fo.kv_dequantize_vector(kc[b, s], km[b, s].reshape(-1), Hkv * D,
                                                D).reshape(Hkv, D)
    return out


def exact_decode(q, kd, vd, Hq, Hkv, scale=None):
    """float64 softmax attention over dequantised K/V [B, S, Hkv, D], q [B, Hq, D]."""
    B = q.shape[0]
    G = Hq // Hkv
    scale = 1.0 / np.sqrt(D) if scale is None else scale
    out = np.zeros((B, Hq, D))
    for b in range(B):
        for h in range(Hq):
            kk = kd[b, :, h // G, :].astype(np.float64)
            s = kk @ q[b, h].astype(np.float64) * scale
            w = np.exp(s - s.max())
            out[b, h] = (w[:, None] * vd[b, :, h // G, :]).sum(0) / w.sum()
    return out


def check_decode(out, q, store, Hq, Hkv):
    kc, km, vc, vm = store
    B, S = kc.shape[:2]
    ref = fo.flash_decode_3bit(q, kc, km, vc, vm, B, S, Hq, Hkv, D).reshape(B, Hq, D)
    ex = exact_decode(q, oracle_dequant(kc, km, Hkv), oracle_dequant(vc, vm, Hkv), Hq, Hkv)
    out = out.reshape(B, Hq, D).astype(np.float64)
    bound = 1.0 + np.abs(ex)
    e_ex = np.max(np.abs(out - ex) / bound)
    e_or = np.max(np.abs(out - ref) / bound)
    assert e_ex <= 1e-5, f"vs float64: {e_ex:.3e}"
    assert e_or <= 2e-5, f"vs oracle: {e_or:.3e}"
    return e_ex, e_or


def to_dev(a):
    return torch.from_numpy(np.ascontiguousarray(a)).cuda()


def test_append_export_bit_exact(kv):
    rng = np.random.default_rng(1)
    B, S, Hkv = 2, 77, 2
    k, v = rand_kv(rng, B, S, Hkv)
    c = kv.Kv3Cache(B, Hkv, 128)
    for a, e in ((0, 1), (1, 31), (31, 77)):  # partial blocks, a block boundary
        c.append(to_dev(k[:, a:e]), to_dev(v[:, a:e]))
    assert len(c) == S
    kc, km, vc, vm = (t.cpu().numpy() for t in c.export_range(0, S))
    rk, rkm, rv, rvm = oracle_store(k, v)
    assert (kc == rk).all() and (vc == rv).all()
    assert (km.view(np.uint32) == rkm.view(np.uint32)).all()
    assert (vm.view(np.uint32) == rvm.view(np.uint32)).all()
    # get_range: the reference dequantisation, bit for bit
    gk, gv = (t.cpu().numpy() for t in c.get_range(5, 70))
    assert (gk.view(np.uint32) == oracle_dequant(rk, rkm, Hkv)[:, 5:70].view(np.uint32)).all()
    assert (gv.view(np.uint32) == oracle_dequant(rv, rvm, Hkv)[:, 5:70].view(np.uint32)).all()
    c.close()


def test_append_bf16(kv):
    rng = np.random.default_rng(2)
    B, S, Hkv = 1, 40, 3
    k, v = rand_kv(rng, B, S, Hkv)
    kb = torch.from_numpy(k).to(torch.bfloat16)
    vb = torch.from_numpy(v).to(torch.bfloat16)
    c = kv.Kv3Cache(B, Hkv, 64)
    c.append(kb.cuda(), vb.cuda())
    got = [t.cpu().numpy() for t in c.export_range(0, S)]
    ref = oracle_store(kb.float().numpy(), vb.float().numpy())
    assert (got[0] == ref[0]).all() and (got[2] == ref[2]).all()
    assert (got[1] == ref[1]).all() and (got[3] == ref[3]).all()
    c.close()


def test_reference_kats_on_device(kv):
    # turboquant_kv.rs:457-474: values 0..7 -> codes 0..7; a constant -> codes 0
    k = (np.arange(D) % 8).astype(np.float32).reshape(1, 1, 1, D)
    v = np.full((1, 1, 1, D), 3.14, np.float32)
    c = kv.Kv3Cache(1, 1, 32)
    c.append(to_dev(k), to_dev(v))
    kc, km, vc, vm = (t.cpu().numpy() for t in c.export_range(0, 1))
    assert (fo.unpack_3bit(kc.reshape(-1), D) == np.arange(D) % 8).all()
    assert km.reshape(-1).tolist() == [0.0, 7.0]
    assert (fo.unpack_3bit(vc.reshape(-1), D) == 0).all()
    assert (vm.reshape(-1) == np.float32(3.14)).all()
    gk, gv = (t.cpu().numpy().reshape(-1) for t in c.get_range(0, 1))
    assert (gk == np.arange(D) % 8).all() and (gv == np.float32(3.14)).all()
    c.close()


def test_append_packed_roundtrip(kv):
    rng = np.random.default_rng(3)
    B, S, Hkv = 2, 45, 2
    k, v = rand_kv(rng, B, S, Hkv)
    store = oracle_store(k, v)
    c = kv.Kv3Cache(B, Hkv, 64)
    c.append_packed(*(to_dev(a) for a in store))
    got = [t.cpu().numpy() for t in c.export_range(0, S)]
    for g, r in zip(got, store):
        assert (g.view(np.uint8) == r.view(np.uint8)).all()
    c.close()


@pytest.mark.parametrize("B,Hq,Hkv,S", [
    (2, 8, 2, 1),       # a single position
    (2, 8, 2, 33),      # one full block + 1
    (1, 4, 1, 1000),    # G = 4, several tiles
    (2, 8, 8, 300),     # G = 1
    (1, 16, 2, 515),    # G = 8 (two head groups per kv head)
    (3, 6, 2, 200),     # G = 3 (padded head group)
])
def test_flash_decode_vs_oracle(kv, B, Hq, Hkv, S):
    rng = np.random.default_rng(100 + S + Hq)
    k, v = rand_kv(rng, B, S, Hkv)
    q = rng.standard_normal((B, Hq, D)).astype(np.float32)
    c = kv.Kv3Cache(B, Hkv, S)
    c.append(to_dev(k), to_dev(v))
    out = c.flash_decode(to_dev(q)).cpu().numpy()
    c.ctx.check()
    check_decode(out, q, oracle_store(k, v), Hq, Hkv)
    c.close()


def test_flash_decode_scale_and_peaked(kv):
    # large logits: the softmax is nearly one-hot; explicit scale 1.0 (the
    # cpu_attention_raw convention)
    rng = np.random.default_rng(7)
    B, Hq, Hkv, S = 1, 4, 1, 700
    k, v = rand_kv(rng, B, S, Hkv, special=False)
    q = (rng.standard_normal((B, Hq, D)) * 3).astype(np.float32)
    c = kv.Kv3Cache(B, Hkv, S)
    c.append(to_dev(k), to_dev(v))
    out = c.flash_decode(to_dev(q), scale=1.0).cpu().numpy().reshape(B, Hq, D)
    kc, km, vc, vm = oracle_store(k, v)
    ex = exact_decode(q, oracle_dequant(kc, km, Hkv), oracle_dequant(vc, vm, Hkv), Hq, Hkv,
                      scale=1.0)
    assert np.max(np.abs(out - ex) / (1 + np.abs(ex))) <= 1e-5
    c.close()


def test_ring_eviction_and_growth(kv):
    rng = np.random.default_rng(11)
    B, Hq, Hkv = 2, 8, 2
    k, v = rand_kv(rng, B, 260, Hkv)
    q = rng.standard_normal((B, Hq, D)).astype(np.float32)
    c = kv.Kv3Cache(B, Hkv, 64)
    c.append(to_dev(k[:, :60]), to_dev(v[:, :60]))
    c.evict_front(37)                      # head moves to slot 37
    c.append(to_dev(k[:, 60:96]), to_dev(v[:, 60:96]))  # slots 60..63, 0..31: wraps
    assert len(c) == 59 and c.capacity == 64
    store = oracle_store(k[:, 37:96], v[:, 37:96])
    got = [t.cpu().numpy() for t in c.export_range(0, 59)]
    for g, r in zip(got, store):
        assert (g.view(np.uint8) == r.view(np.uint8)).all()
    check_decode(c.flash_decode(to_dev(q)).cpu().numpy(), q, store, Hq, Hkv)
    c.append(to_dev(k[:, 96:260]), to_dev(v[:, 96:260]))  # grows the ring
    assert len(c) == 223 and c.capacity >= 223
    store = oracle_store(k[:, 37:260], v[:, 37:260])
    got = [t.cpu().numpy() for t in c.export_range(0, 223)]
    for g, r in zip(got, store):
        assert (g.view(np.uint8) == r.view(np.uint8)).all()
    check_decode(c.flash_decode(to_dev(q)).cpu().numpy(), q, store, Hq, Hkv)
    c.ctx.check()
    c.close()


def test_append_wrapping_onto_its_own_block(kv):
    # head at slot 20 of block 0 and an append that would end inside block 0
    # again: the cache grows instead of writing one block from two CTAs
    rng = np.random.default_rng(12)
    k, v = rand_kv(rng, 1, 200, 1, special=False)
    c = kv.Kv3Cache(1, 1, 64)
    c.append(to_dev(k[:, :20]), to_dev(v[:, :20]))
    c.evict_front(20)
    c.append(to_dev(k[:, 20:76]), to_dev(v[:, 20:76]))
    assert len(c) == 56
    store = oracle_store(k[:, 20:76], v[:, 20:76])
    got = [t.cpu().numpy() for t in c.export_range(0, 56)]
    for g, r in zip(got, store):
        assert (g.view(np.uint8) == r.view(np.uint8)).all()
    c.close()


def test_mirror_api(kv):
    rng = np.random.default_rng(13)
    L, kv_dim = 2, 256
    cache = kv.TurboQuantKVCache(L, kv_dim, 8, 128)
    ks = rng.standard_normal((12, kv_dim)).astype(np.float32)
    vs = rng.standard_normal((12, kv_dim)).astype(np.float32)
    for p in range(12):  # past max_seq_len: the storage grows like the reference's Vec
        for layer in range(L):
            cache.append(layer, ks[p], vs[p])
    assert cache.seq_len() == 12
    k, v = cache.get_range(1, 3, 14)  # positions 12, 13 are past the end: zeros
    for i, p in enumerate(range(3, 12)):
        rk = fo.kv_dequantize_vector(*fo.kv_quantize_vector(ks[p], 128), kv_dim, 128)
        assert (k[i * kv_dim:(i + 1) * kv_dim] == rk).all()
    assert (k[9 * kv_dim:] == 0).all() and (v[9 * kv_dim:] == 0).all()
    cache.evict_to(4)
    assert cache.seq_len() == 4 and len(cache.layers[0]) == 4
    k0, _ = cache.get(0, 0)  # oldest remaining = position 8
    rk = fo.kv_dequantize_vector(*fo.kv_quantize_vector(ks[8], 128), kv_dim, 128)
    assert (k0 == rk).all()
    # memory_bytes / compression_ratio: (96*2 + 2*2*4*2) bytes per position per layer
    assert cache.memory_bytes() == (96 * 2 + 32) * 4 * L
    assert abs(cache.compression_ratio() - 2048 / 224) < 1e-6
    cache.reset()
    assert cache.seq_len() == 0 and cache.memory_bytes() == 0
    cache.close()


def test_errors(kv):
    from ferrisres_b200._lib import ShapeError, UnsupportedError
    c = kv.Kv3Cache(1, 2, 32)
    q = torch.zeros((1, 4, D), device="cuda")
    with pytest.raises(ShapeError):
        c.flash_decode(q)  # empty cache
    c.append(torch.zeros((1, 1, 2, D), device="cuda"), torch.zeros((1, 1, 2, D), device="cuda"))
    with pytest.raises(ShapeError):
        c.flash_decode(torch.zeros((1, 3, D), device="cuda"))  # 3 % 2 != 0
    with pytest.raises(ShapeError):
        c.get_range(0, 2)
    with pytest.raises(UnsupportedError):
        kv.Kv3Cache(1, 1, 32, head_dim=64)
    with pytest.raises(UnsupportedError):
        kv.TurboQuantKVCache(1, 16, 8, 8)
    c.ctx.check()
    c.close()


def test_full_cfg5_sampled(kv):
    """cfg5 at full size (B=32, Hq=32, Hkv=8, ctx 32768): every sequence decoded on
    the GPU; three of them checked against the oracle, and their stored form at
    512 sampled positions against the oracle's quantisation of what was appended."""
    rng = np.random.default_rng(5)
    B, Hq, Hkv, S = 32, 32, 8, 32768
    c = kv.Kv3Cache(B, Hkv, S)
    gen = torch.Generator(device="cuda").manual_seed(5)
    sample_pos = np.sort(rng.choice(S, 512, replace=False))
    kept = {}  # (b, chunk) -> appended K and V of the sampled positions, on the host
    for a in range(0, S, 4096):
        kk = torch.randn((B, 4096, Hkv, D), device="cuda", generator=gen).to(torch.bfloat16)
        vv = torch.randn((B, 4096, Hkv, D), device="cuda", generator=gen).to(torch.bfloat16)
        c.append(kk, vv)
        sel = sample_pos[(sample_pos >= a) & (sample_pos < a + 4096)] - a
        for b in (0, 17, 31):
            kept[(b, a)] = (sel + a, kk[b, sel].float().cpu().numpy(), vv[b, sel].float().cpu().numpy())
    q = rng.standard_normal((B, Hq, D)).astype(np.float32)
    out = c.flash_decode(to_dev(q)).cpu().numpy()
    c.ctx.check()
    assert np.isfinite(out).all()
    kc, km, vc, vm = (t.cpu().numpy() for t in c.export_range(0, S))
    # the appends at full size: the stored form of sampled positions equals the
    # oracle's quantisation of the appended values, bit for bit
    for (b, a), (pos, ks, vs) in kept.items():
        for i, p in enumerate(pos):
            for src, codes, mm in ((ks, kc, km), (vs, vc, vm)):
                rp, rmm = fo.kv_quantize_vector(src[i].reshape(-1), D)
                assert (codes[b, p] == rp).all(), f"codes of sequence {b}, position {p}"
                assert (mm[b, p].reshape(-1).view(np.uint32) == rmm.view(np.uint32)).all()
    for b in (0, 17, 31):
        store = (kc[b:b + 1], km[b:b + 1], vc[b:b + 1], vm[b:b + 1])
        ref = fo.flash_decode_3bit(q[b:b + 1], *store, 1, S, Hq, Hkv, D).reshape(Hq, D)
        err = np.max(np.abs(out[b] - ref) / (1 + np.abs(ref)))
        assert err <= 2e-5, f"sequence {b}: {err:.3e}"
    c.close()
