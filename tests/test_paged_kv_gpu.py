"""GPU parity of the paged 3-bit KV cache (device page pool behind
PagedAttention's block tables, src/inference/paged_attention.rs).

* stored form through the block tables: bit-exact against the oracle's
  restatement of the reference quantiser (mode R) and against mode T's oracle;
* flash decode over requests of ragged lengths: the per-request oracle
  flash_decode_ref with the tolerances of the ring cache's tests, and bit-equal
  to the ring cache's decode for equal lengths (same kernel, same splits);
* fork + copy-on-write: the shared full pages stay shared, a shared partial
  page is copied before either side writes into it, and both sides read back
  their own data;
* out-of-range page ids in a caller's table are skipped by the kernels and
  reported by ft_ctx_check (FT_ERR_SHAPE); pool exhaustion raises OOMError.
"""
import ctypes as C

import numpy as np
import pytest
import torch

from oracle import oracle as fo

pytestmark = pytest.mark.gpu

D = 128


@pytest.fixture(scope="module")
def pg():
    assert torch.cuda.is_available()
    from ferrisres_b200 import paged
    return paged


def to_dev(a):
    return torch.from_numpy(np.ascontiguousarray(a)).cuda()


def store_r(x):
    """[S, Hkv, D] -> reference stored form (codes [S, Hkv*48], min/max [S, Hkv, 2])."""
    S, Hkv, _ = x.shape
    codes = np.zeros((S, Hkv * 48), np.uint8)
    mm = np.zeros((S, Hkv, 2), np.float32)
    for s in range(S):
        p, m = fo.kv_quantize_vector(x[s].reshape(-1), D)
        codes[s], mm[s] = p, m.reshape(Hkv, 2)
    return codes, mm


def store_t(x, signs):
    S, Hkv, _ = x.shape
    codes = np.zeros((S, Hkv * 48), np.uint8)
    mm = np.zeros((S, Hkv, 2), np.float32)
    for s in range(S):
        for h in range(Hkv):
            p, m = fo.kvt_store_vector(x[s, h], signs)
            codes[s, h * 48:(h + 1) * 48], mm[s, h] = p, m
    return codes, mm


def dequant_r(codes, mm):
    S, Hkv = mm.shape[:2]
    return np.stack([fo.kv_dequantize_vector(codes[s], mm[s].reshape(-1), Hkv * D, D)
                     .reshape(Hkv, D) for s in range(S)])


def exact_decode(q, kd, vd):
    """float64 attention of q [Hq, D] over one request's dequantised K/V [S, Hkv, D]."""
    Hq, Hkv = q.shape[0], kd.shape[1]
    G = Hq // Hkv
    out = np.zeros((Hq, D))
    for h in range(Hq):
        s = kd[:, h // G].astype(np.float64) @ q[h].astype(np.float64) / np.sqrt(D)
        w = np.exp(s - s.max())
        out[h] = (w[:, None] * vd[:, h // G]).sum(0) / w.sum()
    return out


def fill(cache, layer, rids, data, chunks):
    """Appends data[i] ([S_i, Hkv, D] pairs) of each request in the given chunk sizes."""
    done = [0] * len(rids)
    for n in chunks:
        live = [i for i in range(len(rids)) if done[i] + n <= data[i][0].shape[0]]
        if not live:
            continue
        k = np.stack([data[i][0][done[i]:done[i] + n] for i in live])
        v = np.stack([data[i][1][done[i]:done[i] + n] for i in live])
        cache.append(layer, [rids[i] for i in live], to_dev(k), to_dev(v))
        for i in live:
            done[i] += n
    for i, r in enumerate(rids):  # the rest one position at a time
        while done[i] < data[i][0].shape[0]:
            j = done[i]
            cache.append(layer, [r], to_dev(data[i][0][None, j:j + 1]),
                         to_dev(data[i][1][None, j:j + 1]))
            done[i] += 1


@pytest.mark.parametrize("mode", ["R", "T"])
def test_paged_store_and_decode_ragged(pg, mode):
    rng = np.random.default_rng(21)
    Hkv, Hq, lens = 2, 8, [1, 45, 100, 257]
    cache = pg.PagedKv3Cache(num_layers=2, num_pages=64, kv_heads=Hkv, mode=mode, seed=4)
    rids = [cache.create_request() for _ in lens]
    data = [(rng.standard_normal((n, Hkv, D)).astype(np.float32),
             rng.standard_normal((n, Hkv, D)).astype(np.float32)) for n in lens]
    fill(cache, 1, rids, data, [1, 31, 40])
    assert [cache.seq_len(r, 1) for r in rids] == lens
    assert all(cache.seq_len(r, 0) == 0 for r in rids)
    signs = cache.signs() if mode == "T" else None
    stores = []
    for r, (k, v) in zip(rids, data):
        kc, km, vc, vm = (t.cpu().numpy()[0] for t in cache.export_range(1, [r], 0, k.shape[0]))
        rk = store_r(k) if mode == "R" else store_t(k, signs)
        rv = store_r(v) if mode == "R" else store_t(v, signs)
        assert (kc == rk[0]).all() and (vc == rv[0]).all()
        assert (km.view(np.uint32) == rk[1].view(np.uint32)).all()
        assert (vm.view(np.uint32) == rv[1].view(np.uint32)).all()
        stores.append((rk, rv))
    # batched range read of the common prefix
    gk, gv = (t.cpu().numpy() for t in cache.get_range(1, rids, 0, 1))
    for i, (rk, rv) in enumerate(stores):
        if mode == "R":
            assert (gk[i].view(np.uint32) == dequant_r(*rk)[:1].view(np.uint32)).all()
        else:
            ref = fo.kvt_load_vector(rk[0][0, :48], rk[1][0, 0], signs)
            assert (gk[i, 0, 0].view(np.uint32) == ref.view(np.uint32)).all()
    # ragged decode of all four requests in one launch
    q = rng.standard_normal((len(rids), Hq, D)).astype(np.float32)
    out = cache.flash_decode(1, rids, to_dev(q)).cpu().numpy().astype(np.float64)
    for i, (rk, rv) in enumerate(stores):
        S = lens[i]
        if mode == "R":
            kd, vd = dequant_r(*rk), dequant_r(*rv)
            ref = fo.flash_decode_3bit(q[i:i + 1], rk[0][None], rk[1][None], rv[0][None],
                                       rv[1][None], 1, S, Hq, Hkv, D).reshape(Hq, D)
        else:
            kd = np.stack([[fo.kvt_load_vector(rk[0][s, h * 48:(h + 1) * 48], rk[1][s, h], signs)
                            for h in range(Hkv)] for s in range(S)])
            vd = np.stack([[fo.kvt_load_vector(rv[0][s, h * 48:(h + 1) * 48], rv[1][s, h], signs)
                            for h in range(Hkv)] for s in range(S)])
            ref = None
        ex = exact_decode(q[i], kd, vd)
        bound = 1.0 + np.abs(ex)
        assert np.max(np.abs(out[i] - ex) / bound) <= 2e-5
        if ref is not None:
            assert np.max(np.abs(out[i] - ref) / bound) <= 2e-5
    cache.ctx.check()
    cache.close()


def test_paged_decode_equals_ring_decode(pg):
    from ferrisres_b200 import kv
    rng = np.random.default_rng(22)
    B, Hkv, Hq, S = 3, 2, 8, 300
    k = rng.standard_normal((B, S, Hkv, D)).astype(np.float32)
    v = rng.standard_normal((B, S, Hkv, D)).astype(np.float32)
    q = rng.standard_normal((B, Hq, D)).astype(np.float32)
    ring = kv.Kv3Cache(B, Hkv, S)
    ring.append(to_dev(k), to_dev(v))
    a = ring.flash_decode(to_dev(q)).cpu().numpy()
    cache = pg.PagedKv3Cache(1, 64, Hkv)
    rids = [cache.create_request() for _ in range(B)]
    cache.append(0, rids, to_dev(k[:, :100]), to_dev(v[:, :100]))
    cache.append(0, rids, to_dev(k[:, 100:]), to_dev(v[:, 100:]))
    b = cache.flash_decode(0, rids, to_dev(q)).cpu().numpy()
    assert (a.view(np.uint32) == b.view(np.uint32)).all()
    # the stored bytes agree too
    got = [t.cpu().numpy() for t in cache.export_range(0, rids, 0, S)]
    ref = [t.cpu().numpy() for t in ring.export_range(0, S)]
    for g, r in zip(got, ref):
        assert (g.view(np.uint8) == r.view(np.uint8)).all()
    ring.close()
    cache.close()


def test_fork_copy_on_write(pg):
    rng = np.random.default_rng(23)
    Hkv = 1
    cache = pg.PagedKv3Cache(1, 16, Hkv)
    a = cache.create_request()
    base = rng.standard_normal((2, 40, Hkv, D)).astype(np.float32)
    cache.append(0, [a], to_dev(base[0][None]), to_dev(base[1][None]))
    b = cache.fork_request(a)
    pages_before = cache.block_table(a)
    alloc = cache.manager.allocator
    assert cache.block_table(b) == pages_before and alloc.ref_count(pages_before[1]) == 2
    ta = rng.standard_normal((2, 30, Hkv, D)).astype(np.float32)
    tb = rng.standard_normal((2, 5, Hkv, D)).astype(np.float32)
    cache.append(0, [b], to_dev(tb[0][None]), to_dev(tb[1][None]))  # copies page 1
    cache.append(0, [a], to_dev(ta[0][None]), to_dev(ta[1][None]))  # page 1 now private
    pa, pb = cache.block_table(a), cache.block_table(b)
    assert pa[0] == pb[0] == pages_before[0] and alloc.ref_count(pa[0]) == 2
    assert pa[1] == pages_before[1] != pb[1]
    for r, tail in ((a, ta), (b, tb)):
        k = np.concatenate([base[0], tail[0]])
        v = np.concatenate([base[1], tail[1]])
        kc, km, vc, vm = (t.cpu().numpy()[0] for t in cache.export_range(0, [r], 0, k.shape[0]))
        rk, rv = store_r(k), store_r(v)
        assert (kc == rk[0]).all() and (vc == rv[0]).all()
        assert (km == rk[1]).all() and (vm == rv[1]).all()
    cache.free_request(a)
    cache.free_request(b)
    assert cache.manager.num_free_blocks() == 16
    cache.close()


def test_bad_tables_and_exhaustion(pg):
    from ferrisres_b200._lib import OOMError, ShapeError, call
    from ferrisres_b200.gpu import _dptr, _stream_ptr
    cache = pg.PagedKv3Cache(1, 4, 1)
    r = cache.create_request()
    x = torch.randn((1, 33, 1, D), device="cuda")
    cache.append(0, [r], x, x)
    with pytest.raises(OOMError):
        cache.append(0, [r], torch.randn((1, 200, 1, D), device="cuda"),
                     torch.randn((1, 200, 1, D), device="cuda"))
    cache.ctx.check()
    # a table naming page 99 of a 4-page pool: skipped on the device, reported
    tables = torch.tensor([[0, 99]], dtype=torch.int32, device="cuda")
    lens = torch.tensor([40], dtype=torch.int32, device="cuda")
    q = torch.randn((1, 1, D), device="cuda")
    out = torch.empty_like(q)
    call("ft_kvp_flash_decode", cache.ctx.handle, cache.handle, 1, _dptr(tables), 2, _dptr(lens),
         40, _dptr(q), 1, C.c_float(0.0), _dptr(out), _stream_ptr())
    with pytest.raises(ShapeError):
        cache.ctx.check()
    start = torch.tensor([32], dtype=torch.int32, device="cuda")
    call("ft_kvp_append", cache.ctx.handle, cache.handle, 1, 1, _dptr(tables), 2, _dptr(start),
         _dptr(x[:, :1]), _dptr(x[:, :1]), 0, _stream_ptr())
    with pytest.raises(ShapeError):
        cache.ctx.check()
    cache.ctx.check()  # the report was cleared
    cache.close()
