"""ctypes bindings for the CPU oracle (``libferris_oracle.so``).

TEST INFRASTRUCTURE ONLY.  The oracle restates the reference crate's CPU
functions (shift/FerrisRes v0.2.3, Rust) in C; each C function cites the
reference file:line it follows.  It is the checker for the CUDA path and the
CPU baseline that ``bench.py`` times.  Only ``tests/``, ``__graft_entry__.smoke``
and ``bench.py``'s CPU-baseline leg may import this module; the product path in
``ferrisres_b200`` never does.

The reference cannot be built here (Rust, no toolchain), so the restatement is
pinned against the reference's own unit-test known answers
(tests/test_oracle_kats.py).
"""
from __future__ import annotations

import ctypes as C
import os
import subprocess

import numpy as np

_HERE = os.path.dirname(os.path.abspath(__file__))
_SO = os.path.join(_HERE, "libferris_oracle.so")
_lib = None


def build() -> str:
    """Compile the oracle with its Makefile (no-op when up to date)."""
    subprocess.run(["make", "-s", "-C", _HERE], check=True)
    return _SO


def lib():
    global _lib
    if _lib is None:
        if not os.path.exists(_SO):
            build()
        _lib = C.CDLL(_SO)
        _declare(_lib)
    return _lib


_p = C.c_void_p
_sz = C.c_size_t


def _declare(L):
    sig = {
        "fo_pack_ternary": (None, [_p, _sz, _p]),
        "fo_unpack_ternary": (None, [_p, _sz, _p]),
        "fo_pack_ternary_u32": (None, [_p, _sz, _sz, _p]),
        "fo_pack_ternary_rows_u32": (None, [_p, _sz, _sz, _p]),
        "fo_quantize_ternary": (C.c_float, [_p, _sz, _p]),
        "fo_ternary_matmul": (None, [_p, C.c_float, _p, _sz, _sz, _sz, _p]),
        "fo_ternary_matmul_packed": (None, [_p, C.c_float, _p, _sz, _sz, _sz, _p]),
        "fo_ternary_matmul_decode": (None, [_p, C.c_float, _p, _sz, _sz, _p]),
        "fo_ternary_matmul_blocked": (None, [_p, _p, _sz, _p, _sz, _sz, _sz, _p]),
        "fo_quantize_ternary_blocked": (None, [_p, _sz, _sz, _p, _p]),
        "fo_ternary_sparse_indices": (None, [_p, _sz, _sz, _p, _p, _p, _p]),
        "fo_ternary_matmul_sparse_decode": (None, [_p, _p, _p, _p, C.c_float, _p, _sz, _p]),
        "fo_bitmoe_requantize": (None, [_p, _sz, C.c_float, _p]),
        "fo_bitmoe_recompute_alpha": (C.c_int, [_p, _p, _sz, _p]),
        "fo_kvt_quantize": (None, [_p, _p, _p, _p]),
        "fo_kvt_mm_const": (C.c_float, []),
        "fo_kvt_rotate": (None, [_p, _p, C.c_int, _p]),
        "fo_ternary_matmul_packed_parallel_rows": (None, [_p, _p, _p, _sz, _sz, _p, C.c_int]),
        "fo_gpu_ternary_mm_cpu": (None, [_p, _p, _p, _sz, _sz, _sz, _p]),
        "fo_ternary_matmul_parallel": (None, [_p, C.c_float, _p, _sz, _sz, _sz, _p, C.c_int]),
        "fo_quantize_absmax_i8": (None, [_p, _sz, _sz, _p, _p]),
        "fo_ternary_matmul_i8": (None, [_p, _p, _p, _p, _sz, _sz, _sz, _p, C.c_int]),
        "fo_ternary_matmul_i8_via_f32": (None, [_p, _p, _p, _p, _sz, _sz, _sz, _p, C.c_int]),
        "fo_sparse_from_ternary": (None, [_p, _sz, _sz, _p, _p]),
        "fo_sparse_to_ternary": (None, [_p, _p, _sz, _sz, _p]),
        "fo_sparse_ternary_matmul": (None, [_p, _p, C.c_float, _p, _sz, _sz, _p, _sz, _p, C.c_int]),
        "fo_sparse_wgsl_words_per_row": (_sz, [_sz]),
        "fo_sparse_wgsl_pack": (C.c_int, [_p, _sz, _sz, _p]),
        "fo_sparse_wgsl_ref": (None, [_p, _p, _p, _sz, _sz, _sz, _p]),
        "fo_moe_forward": (None, [_p, _p, _p, _p, _p, _p, _p, _sz, _sz, _sz, _sz, C.c_int, _p,
                                  _sz, _p, _p, _p, C.c_int]),
        "fo_pack_3bit": (None, [_p, _sz, _p]),
        "fo_unpack_3bit": (None, [_p, _sz, _p]),
        "fo_quantize_3bit": (None, [_p, _sz, _p, _p, _p]),
        "fo_dequantize_3bit": (None, [_p, _sz, C.c_float, C.c_float, _p]),
        "fo_kv_quantize_vector": (None, [_p, _sz, _sz, _p, _p]),
        "fo_kv_dequantize_vector": (None, [_p, _p, _sz, _sz, _p]),
        "fo_flash_decode_gqa": (None, [_p, _p, _p, _sz, _sz, _sz, _sz, _sz, _p, C.c_int]),
        "fo_flash_decode_3bit": (None, [_p, _p, _p, _p, _p, _sz, _sz, _sz, _sz, _sz, _p, C.c_int]),
        "fo_num_threads": (C.c_int, [C.c_int]),
    }
    for name, (res, args) in sig.items():
        f = getattr(L, name)
        f.restype = res
        f.argtypes = args


def _c(a: np.ndarray, dtype) -> np.ndarray:
    return np.ascontiguousarray(a, dtype=dtype)


def _ptr(a: np.ndarray):
    return a.ctypes.data_as(C.c_void_p)


# ---------------------------------------------------------------- codes ----
def pack_ternary(values) -> np.ndarray:
    v = _c(values, np.int8)
    out = np.zeros((v.size + 3) // 4, np.uint8)
    lib().fo_pack_ternary(_ptr(v), v.size, _ptr(out))
    return out


def unpack_ternary(packed, n: int) -> np.ndarray:
    p = _c(packed, np.uint8)
    out = np.zeros(n, np.int8)
    lib().fo_unpack_ternary(_ptr(p), n, _ptr(out))
    return out


def pack_ternary_u32(packed_u8, total_values: int) -> np.ndarray:
    p = _c(packed_u8, np.uint8)
    out = np.zeros((total_values + 15) // 16, np.uint32)
    lib().fo_pack_ternary_u32(_ptr(p), p.size, total_values, _ptr(out))
    return out


def pack_ternary_rows_u32(values, rows: int, cols: int) -> np.ndarray:
    v = _c(values, np.int8)
    out = np.zeros(rows * ((cols + 15) // 16), np.uint32)
    lib().fo_pack_ternary_rows_u32(_ptr(v), rows, cols, _ptr(out))
    return out


def quantize_ternary(w):
    w = _c(w, np.float32)
    q = np.zeros(w.size, np.int8)
    a = lib().fo_quantize_ternary(_ptr(w), w.size, _ptr(q))
    return q, np.float32(a)


# --------------------------------------------------------------- matmul ----
def ternary_matmul(t, scale, x, out_rows, in_cols, seq):
    t, x = _c(t, np.int8), _c(x, np.float32)
    y = np.zeros(seq * out_rows, np.float32)
    lib().fo_ternary_matmul(_ptr(t), float(scale), _ptr(x), out_rows, in_cols, seq, _ptr(y))
    return y


def ternary_matmul_packed(packed, scale, x, out_rows, in_cols, seq):
    p, x = _c(packed, np.uint8), _c(x, np.float32)
    y = np.zeros(seq * out_rows, np.float32)
    lib().fo_ternary_matmul_packed(_ptr(p), float(scale), _ptr(x), out_rows, in_cols, seq, _ptr(y))
    return y


def ternary_matmul_decode(t, scale, x, out_rows, in_cols):
    t, x = _c(t, np.int8), _c(x, np.float32)
    y = np.zeros(out_rows, np.float32)
    lib().fo_ternary_matmul_decode(_ptr(t), float(scale), _ptr(x), out_rows, in_cols, _ptr(y))
    return y


def ternary_matmul_blocked(t, scales, block_size, x, out_rows, in_cols, seq):
    """src/model/ternary.rs:541-579."""
    t, sc, x = _c(t, np.int8), _c(scales, np.float32), _c(x, np.float32)
    y = np.zeros(seq * out_rows, np.float32)
    lib().fo_ternary_matmul_blocked(_ptr(t), _ptr(sc), block_size, _ptr(x), out_rows, in_cols,
                                    seq, _ptr(y))
    return y


def quantize_ternary_blocked(w, block_size):
    """src/model/ternary.rs:76-110: (int8 values, per-block scales)."""
    w = _c(w, np.float32)
    q = np.zeros(w.size, np.int8)
    sc = np.zeros((w.size + block_size - 1) // block_size, np.float32)
    if w.size:
        lib().fo_quantize_ternary_blocked(_ptr(w), w.size, block_size, _ptr(q), _ptr(sc))
    return q, sc


def ternary_sparse_indices(t, out_rows, in_cols):
    """src/model/ternary.rs:681-707 as CSR: (pos_off, pos_idx, neg_off, neg_idx)."""
    t = _c(t, np.int8)
    po, no = np.zeros(out_rows + 1, np.int64), np.zeros(out_rows + 1, np.int64)
    pi, ni = np.zeros(max(1, t.size), np.int64), np.zeros(max(1, t.size), np.int64)
    lib().fo_ternary_sparse_indices(_ptr(t), out_rows, in_cols, _ptr(po), _ptr(pi), _ptr(no),
                                    _ptr(ni))
    return po, pi[:po[-1]].copy(), no, ni[:no[-1]].copy()


def ternary_matmul_sparse_decode(pos_off, pos_idx, neg_off, neg_idx, scale, x, out_rows):
    """src/model/ternary.rs:647-672."""
    po, no = _c(pos_off, np.int64), _c(neg_off, np.int64)
    pi = _c(pos_idx if len(pos_idx) else np.zeros(1, np.int64), np.int64)
    ni = _c(neg_idx if len(neg_idx) else np.zeros(1, np.int64), np.int64)
    x = _c(x, np.float32)
    y = np.zeros(out_rows, np.float32)
    lib().fo_ternary_matmul_sparse_decode(_ptr(po), _ptr(pi), _ptr(no), _ptr(ni), float(scale),
                                          _ptr(x), out_rows, _ptr(y))
    return y


def bitmoe_requantize(shadow_bf16_bits, alpha):
    """src/training/bit_moe.rs:243-262 on bf16 bit patterns (uint16)."""
    sh = _c(shadow_bf16_bits, np.uint16)
    q = np.zeros(sh.size, np.int8)
    lib().fo_bitmoe_requantize(_ptr(sh), sh.size, float(alpha), _ptr(q))
    return q


def bitmoe_recompute_alpha(shadows_bf16_bits):
    """src/training/bit_moe.rs:210-241; None when there is no element."""
    arrs = [_c(a, np.uint16) for a in shadows_bf16_bits]
    ptrs = (C.c_void_p * max(1, len(arrs)))(*[a.ctypes.data for a in arrs])
    cnt = (C.c_size_t * max(1, len(arrs)))(*[a.size for a in arrs])
    out = C.c_float(0.0)
    ok = lib().fo_bitmoe_recompute_alpha(ptrs, cnt, len(arrs), C.byref(out))
    return np.float32(out.value) if ok else None


def ternary_matmul_packed_parallel_rows(packed, row_scales, x, out_rows, in_cols, nthreads=0):
    p, s, x = _c(packed, np.uint8), _c(row_scales, np.float32), _c(x, np.float32)
    y = np.zeros(out_rows, np.float32)
    lib().fo_ternary_matmul_packed_parallel_rows(_ptr(p), _ptr(s), _ptr(x), out_rows, in_cols,
                                                 _ptr(y), nthreads)
    return y


def gpu_ternary_mm_cpu(packed_u32, scales, x, seq, in_cols, out_rows):
    p, s, x = _c(packed_u32, np.uint32), _c(scales, np.float32), _c(x, np.float32)
    y = np.zeros(seq * out_rows, np.float32)
    lib().fo_gpu_ternary_mm_cpu(_ptr(p), _ptr(s), _ptr(x), seq, in_cols, out_rows, _ptr(y))
    return y


def ternary_matmul_parallel(t, scale, x, out_rows, in_cols, seq, nthreads=0):
    t, x = _c(t, np.int8), _c(x, np.float32)
    y = np.zeros(seq * out_rows, np.float32)
    lib().fo_ternary_matmul_parallel(_ptr(t), float(scale), _ptr(x), out_rows, in_cols, seq,
                                     _ptr(y), nthreads)
    return y


def quantize_absmax_i8(x, seq, cols):
    x = _c(x, np.float32)
    q = np.zeros(seq * cols, np.int8)
    sx = np.zeros(seq, np.float32)
    lib().fo_quantize_absmax_i8(_ptr(x), seq, cols, _ptr(q), _ptr(sx))
    return q, sx


def ternary_matmul_i8(t, q, sx, sw, seq, in_cols, out_rows, nthreads=0, via_f32=False):
    t, q = _c(t, np.int8), _c(q, np.int8)
    sx, sw = _c(sx, np.float32), _c(sw, np.float32)
    y = np.zeros(seq * out_rows, np.float32)
    f = lib().fo_ternary_matmul_i8_via_f32 if via_f32 else lib().fo_ternary_matmul_i8
    f(_ptr(t), _ptr(q), _ptr(sx), _ptr(sw), seq, in_cols, out_rows, _ptr(y), nthreads)
    return y


# --------------------------------------------------------------- sparse ----
def sparse_from_ternary(t, rows, cols):
    t = _c(t, np.int8)
    ng = rows * cols // 4
    pat = np.zeros((ng + 1) // 2, np.uint8)
    sg = np.zeros((ng + 3) // 4, np.uint8)
    lib().fo_sparse_from_ternary(_ptr(t), rows, cols, _ptr(pat), _ptr(sg))
    return pat, sg


def sparse_to_ternary(pat, sg, rows, cols):
    pat, sg = _c(pat, np.uint8), _c(sg, np.uint8)
    t = np.zeros(rows * cols, np.int8)
    lib().fo_sparse_to_ternary(_ptr(pat), _ptr(sg), rows, cols, _ptr(t))
    return t


def sparse_ternary_matmul(pat, sg, scale, row_scales, rows, cols, x, seq, nthreads=0):
    pat, sg, x = _c(pat, np.uint8), _c(sg, np.uint8), _c(x, np.float32)
    rs = None if row_scales is None else _c(row_scales, np.float32)
    y = np.zeros(seq * rows, np.float32)
    lib().fo_sparse_ternary_matmul(_ptr(pat), _ptr(sg), float(scale),
                                   None if rs is None else _ptr(rs), rows, cols, _ptr(x), seq,
                                   _ptr(y), nthreads)
    return y


def sparse_wgsl_pack(t, rows, cols):
    t = _c(t, np.int8)
    wpr = lib().fo_sparse_wgsl_words_per_row(cols)
    out = np.zeros(rows * wpr, np.uint32)
    rc = lib().fo_sparse_wgsl_pack(_ptr(t), rows, cols, _ptr(out))
    if rc != 0:
        raise ValueError("each group of 4 must hold exactly 2 nonzeros")
    return out


def sparse_wgsl_ref(packed, scales, x, seq, cols, rows):
    p, s, x = _c(packed, np.uint32), _c(scales, np.float32), _c(x, np.float32)
    y = np.zeros(seq * rows, np.float32)
    lib().fo_sparse_wgsl_ref(_ptr(p), _ptr(s), _ptr(x), seq, cols, rows, _ptr(y))
    return y


# ------------------------------------------------------------------ MoE ----
def moe_forward(router, gate, gate_s, up, up_s, down, down_s, hidden, inter, top_k, x, seq,
                use_gelu=False, nthreads=0):
    """router [E*H] f32; gate/up/down: lists of int8 arrays; *_s: lists of f32 row scales."""
    E = len(gate)
    router = _c(router, np.float32)
    keep = []

    def arr_of_ptrs(lst, dt):
        arrs = [_c(a, dt) for a in lst]
        keep.extend(arrs)
        return (C.c_void_p * len(arrs))(*[a.ctypes.data for a in arrs])

    pg, pgs = arr_of_ptrs(gate, np.int8), arr_of_ptrs(gate_s, np.float32)
    pu, pus = arr_of_ptrs(up, np.int8), arr_of_ptrs(up_s, np.float32)
    pd, pds = arr_of_ptrs(down, np.int8), arr_of_ptrs(down_s, np.float32)
    x = _c(x, np.float32)
    y = np.zeros(seq * hidden, np.float32)
    route = np.zeros(seq * top_k, np.int32)
    probs = np.zeros(seq * E, np.float32)
    lib().fo_moe_forward(_ptr(router), pg, pgs, pu, pus, pd, pds, hidden, inter, E, top_k,
                         int(use_gelu), _ptr(x), seq, _ptr(y), _ptr(route), _ptr(probs), nthreads)
    return y, route, probs


# ------------------------------------------------------------ 3-bit KV ----
def pack_3bit(codes):
    c = _c(codes, np.uint8)
    out = np.zeros(3 * ((c.size + 7) // 8), np.uint8)
    lib().fo_pack_3bit(_ptr(c), c.size, _ptr(out))
    return out


def unpack_3bit(packed, n):
    p = _c(packed, np.uint8)
    out = np.zeros(n, np.uint8)
    lib().fo_unpack_3bit(_ptr(p), n, _ptr(out))
    return out


def quantize_3bit(v):
    v = _c(v, np.float32)
    codes = np.zeros(v.size, np.uint8)
    mn, mx = C.c_float(), C.c_float()
    lib().fo_quantize_3bit(_ptr(v), v.size, _ptr(codes), C.byref(mn), C.byref(mx))
    return codes, np.float32(mn.value), np.float32(mx.value)


def dequantize_3bit(codes, mn, mx):
    c = _c(codes, np.uint8)
    out = np.zeros(c.size, np.float32)
    lib().fo_dequantize_3bit(_ptr(c), c.size, float(mn), float(mx), _ptr(out))
    return out


def kv_quantize_vector(v, group):
    v = _c(v, np.float32)
    ng = (v.size + group - 1) // group
    packed = np.zeros(3 * ((v.size + 7) // 8), np.uint8)
    mm = np.zeros(2 * ng, np.float32)
    lib().fo_kv_quantize_vector(_ptr(v), v.size, group, _ptr(packed), _ptr(mm))
    return packed, mm


def kv_dequantize_vector(packed, minmax, kv_dim, group):
    p, mm = _c(packed, np.uint8), _c(minmax, np.float32)
    out = np.zeros(kv_dim, np.float32)
    lib().fo_kv_dequantize_vector(_ptr(p), _ptr(mm), kv_dim, group, _ptr(out))
    return out


def flash_decode_gqa(q, k, v, batch, seq, hq, hkv, d, nthreads=0):
    q, k, v = _c(q, np.float32), _c(k, np.float32), _c(v, np.float32)
    out = np.zeros(batch * hq * d, np.float32)
    lib().fo_flash_decode_gqa(_ptr(q), _ptr(k), _ptr(v), batch, seq, hq, hkv, d, _ptr(out), nthreads)
    return out


def flash_decode_3bit(q, kc, kmm, vc, vmm, batch, seq, hq, hkv, d, nthreads=0):
    q = _c(q, np.float32)
    kc, vc = _c(kc, np.uint8), _c(vc, np.uint8)
    kmm, vmm = _c(kmm, np.float32), _c(vmm, np.float32)
    out = np.zeros(batch * hq * d, np.float32)
    lib().fo_flash_decode_3bit(_ptr(q), _ptr(kc), _ptr(kmm), _ptr(vc), _ptr(vmm), batch, seq, hq,
                               hkv, d, _ptr(out), nthreads)
    return out


def num_threads(requested=0):
    return lib().fo_num_threads(requested)


# --------------------------------------------- 3-bit KV mode T (own spec) --
def kvt_quantize(v, signs):
    """One 128-vector -> (codes uint8[128], norm) under mode T (ferris_oracle.c)."""
    v, sg = _c(v, np.float32), _c(signs, np.float32)
    codes = np.zeros(128, np.uint8)
    n = C.c_float()
    lib().fo_kvt_quantize(_ptr(v), _ptr(sg), _ptr(codes), C.byref(n))
    return codes, np.float32(n.value)


def kvt_signs(seed):
    """The 128 mode-T rotation signs: SplitMix64 draws from ``seed``, -1 where
    bit 63 of the draw is set (the published SplitMix64 of Steele, Lea and
    Flood, OOPSLA 2014)."""
    m = (1 << 64) - 1
    z, out = int(seed) & m, np.empty(128, np.float32)
    for i in range(128):
        z = (z + 0x9E3779B97F4A7C15) & m
        r = ((z ^ (z >> 30)) * 0xBF58476D1CE4E5B9) & m
        r = ((r ^ (r >> 27)) * 0x94D049BB133111EB) & m
        r ^= r >> 31
        out[i] = -1.0 if r >> 63 else 1.0
    return out


def kvt_store_vector(v, signs):
    """One 128-vector in mode T's stored form: (48 packed code bytes,
    (min, max) = -/+ norm * kvt_mm_const())."""
    codes, norm = kvt_quantize(v, signs)
    mx = np.float32(kvt_mm_const() * norm)
    return pack_3bit(codes), np.array([-mx, mx], np.float32)


def kvt_load_vector(packed, minmax, signs):
    """The stored form back in the original domain: the affine dequantisation
    of the rotated codes, then the inverse rotation."""
    return kvt_rotate(dequantize_3bit(unpack_3bit(packed, 128), minmax[0], minmax[1]), signs,
                      inverse=True)


def kvt_mm_const():
    return np.float32(lib().fo_kvt_mm_const())


def kvt_rotate(x, signs, inverse=False):
    x, sg = _c(x, np.float32), _c(signs, np.float32)
    out = np.zeros(128, np.float32)
    lib().fo_kvt_rotate(_ptr(x), _ptr(sg), int(inverse), _ptr(out))
    return out
