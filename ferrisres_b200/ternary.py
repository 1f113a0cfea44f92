"""Host-side ternary types and packing, mirroring src/model/ternary.rs.

These produce the exact byte layouts the reference writes (so weights packed
by the reference load unchanged) and are vectorised with numpy.  They run
once per weight at load time; the matmuls themselves run on the GPU through
``ferrisres_b200.gpu``.
"""
from __future__ import annotations

import numpy as np

ABSMEAN_NORM = np.float32(0.7978845608)  # src/model/ternary.rs:15
_ENCODE = {-1: 0b00, 0: 0b01, 1: 0b10}   # src/model/ternary.rs:134
TERNARY_DECODE = np.array([-1, 0, 1, 0], np.int8)  # src/model/ternary.rs:138


def pack_ternary(values) -> np.ndarray:
    """2-bit pack, 4 values per byte, LSB first (src/model/ternary.rs:141-163).

    Out-of-range values are treated as 0, as the reference does."""
    v = np.asarray(values, dtype=np.int8).ravel()
    codes = np.full(v.size, 1, np.uint8)
    codes[v == -1] = 0
    codes[v == 1] = 2
    pad = (-v.size) % 4
    if pad:
        codes = np.concatenate([codes, np.zeros(pad, np.uint8)])  # padding bits stay 0
    c = codes.reshape(-1, 4)
    return (c[:, 0] | (c[:, 1] << 2) | (c[:, 2] << 4) | (c[:, 3] << 6)).astype(np.uint8)


def unpack_ternary(packed, n: int) -> np.ndarray:
    """Inverse of pack_ternary (src/model/ternary.rs:168-179)."""
    p = np.asarray(packed, dtype=np.uint8).ravel()
    codes = np.stack([(p >> s) & 3 for s in (0, 2, 4, 6)], axis=1).ravel()[:n]
    return TERNARY_DECODE[codes]


def pack_ternary_u32(packed_u8, total_values: int) -> np.ndarray:
    """u8 stream -> u32 words of 16 codes, little endian (src/model/ternary.rs:1317-1328)."""
    p = np.asarray(packed_u8, dtype=np.uint8).ravel()
    nw = (total_values + 15) // 16
    buf = np.zeros(nw * 4, np.uint8)
    m = min(p.size, buf.size)
    buf[:m] = p[:m]
    return buf.view("<u4").astype(np.uint32)


def quantize_ternary(weights):
    """Absmean quantizer (src/model/ternary.rs:31-57): returns (int8 values, alpha).

    Accumulation of sum|W| is sequential fp32, as in the reference."""
    w = np.asarray(weights, dtype=np.float32).ravel()
    if w.size == 0:
        return np.zeros(0, np.int8), np.float32(0.0)
    s = np.float32(0.0)
    for a in np.abs(w):  # sequential f32 sum (reference order)
        s = np.float32(s + a)
    alpha = np.float32(np.float32(s / np.float32(w.size)) / ABSMEAN_NORM) if s > 0 else np.float32(1.0)
    inv = np.float32(np.float32(1.0) / alpha)
    scaled = (w * inv).astype(np.float32)
    return np.clip(round_half_away(scaled), -1, 1).astype(np.int8), alpha


def round_half_away(a) -> np.ndarray:
    """f32::round / C roundf: round half away from zero (x - trunc(x) is exact)."""
    a = np.asarray(a, np.float32)
    t = np.trunc(a)
    return t + np.where(np.abs(a - t) >= np.float32(0.5), np.sign(a), np.float32(0)).astype(np.float32)


def dequantize_ternary(values, scale) -> np.ndarray:
    """src/model/ternary.rs:62-64."""
    return np.asarray(values, np.int8).astype(np.float32) * np.float32(scale)


def quantize_ternary_blocked(weights, block_size: int):
    """Block-wise absmean quantizer (src/model/ternary.rs:76-110): flat blocks of
    ``block_size`` elements, one alpha per block.  Returns (int8 values, scales)."""
    w = np.asarray(weights, dtype=np.float32).ravel()
    if w.size == 0:
        return np.zeros(0, np.int8), np.zeros(0, np.float32)
    q = np.zeros(w.size, np.int8)
    scales = []
    for b0 in range(0, w.size, block_size):
        qb, a = quantize_ternary(w[b0:b0 + block_size])
        q[b0:b0 + block_size] = qb
        scales.append(a)
    return q, np.asarray(scales, np.float32)


def dequantize_ternary_blocked(values, scales, block_size: int) -> np.ndarray:
    """src/model/ternary.rs:113-130."""
    v = np.asarray(values, np.int8).astype(np.float32)
    s = np.repeat(np.asarray(scales, np.float32), block_size)[:v.size]
    return (s * v).astype(np.float32)


def ternary_sparse_indices(values, out_rows: int, in_cols: int):
    """src/model/ternary.rs:681-707: per row, the columns holding +1 and -1.
    Returns (pos, neg), two lists of ``out_rows`` int64 arrays in column order."""
    t = np.asarray(values, np.int8).reshape(out_rows, in_cols)
    pos = [np.nonzero(row == 1)[0].astype(np.int64) for row in t]
    neg = [np.nonzero(row == -1)[0].astype(np.int64) for row in t]
    return pos, neg


def index_lists_to_csr(lists):
    """A list of per-row index arrays -> (offsets [rows + 1], concatenated indices)."""
    off = np.zeros(len(lists) + 1, np.int64)
    off[1:] = np.cumsum([len(a) for a in lists])
    idx = np.concatenate([np.asarray(a, np.int64) for a in lists]) if off[-1] else \
        np.zeros(0, np.int64)
    return off, idx
