"""`.stm` expert files (sparse ternary matrices) straight into device weights.

Mirror of the reference's expert file format and lazy loader
(src/model/expert_loader.rs:6-152):

    [magic u32 = 0x53544D31 "STM1"][rows u32][cols u32][scale f32]
    [pattern_bytes u32][sign_bytes u32][patterns: u8 * pattern_bytes][signs: u8 * sign_bytes]

little-endian, 24-byte header, then the host SparseTernaryMatrix layout
(src/model/sparse_ternary.rs:52-70: 3-bit pattern index per 4-group, two per
byte; two sign bits per group, four groups per byte, bit set = +1).  The
reference decodes a file into a host SparseTernaryMatrix on first access; here
the pattern and sign bytes go to the device as they are and are repacked there
into the 1.5 bit/weight 2:4 format (`ft_sparse_upload_host`), with the file's
single scale broadcast to every row (the reference's `gpu_packed()` semantics,
src/model/cpu_moe.rs:73-78).
"""
from __future__ import annotations

import mmap
import os
import struct
from dataclasses import dataclass, field

import numpy as np

STM_MAGIC = 0x53544D31
STM_HEADER_SIZE = 24


class StmFormatError(ValueError):
    """Malformed .stm data (the reference's std::io::ErrorKind::InvalidData)."""


@dataclass
class SparseTernaryMatrix:
    """Host 2:4 ternary matrix in the reference layout."""

    patterns: np.ndarray  # uint8
    signs: np.ndarray     # uint8
    scale: float
    rows: int
    cols: int


def _parse(buf, what: str) -> SparseTernaryMatrix:
    """Header checks and field extraction shared by file and mmap readers
    (src/model/expert_loader.rs:62-100 and 107-145)."""
    n = len(buf)
    if n < STM_HEADER_SIZE:
        raise StmFormatError(f"STM {what} too small: {n} bytes")
    magic, rows, cols, scale, pb, sb = struct.unpack_from("<IIIfII", buf, 0)
    if magic != STM_MAGIC:
        raise StmFormatError(f"Invalid STM magic: 0x{magic:08X}")
    expected = STM_HEADER_SIZE + pb + sb
    if n < expected:
        raise StmFormatError(f"STM {what} truncated: expected {expected} bytes, got {n}")
    raw = np.frombuffer(buf, dtype=np.uint8, count=pb + sb, offset=STM_HEADER_SIZE)
    return SparseTernaryMatrix(raw[:pb].copy(), raw[pb:].copy(), float(scale), int(rows),
                               int(cols))


def read_stm(path) -> SparseTernaryMatrix:
    """`read_stm_file` (src/model/expert_loader.rs:61-100)."""
    with open(path, "rb") as f:
        data = f.read()
    return _parse(data, "data")


def read_stm_mmap(m) -> SparseTernaryMatrix:
    """`read_stm_mmap` (src/model/expert_loader.rs:107-145)."""
    return _parse(m, "mmap")


def write_stm(path, mat: SparseTernaryMatrix) -> None:
    """`write_stm_file` (src/model/expert_loader.rs:45-58)."""
    pat = np.ascontiguousarray(mat.patterns, dtype=np.uint8)
    sg = np.ascontiguousarray(mat.signs, dtype=np.uint8)
    with open(path, "wb") as f:
        f.write(struct.pack("<IIIfII", STM_MAGIC, int(mat.rows), int(mat.cols), float(mat.scale),
                            pat.size, sg.size))
        f.write(pat.tobytes())
        f.write(sg.tobytes())


def expected_sizes(rows: int, cols: int):
    """Pattern and sign byte counts of a [rows, cols] 2:4 matrix
    (src/model/sparse_ternary.rs:82-84)."""
    groups = rows * cols // 4
    return (groups + 1) // 2, (groups + 3) // 4


def to_device(mat: SparseTernaryMatrix, device=None):
    """Upload a host 2:4 matrix as a resident sparse weight (one scale per row,
    all equal to the file's scale)."""
    from . import gpu
    pb, sb = expected_sizes(mat.rows, mat.cols)
    if mat.cols % 4 != 0 or mat.patterns.size < pb or mat.signs.size < sb:
        raise StmFormatError(f"2:4 data does not fit a [{mat.rows}, {mat.cols}] matrix")
    scales = np.full(mat.rows, mat.scale, dtype=np.float32)
    return gpu.DeviceTernaryWeight.from_sparse_host(mat.patterns[:pb], mat.signs[:sb], mat.rows,
                                                    mat.cols, scales, device=device)


def upload_stm(path, device=None):
    """A .stm file straight into a resident sparse device weight."""
    return to_device(read_stm(path), device=device)


@dataclass
class LoaderStats:
    """`LoaderStats` (src/model/expert_loader.rs:188-193)."""

    cache_hits: int = 0
    cache_misses: int = 0
    total_loads: int = 0


@dataclass
class ExpertLoader:
    """Memory-mapped expert files, uploaded to the device on first use
    (`ExpertLoader`, src/model/expert_loader.rs:158-330).  Files are named
    `layer_{layer:02}_expert_{e}.stm`; a missing file leaves its slot empty."""

    expert_dir: str
    num_layers: int
    num_experts: int
    hidden_dim: int
    top_k: int
    device: int | None = None
    routers: list = field(default_factory=list)
    stats: LoaderStats = field(default_factory=LoaderStats)

    def __post_init__(self):
        self._maps = []
        self._files = []
        for layer in range(self.num_layers):
            row = []
            for e in range(self.num_experts):
                p = os.path.join(self.expert_dir, f"layer_{layer:02}_expert_{e}.stm")
                if os.path.exists(p):
                    f = open(p, "rb")
                    self._files.append(f)
                    row.append(mmap.mmap(f.fileno(), 0, access=mmap.ACCESS_READ))
                else:
                    row.append(None)
            self._maps.append(row)
        self._cache = {}

    @classmethod
    def open(cls, expert_dir, num_layers, num_experts, hidden_dim, top_k, device=None):
        return cls(str(expert_dir), num_layers, num_experts, hidden_dim, top_k, device)

    def set_routers(self, routers) -> None:
        self.routers = [np.asarray(r, dtype=np.float32) for r in routers]

    def route(self, layer: int, hidden) -> list:
        """Softmax top-k over `router[e * hidden_dim + j]` in the reference's
        order (src/model/expert_loader.rs:260-290): scores, max-shifted exp,
        normalise, stable descending sort."""
        r = self.routers[layer]
        h = np.asarray(hidden, dtype=np.float32)
        scores = np.empty(self.num_experts, np.float32)
        for e in range(self.num_experts):
            s = np.float32(0.0)
            row = r[e * self.hidden_dim:(e + 1) * self.hidden_dim]
            for j in range(self.hidden_dim):
                s = np.float32(s + np.float32(row[j] * h[j]))
            scores[e] = s
        m = scores.max()
        ex = np.exp(scores - m).astype(np.float32)
        tot = np.float32(0.0)
        for v in ex:
            tot = np.float32(tot + v)
        p = (ex / tot).astype(np.float32)
        order = sorted(range(self.num_experts), key=lambda i: -p[i])  # stable
        return order[:min(self.top_k, self.num_experts)]

    def ensure_loaded(self, layer: int, expert: int) -> bool:
        key = (layer, expert)
        if key in self._cache:
            self.stats.cache_hits += 1
            return True
        self.stats.cache_misses += 1
        self.stats.total_loads += 1
        m = self._maps[layer][expert]
        if m is None:
            return False
        self._cache[key] = to_device(read_stm_mmap(m), device=self.device)
        return True

    def ensure_loaded_batch(self, layer: int, experts) -> int:
        return sum(1 for e in experts if self.ensure_loaded(layer, e))

    def cache_hit_rate(self) -> float:
        total = self.stats.cache_hits + self.stats.cache_misses
        return 0.0 if total == 0 else self.stats.cache_hits / total

    def cache_size(self) -> int:
        return len(self._cache)

    def get_expert(self, layer: int, expert: int):
        """The resident device weight of a loaded expert, or None."""
        return self._cache.get((layer, expert))

    def evict(self, layer: int, expert: int) -> None:
        self._cache.pop((layer, expert), None)

    def close(self) -> None:
        self._cache.clear()
        for row in self._maps:
            for m in row:
                if m is not None:
                    m.close()
        for f in self._files:
            f.close()
        self._maps, self._files = [], []
