"""GPU 3-bit KV cache and flash decode.

``Kv3Cache`` is one layer of the cache for ``batch`` sequences resident in
HBM (the C ABI's ``ft_kv3``): append, get_range, eviction and the split-S
flash decode over it.  ``TurboQuantKVCache`` keeps the reference's type and
call signatures (src/inference/turboquant_kv.rs:173-411: ``new``, ``append``,
``get_range``, ``get``, ``evict_oldest``, ``evict_to``, ``memory_bytes``,
``compression_ratio``, ``seq_len``, ``reset``) with one ``Kv3Cache`` per
layer, for a single sequence, host slices in and out.

The device cache stores exactly the reference's quantisation (group 128 = one
head vector: per-vector min and max, 3-bit codes), so ``export_range`` returns
the reference's stored bytes bit for bit.  Group sizes other than 128 raise
``UnsupportedError``.
"""
from __future__ import annotations

import ctypes as C

import numpy as np
import torch

from ._lib import ShapeError, UnsupportedError, call
from .gpu import _dptr, _stream_ptr, get_context

HEAD_DIM = 128
REC_BYTES = HEAD_DIM * 3 // 8  # 48


class Kv3Cache:
    """One layer's 3-bit KV cache for ``batch`` sequences on one GPU."""

    def __init__(self, batch: int, kv_heads: int, max_seq: int, head_dim: int = HEAD_DIM,
                 device=None, mode: str = "R", seed: int = 0):
        """mode "R": the reference TurboQuantKVCache scheme (min/max per vector);
        mode "T": rotation + uniform 3-bit codebook + per-vector norm (see
        ft_kv3_create_mode), rotation signs drawn from ``seed``."""
        self.ctx = get_context(device)
        self.batch, self.kv_heads = int(batch), int(kv_heads)
        if mode not in ("R", "T"):
            raise ShapeError("mode must be 'R' or 'T'")
        self.mode = mode
        h = C.c_void_p()
        call("ft_kv3_create_mode", self.ctx.handle, self.batch, self.kv_heads, int(head_dim),
             int(max_seq), 0 if mode == "R" else 1, int(seed) & (2**64 - 1), C.byref(h))
        self.handle = h
        self.device = torch.device("cuda", self.ctx.device)

    def signs(self):
        """Mode T: the 128 rotation signs (numpy float32)."""
        import numpy as np
        out = np.empty(HEAD_DIM, np.float32)
        call("ft_kv3_signs", self.handle, out.ctypes.data_as(C.c_void_p))
        return out

    # ---- state
    def __len__(self) -> int:
        n = C.c_int64()
        call("ft_kv3_len", self.handle, C.byref(n))
        return n.value

    @property
    def capacity(self) -> int:
        n = C.c_int64()
        call("ft_kv3_capacity", self.handle, C.byref(n))
        return n.value

    def evict_front(self, n: int = 1) -> None:
        call("ft_kv3_evict_front", self.handle, int(n))

    def reset(self) -> None:
        call("ft_kv3_reset", self.handle)

    # ---- write
    def _kv_view(self, t: torch.Tensor) -> torch.Tensor:
        if t.dtype not in (torch.float32, torch.bfloat16):
            raise ShapeError("K/V must be fp32 or bf16")
        t = t.contiguous()
        if t.numel() % (self.batch * self.kv_heads * HEAD_DIM):
            raise ShapeError("K/V must be [batch, n_pos, kv_heads, 128]")
        return t

    def append(self, k: torch.Tensor, v: torch.Tensor, stream=None) -> None:
        """k, v: [batch, n_pos, kv_heads, 128] (or [batch, n_pos, kv_dim]), fp32 or bf16."""
        k, v = self._kv_view(k), self._kv_view(v)
        if k.shape != v.shape or k.dtype != v.dtype:
            raise ShapeError("K and V must have the same shape and dtype")
        n = k.numel() // (self.batch * self.kv_heads * HEAD_DIM)
        call("ft_kv3_append", self.ctx.handle, self.handle, n, _dptr(k), _dptr(v),
             int(k.dtype == torch.bfloat16), _stream_ptr(stream))

    def append_packed(self, k_codes, k_minmax, v_codes, v_minmax, stream=None) -> None:
        """Positions in the reference's stored form: codes uint8 [batch, n, kv_heads*48],
        (min, max) fp32 [batch, n, kv_heads, 2]."""
        tens = [t.contiguous() for t in (k_codes, k_minmax, v_codes, v_minmax)]
        per = self.batch * self.kv_heads * REC_BYTES
        if tens[0].dtype != torch.uint8 or tens[0].numel() % per:
            raise ShapeError("codes must be uint8 [batch, n, kv_heads*48]")
        n = tens[0].numel() // per
        for t, w in ((tens[1], 2), (tens[3], 2)):
            if t.dtype != torch.float32 or t.numel() != self.batch * n * self.kv_heads * w:
                raise ShapeError("min/max must be fp32 [batch, n, kv_heads, 2]")
        if tens[2].shape != tens[0].shape or tens[2].dtype != torch.uint8:
            raise ShapeError("K and V codes must match")
        call("ft_kv3_append_packed", self.ctx.handle, self.handle, n, _dptr(tens[0]),
             _dptr(tens[1]), _dptr(tens[2]), _dptr(tens[3]), _stream_ptr(stream))

    # ---- read
    def get_range(self, start: int, end: int, stream=None):
        """Dequantised K, V [batch, end-start, kv_heads, 128] fp32 (reference get_range)."""
        n = int(end) - int(start)
        if n < 0:
            raise ShapeError("end < start")
        shape = (self.batch, n, self.kv_heads, HEAD_DIM)
        k = torch.empty(shape, dtype=torch.float32, device=self.device)
        v = torch.empty_like(k)
        call("ft_kv3_get_range", self.ctx.handle, self.handle, int(start), int(end), _dptr(k),
             _dptr(v), _stream_ptr(stream))
        return k, v

    def export_range(self, start: int, end: int, stream=None):
        """Reference stored form of positions [start, end): (k_codes, k_minmax, v_codes,
        v_minmax) with codes uint8 [batch, n, kv_heads*48] and min/max [batch, n, kv_heads, 2]."""
        n = int(end) - int(start)
        if n < 0:
            raise ShapeError("end < start")
        kc = torch.empty((self.batch, n, self.kv_heads * REC_BYTES), dtype=torch.uint8,
                         device=self.device)
        vc = torch.empty_like(kc)
        km = torch.empty((self.batch, n, self.kv_heads, 2), dtype=torch.float32,
                         device=self.device)
        vm = torch.empty_like(km)
        call("ft_kv3_export_range", self.ctx.handle, self.handle, int(start), int(end),
             _dptr(kc), _dptr(km), _dptr(vc), _dptr(vm), _stream_ptr(stream))
        return kc, km, vc, vm

    def flash_decode(self, q: torch.Tensor, scale: float = 0.0, out: torch.Tensor | None = None,
                     stream=None) -> torch.Tensor:
        """q [batch, q_heads, 128] fp32 -> out [batch, q_heads, 128] fp32 over the whole
        cache; scale 0 selects 1/sqrt(128)."""
        if q.dtype != torch.float32 or q.dim() != 3 or q.shape[0] != self.batch or \
                q.shape[2] != HEAD_DIM:
            raise ShapeError("q must be fp32 [batch, q_heads, 128]")
        q = q.contiguous()
        if out is None:
            out = torch.empty_like(q)
        call("ft_flash_decode_3bit", self.ctx.handle, self.handle, _dptr(q), int(q.shape[1]),
             float(scale), _dptr(out), _stream_ptr(stream))
        return out

    def close(self):
        if getattr(self, "handle", None):
            call("ft_kv3_destroy", self.handle)
            self.handle = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass


class TurboQuantKVCache:
    """The reference's ``TurboQuantKVCache`` (turboquant_kv.rs:173-411) for one
    sequence, one ``Kv3Cache`` per layer in HBM."""

    def __init__(self, num_layers: int, kv_dim: int, max_seq_len: int, group_size: int,
                 device=None):
        if group_size != HEAD_DIM or kv_dim % HEAD_DIM or kv_dim <= 0:
            raise UnsupportedError(
                "the device cache quantises one 128-value head vector per group: group_size "
                "must be 128 and kv_dim a multiple of 128")
        self.num_layers = int(num_layers)
        self.kv_dim = int(kv_dim)
        self.group_size = int(group_size)
        self.max_seq_len = int(max_seq_len)
        self.num_groups = (kv_dim + group_size - 1) // group_size
        self.bytes_per_pos = (kv_dim * 3 + 7) // 8
        self.current_len = 0
        self.layers = [Kv3Cache(1, kv_dim // HEAD_DIM, max(1, max_seq_len), device=device)
                       for _ in range(self.num_layers)]
        self.device = self.layers[0].device

    def _vec(self, a) -> torch.Tensor:
        t = a if isinstance(a, torch.Tensor) else torch.from_numpy(
            np.ascontiguousarray(np.asarray(a, dtype=np.float32)))
        if t.numel() != self.kv_dim:
            raise ShapeError(f"expected a vector of kv_dim = {self.kv_dim} values")
        if t.dtype not in (torch.float32, torch.bfloat16):
            t = t.float()
        return t.to(self.device).reshape(1, 1, self.kv_dim)

    def append(self, layer: int, k, v) -> None:
        """append (:240-266): quantise and store one position of ``layer``."""
        self.layers[layer].append(self._vec(k), self._vec(v))
        if layer == self.num_layers - 1:
            self.current_len += 1

    def get_range(self, layer: int, start: int, end: int):
        """get_range (:271-291): (K, V) as flat fp32 host arrays of (end-start)*kv_dim;
        positions past the layer's stored length are zeros."""
        if end < start:
            raise ShapeError("end < start")
        n = end - start
        k = np.zeros(n * self.kv_dim, np.float32)
        v = np.zeros(n * self.kv_dim, np.float32)
        have = min(end, len(self.layers[layer])) - start
        if have > 0:
            kd, vd = self.layers[layer].get_range(start, start + have)
            k[:have * self.kv_dim] = kd.reshape(-1).cpu().numpy()
            v[:have * self.kv_dim] = vd.reshape(-1).cpu().numpy()
        return k, v

    def get(self, layer: int, pos: int):
        """get (:294-305)."""
        return self.get_range(layer, pos, pos + 1)

    def evict_oldest(self) -> None:
        """evict_oldest (:308-320)."""
        for c in self.layers:
            if len(c):
                c.evict_front(1)
        if self.current_len > 0:
            self.current_len -= 1

    def evict_to(self, target_len: int) -> None:
        """evict_to (:323-327)."""
        while self.current_len > target_len:
            self.evict_oldest()

    def memory_bytes(self) -> int:
        """memory_bytes (:330-336): the reference's per-position accounting."""
        per_pos = self.bytes_per_pos * 2 + self.num_groups * 2 * 4 * 2
        return per_pos * self.current_len * self.num_layers

    def compression_ratio(self) -> float:
        """compression_ratio (:338-343)."""
        fp32_per_pos = self.kv_dim * 4 * 2
        denom = self.current_len * self.num_layers
        actual = self.memory_bytes() / denom if denom else float("nan")
        return fp32_per_pos / actual if actual > 0 else 1.0

    def seq_len(self) -> int:
        return self.current_len

    def reset(self) -> None:
        for c in self.layers:
            c.reset()
        self.current_len = 0

    def flash_decode(self, layer: int, q, q_heads: int, scale: float = 0.0) -> np.ndarray:
        """Attention of q [q_heads * 128] over the layer's cache (flash_decode_ref math
        with the GQA head map); host in, host out."""
        qt = q if isinstance(q, torch.Tensor) else torch.from_numpy(
            np.ascontiguousarray(np.asarray(q, dtype=np.float32)))
        qt = qt.float().to(self.device).reshape(1, q_heads, HEAD_DIM)
        return self.layers[layer].flash_decode(qt, scale).reshape(-1).cpu().numpy()

    def close(self):
        for c in self.layers:
            c.close()
