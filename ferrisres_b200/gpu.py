"""GPU-side mirror of the reference's ternary compute API.

Classes keep the reference names and argument meanings:

* ``TernaryMatMulOp`` -- src/compute/kernels/ternary_matmul.rs:78-225
  (``new`` + ``dispatch`` over raw u32 buffers).
* ``GpuMatmulAccelerator`` -- src/model/gpu_forward.rs:1154-1297
  (``gpu_ternary_matmul`` host slices in, host vector out; ``_vram`` variant).
* ``DeviceTernaryWeight`` -- an uploaded weight (the role of the reference's
  ``GpuVramCache`` entries, src/model/cpu_block_attn_res.rs:3072-3120).

Device buffers are torch CUDA tensors; every call goes through the C ABI of
libferris_ternary.so on the caller's current torch stream.
"""
from __future__ import annotations

import ctypes as C
import threading

import numpy as np
import torch

from . import _lib
from ._lib import ShapeError, call, check, lib

_ctxs: dict[int, "Context"] = {}
_ctx_lock = threading.Lock()


class Context:
    """One CUDA device bound to the library (ft_ctx)."""

    def __init__(self, device: int = 0):
        h = C.c_void_p()
        call("ft_ctx_create", int(device), C.byref(h))
        self.handle = h
        self.device = int(device)

    def check(self):
        """Synchronise and raise CommTimeoutError if a kernel's bounded wait gave up."""
        call("ft_ctx_check", self.handle)

    def close(self):
        if self.handle:
            _lib.lib().ft_ctx_destroy(self.handle)
            self.handle = None


def get_context(device: int | None = None) -> Context:
    if device is None:
        device = torch.cuda.current_device()
    with _ctx_lock:
        c = _ctxs.get(device)
        if c is None:
            c = _ctxs[device] = Context(device)
        return c


def _stream_ptr(stream=None):
    s = stream if stream is not None else torch.cuda.current_stream()
    return C.c_void_p(s.cuda_stream)


def _dptr(t: torch.Tensor):
    if not t.is_cuda:
        raise ShapeError("expected a CUDA tensor")
    if not t.is_contiguous():
        raise ShapeError("expected a contiguous tensor")
    return C.c_void_p(t.data_ptr())


_VRAM = None


def _vram_fn():
    global _VRAM
    if _VRAM is None:
        _VRAM = lib().ft_gpu_ternary_matmul_vram
    return _VRAM


def _host(a, dtype):
    return np.ascontiguousarray(np.asarray(a), dtype=dtype)


def _addr(a):
    """Address of a contiguous numpy array's data (a writable array through
    its buffer, which is cheaper than ``a.ctypes``)."""
    try:
        return C.addressof(C.c_char.from_buffer(a))
    except (TypeError, ValueError, BufferError):
        return a.ctypes.data


class DeviceTernaryWeight:
    """A dense ternary matrix [rows, cols] resident in HBM with per-row scales."""

    def __init__(self, handle, rows: int, cols: int, ctx: Context):
        self.handle = handle
        self.rows, self.cols = int(rows), int(cols)
        self.ctx = ctx

    @classmethod
    def from_packed_u8(cls, packed, rows, cols, row_scales, device=None):
        """Reference pack_ternary byte stream (src/model/ternary.rs:141-163)."""
        ctx = get_context(device)
        p = _host(packed, np.uint8)
        s = _host(row_scales, np.float32)
        if p.size < (rows * cols + 3) // 4 or s.size < rows:
            raise ShapeError("packed/scales too short for the given shape")
        h = C.c_void_p()
        call("ft_weight_upload_packed_u8", ctx.handle, p.ctypes.data_as(C.c_void_p), int(rows),
             int(cols), s.ctypes.data_as(C.c_void_p), C.byref(h))
        return cls(h, rows, cols, ctx)

    @classmethod
    def from_packed_u32(cls, words, rows, cols, row_scales, device=None):
        """pack_ternary_u32 / WGSL layout (src/model/ternary.rs:1317-1328)."""
        ctx = get_context(device)
        w = _host(words, np.uint32)
        s = _host(row_scales, np.float32)
        if w.size < rows * ((cols + 15) // 16) or s.size < rows:
            raise ShapeError("words/scales too short for the given shape")
        h = C.c_void_p()
        call("ft_weight_upload_packed_u32", ctx.handle, w.ctypes.data_as(C.c_void_p), int(rows),
             int(cols), s.ctypes.data_as(C.c_void_p), C.byref(h))
        return cls(h, rows, cols, ctx)

    @classmethod
    def from_sparse_host(cls, patterns, signs, rows, cols, row_scales, device=None):
        """2:4 weights in the reference SparseTernaryMatrix layout
        (src/model/sparse_ternary.rs:52-70); stored at 1.5 bits/weight."""
        ctx = get_context(device)
        ng = rows * cols // 4
        pt, sg = _host(patterns, np.uint8), _host(signs, np.uint8)
        s = _host(row_scales, np.float32)
        if cols % 4 or pt.size < (ng + 1) // 2 or sg.size < (ng + 3) // 4 or s.size < rows:
            raise ShapeError("bad 2:4 sparse buffers for the given shape")
        h = C.c_void_p()
        call("ft_sparse_upload_host", ctx.handle, pt.ctypes.data_as(C.c_void_p),
             sg.ctypes.data_as(C.c_void_p), int(rows), int(cols), s.ctypes.data_as(C.c_void_p),
             C.byref(h))
        return cls(h, rows, cols, ctx)

    @classmethod
    def from_sparse_wgsl(cls, words, rows, cols, row_scales, device=None):
        """2:4 weights in the WGSL SparseTernaryMatMulOp layout
        (src/compute/kernels/sparse_ternary.rs:71-100)."""
        ctx = get_context(device)
        w = _host(words, np.uint32)
        s = _host(row_scales, np.float32)
        if cols % 4 or w.size < rows * ((cols // 4 + 5) // 6) or s.size < rows:
            raise ShapeError("bad 2:4 sparse buffers for the given shape")
        h = C.c_void_p()
        call("ft_sparse_upload_wgsl", ctx.handle, w.ctypes.data_as(C.c_void_p), int(rows),
             int(cols), s.ctypes.data_as(C.c_void_p), C.byref(h))
        return cls(h, rows, cols, ctx)

    @classmethod
    def from_ternary(cls, values, rows, cols, row_scales, device=None):
        from .ternary import pack_ternary
        return cls.from_packed_u8(pack_ternary(values), rows, cols, row_scales, device)

    @classmethod
    def from_sparse_indices(cls, pos, neg, rows, cols, row_scales, device=None):
        """Index-list weights (ternary_sparse_indices, src/model/ternary.rs:681-707):
        per row the columns of +1 (``pos``) and -1 (``neg``).  Stored densely at
        2 bits/weight."""
        from .ternary import index_lists_to_csr
        ctx = get_context(device)
        if len(pos) != rows or len(neg) != rows:
            raise ShapeError("pos/neg need one index list per row")
        po, pi = index_lists_to_csr(pos)
        no, ni = index_lists_to_csr(neg)
        s = _host(row_scales, np.float32)
        if s.size == 1:
            s = np.full(rows, s[0], np.float32)
        if s.size < rows:
            raise ShapeError("row_scales too short")
        pi = pi if pi.size else np.zeros(1, np.int64)
        ni = ni if ni.size else np.zeros(1, np.int64)
        h = C.c_void_p()
        call("ft_weight_upload_index_lists", ctx.handle, int(rows), int(cols),
             po.ctypes.data_as(C.c_void_p), pi.ctypes.data_as(C.c_void_p),
             no.ctypes.data_as(C.c_void_p), ni.ctypes.data_as(C.c_void_p),
             s.ctypes.data_as(C.c_void_p), C.byref(h))
        return cls(h, rows, cols, ctx)

    @classmethod
    def from_fp32(cls, weights, rows, cols, device=None):
        """TernaryExpert::from_fp32 (src/model/cpu_moe.rs:33-37): absmean-quantized on
        the device.  Returns the weight; its scale is ``.alpha``."""
        ctx = get_context(device)
        w = _host(weights, np.float32)
        if w.size != rows * cols:
            raise ShapeError("weights must hold rows * cols floats")
        h = C.c_void_p()
        a = C.c_float()
        call("ft_weight_quantize_f32", ctx.handle, w.ctypes.data_as(C.c_void_p), int(rows),
             int(cols), C.byref(a), C.byref(h))
        out = cls(h, rows, cols, ctx)
        out.alpha = np.float32(a.value)
        return out

    def requantize(self, shadow: torch.Tensor, alpha: float, stream=None):
        """STE re-quantization with a layer-shared alpha (src/training/bit_moe.rs:243-262)
        from a [rows, cols] float32 or bfloat16 CUDA tensor."""
        if shadow.numel() != self.rows * self.cols or shadow.dtype not in (torch.float32,
                                                                          torch.bfloat16):
            raise ShapeError("shadow must be float32/bfloat16 [rows, cols]")
        call("ft_weight_requantize", self.ctx.handle, self.handle, _dptr(shadow),
             int(shadow.dtype == torch.bfloat16), float(alpha), _stream_ptr(stream))

    def export_packed_u8(self) -> np.ndarray:
        """The resident codes as the reference pack_ternary byte stream."""
        out = np.empty((self.rows * self.cols + 3) // 4, np.uint8)
        call("ft_weight_export_packed_u8", self.ctx.handle, self.handle,
             out.ctypes.data_as(C.c_void_p))
        return out

    def matmul_blocked_f32(self, x: torch.Tensor, block_scales: torch.Tensor, block_size: int,
                           out: torch.Tensor | None = None, stream=None):
        """ternary_matmul_blocked (src/model/ternary.rs:541-579): one scale per block of
        ``block_size`` columns, shared by all rows (times the row scale)."""
        if x.dtype != torch.float32 or x.shape[-1] != self.cols:
            raise ShapeError(f"x must be float32 [..., {self.cols}]")
        nb = -(-self.cols // int(block_size))
        if block_scales.dtype != torch.float32 or block_scales.numel() != nb:
            raise ShapeError(f"block_scales must be float32 [{nb}]")
        seq = x.numel() // self.cols
        if out is None:
            out = torch.empty(seq, self.rows, dtype=torch.float32, device=x.device)
        call("ft_ternary_matmul_blocked_f32", self.ctx.handle, self.handle, seq, _dptr(x),
             _dptr(block_scales), int(block_size), _dptr(out), _stream_ptr(stream))
        return out

    def device_bytes(self) -> int:
        b = C.c_int64()
        call("ft_weight_info", self.handle, None, None, C.byref(b))
        return b.value

    def matmul_f32(self, x: torch.Tensor, out: torch.Tensor | None = None, stream=None):
        """y[s, r] = scale[r] * sum_k W[r, k] x[s, k]; x float32 [seq, cols]."""
        if x.dtype != torch.float32 or x.shape[-1] != self.cols:
            raise ShapeError(f"x must be float32 [..., {self.cols}], got {tuple(x.shape)} {x.dtype}")
        seq = x.numel() // self.cols
        if out is None:
            out = torch.empty(seq, self.rows, dtype=torch.float32, device=x.device)
        call("ft_ternary_matmul_f32", self.ctx.handle, self.handle, seq, _dptr(x), _dptr(out),
             _stream_ptr(stream))
        return out

    def matmul_bf16(self, x: torch.Tensor, out: torch.Tensor | None = None, stream=None):
        """Same as matmul_f32 with bf16 activations."""
        if x.dtype != torch.bfloat16 or x.shape[-1] != self.cols:
            raise ShapeError(f"x must be bfloat16 [..., {self.cols}]")
        seq = x.numel() // self.cols
        if out is None:
            out = torch.empty(seq, self.rows, dtype=torch.float32, device=x.device)
        call("ft_ternary_matmul_bf16", self.ctx.handle, self.handle, seq, _dptr(x), _dptr(out),
             _stream_ptr(stream))
        return out

    def matmul_i8(self, q: torch.Tensor, sx: torch.Tensor, out: torch.Tensor | None = None,
                  stream=None):
        """Bit-exact int8-activation path: ((float)acc * sx[s]) * scale[r]."""
        if q.dtype != torch.int8 or q.shape[-1] != self.cols:
            raise ShapeError(f"q must be int8 [..., {self.cols}]")
        seq = q.numel() // self.cols
        if sx.dtype != torch.float32 or sx.numel() != seq:
            raise ShapeError("sx must be float32 [seq]")
        if out is None:
            out = torch.empty(seq, self.rows, dtype=torch.float32, device=q.device)
        call("ft_ternary_matmul_i8", self.ctx.handle, self.handle, seq, _dptr(q), _dptr(sx),
             _dptr(out), _stream_ptr(stream))
        return out

    def close(self):
        if self.handle:
            _lib.lib().ft_weight_destroy(self.handle)
            self.handle = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass


class GroupCall:
    """A prepared grouped call: n weights with the same seq in one launch.

    Pointer arrays are built once, so repeated calls (and CUDA-graph capture)
    cost one C call each."""

    def __init__(self, weights, xs, ys, qs_sx=None):
        n = len(weights)
        if not (1 <= n <= 64) or len(xs) != n or len(ys) != n:
            raise ShapeError("group needs 1..64 weights with matching activations/outputs")
        self.ctx = weights[0].ctx
        self.weights, self.xs, self.ys = list(weights), list(xs), list(ys)
        self.seq = xs[0].numel() // weights[0].cols
        for w, x, y in zip(weights, xs, ys):
            if x.shape[-1] != w.cols or x.numel() // w.cols != self.seq:
                raise ShapeError("all group members need [seq, cols] activations, same seq")
            if y.numel() < self.seq * w.rows:
                raise ShapeError("output too small")
            _dptr(x), _dptr(y)
        self._w = (C.c_void_p * n)(*[w.handle.value for w in weights])
        self._x = (C.c_void_p * n)(*[x.data_ptr() for x in xs])
        self._y = (C.c_void_p * n)(*[y.data_ptr() for y in ys])
        self.n = n
        self.i8 = qs_sx is not None
        if self.i8:
            self._sx = (C.c_void_p * n)(*[sx.data_ptr() for sx in qs_sx])

    def __call__(self, stream=None):
        if self.i8:
            call("ft_ternary_matmul_i8_grouped", self.ctx.handle, self.n, self._w, self.seq,
                 self._x, self._sx, self._y, _stream_ptr(stream))
        else:
            call("ft_ternary_matmul_f32_grouped", self.ctx.handle, self.n, self._w, self.seq,
                 self._x, self._y, _stream_ptr(stream))


def quantize_absmax_i8(x: torch.Tensor, stream=None):
    """Per-token absmax int8 (pinned formula; see include/ferris_ternary.h)."""
    if x.dim() != 2:
        raise ShapeError("x must be [seq, cols]")
    seq, cols = x.shape
    q = torch.empty(seq, cols, dtype=torch.int8, device=x.device)
    sx = torch.empty(seq, dtype=torch.float32, device=x.device)
    ctx = get_context(x.device.index)
    if x.dtype == torch.bfloat16:
        call("ft_quantize_absmax_i8_bf16", ctx.handle, seq, cols, _dptr(x), _dptr(q), _dptr(sx),
             _stream_ptr(stream))
    elif x.dtype == torch.float32:
        call("ft_quantize_absmax_i8_f32", ctx.handle, seq, cols, _dptr(x), _dptr(q), _dptr(sx),
             _stream_ptr(stream))
    else:
        raise ShapeError("x must be float32 or bfloat16")
    return q, sx


class TernaryMatMulOp:
    """src/compute/kernels/ternary_matmul.rs:78-225 on raw device u32 buffers."""

    def __init__(self, device=None):
        self.ctx = get_context(device)

    @classmethod
    def new(cls, device=None):
        return cls(device)

    def dispatch(self, ternary: torch.Tensor, scales: torch.Tensor, input: torch.Tensor,
                 output: torch.Tensor, seq_len: int, in_cols: int, out_rows: int, stream=None):
        cp = (in_cols + 15) // 16
        if ternary.dtype not in (torch.int32, torch.uint32) or ternary.numel() < out_rows * cp:
            raise ShapeError("ternary must hold out_rows*ceil(in_cols/16) u32 words")
        if scales.numel() < out_rows or input.numel() < seq_len * in_cols or \
                output.numel() < seq_len * out_rows:
            raise ShapeError("buffer too small for the given dims")
        call("ft_ternary_matmul_op_dispatch", self.ctx.handle, _dptr(ternary), _dptr(scales),
             _dptr(input), _dptr(output), int(seq_len), int(in_cols), int(out_rows),
             _stream_ptr(stream))


class GpuMatmulAccelerator:
    """src/model/gpu_forward.rs:1154-1297: host slices in, host vector out."""

    def __init__(self, device=None):
        self.ctx = get_context(device)

    def gpu_ternary_matmul(self, packed_weights, scales, input, seq_len, in_cols, out_rows):
        w = _host(packed_weights, np.uint32)
        s = _host(scales, np.float32)
        x = _host(input, np.float32)
        if w.size < out_rows * ((in_cols + 15) // 16) or s.size < out_rows or \
                x.size < seq_len * in_cols:
            raise ShapeError("buffer too small for the given dims")
        y = np.empty(seq_len * out_rows, np.float32)
        call("ft_gpu_ternary_matmul", self.ctx.handle, w.ctypes.data_as(C.c_void_p),
             s.ctypes.data_as(C.c_void_p), x.ctypes.data_as(C.c_void_p), int(seq_len),
             int(in_cols), int(out_rows), y.ctypes.data_as(C.c_void_p))
        return y

    def gpu_sparse_ternary_matmul(self, sparse_data, scale, input, seq_len, in_cols, out_rows):
        """src/model/gpu_forward.rs:1299 (a zero-returning stub in the reference)."""
        w = _host(sparse_data, np.uint32)
        x = _host(input, np.float32)
        if in_cols % 4 or w.size < out_rows * ((in_cols // 4 + 5) // 6) or \
                x.size < seq_len * in_cols:
            raise ShapeError("buffer too small for the given dims")
        y = np.empty(seq_len * out_rows, np.float32)
        call("ft_gpu_sparse_ternary_matmul", self.ctx.handle, w.ctypes.data_as(C.c_void_p),
             float(scale), x.ctypes.data_as(C.c_void_p), int(seq_len), int(in_cols),
             int(out_rows), y.ctypes.data_as(C.c_void_p))
        return y

    def gpu_ternary_matmul_vram(self, weight: DeviceTernaryWeight, input, seq_len, in_cols,
                                out_rows):
        if weight.cols != in_cols or weight.rows != out_rows:
            raise ShapeError("weight shape does not match in_cols/out_rows")
        x = input
        if not (type(x) is np.ndarray and x.dtype == np.float32 and x.flags.c_contiguous):
            x = _host(input, np.float32)
        if x.size < seq_len * in_cols:
            raise ShapeError("input too small")
        y = np.empty(seq_len * out_rows, np.float32)
        check(_vram_fn()(self.ctx.handle, weight.handle, _addr(x), int(seq_len), int(in_cols),
                         int(out_rows), _addr(y)))
        return y


def shadow_alpha(shadows, device=None):
    """BitMoELayer::recompute_alpha (src/training/bit_moe.rs:210-241): mean |v| over
    the given float32/bfloat16 CUDA tensors, summed in f64.  None when they are empty."""
    ctx = get_context(device)
    if not shadows:
        return None
    bf16 = shadows[0].dtype == torch.bfloat16
    if any((t.dtype == torch.bfloat16) != bf16 for t in shadows):
        raise ShapeError("shadows must share one dtype")
    ptrs = (C.c_void_p * len(shadows))(*[t.data_ptr() for t in shadows])
    cnts = (C.c_int64 * len(shadows))(*[t.numel() for t in shadows])
    for t in shadows:
        _dptr(t)
    a = C.c_float(np.nan)
    call("ft_shadow_alpha", ctx.handle, len(shadows), ptrs, cnts, int(bf16), C.byref(a))
    return None if np.isnan(a.value) else np.float32(a.value)


def ternary_matmul_sparse_decode(pos_indices, neg_indices, scale, input, out_rows, device=None):
    """src/model/ternary.rs:647-672 with host slices: index lists in, host vector out
    (the lists are uploaded densely; keep a DeviceTernaryWeight.from_sparse_indices
    weight for repeated decode steps)."""
    x = _host(input, np.float32)
    w = DeviceTernaryWeight.from_sparse_indices(pos_indices, neg_indices, out_rows, x.size,
                                                np.float32(scale), device)
    y = w.matmul_f32(torch.from_numpy(x).to(f"cuda:{w.ctx.device}").view(1, -1))
    out = y.cpu().numpy().ravel()
    w.close()
    return out
