"""GPU mirror of the reference's ternary MoE layer.

``TernaryMoELayer`` keeps the reference's constructor data and ``forward``
(src/model/ternary_moe.rs:77-223): router [E, H] fp32 (row e = expert e),
per expert gate/up [F, H] and down [H, F] ternary matrices, top-k softmax
routing with renormalised gates, SwiGLU (or GeLU-tanh) experts.  The weights
live in HBM; ``forward`` runs the whole layer through libferris_ternary.so.
"""
from __future__ import annotations

import ctypes as C

import numpy as np
import torch

from ._lib import ShapeError, call
from .gpu import _dptr, _host, _stream_ptr, get_context
from .ternary import pack_ternary


class TernaryMoELayer:
    def __init__(self, router, gate_packed, gate_scales, up_packed, up_scales, down_packed,
                 down_scales, hidden, inter, top_k=2, use_gelu=False, device=None):
        """gate/up/down: per-expert reference pack_ternary bytes; *_scales: per-row f32."""
        self.ctx = get_context(device)
        E = len(gate_packed)
        if not (len(up_packed) == len(down_packed) == E == len(gate_scales) == len(up_scales)
                == len(down_scales)):
            raise ShapeError("per-expert lists must have equal lengths")
        r = _host(router, np.float32)
        if r.size != E * hidden:
            raise ShapeError("router must be [n_experts * hidden] fp32")
        keep = [r]

        def arr(lst, dt, n):
            ptrs = []
            for a in lst:
                if a is None:  # expert held by another rank
                    ptrs.append(None)
                    continue
                a = _host(a, dt)
                if a.size < n:
                    raise ShapeError("per-expert buffer too small")
                keep.append(a)
                ptrs.append(a.ctypes.data)
            return (C.c_void_p * E)(*ptrs)

        mb = inter * hidden // 4
        h = C.c_void_p()
        call("ft_moe_create", self.ctx.handle, E, hidden, inter, top_k, int(use_gelu),
             r.ctypes.data_as(C.c_void_p), arr(gate_packed, np.uint8, mb),
             arr(gate_scales, np.float32, inter), arr(up_packed, np.uint8, mb),
             arr(up_scales, np.float32, inter), arr(down_packed, np.uint8, mb),
             arr(down_scales, np.float32, hidden), C.byref(h))
        self.handle = h
        self.n_experts, self.hidden_dim, self.intermediate_dim = E, hidden, inter
        self.top_k, self.use_gelu = top_k, use_gelu

    @classmethod
    def from_ternary(cls, router, gate, gate_scales, up, up_scales, down, down_scales, hidden,
                     inter, top_k=2, use_gelu=False, device=None):
        """Per-expert int8 {-1,0,1} value arrays (reference TernaryWeight::from_ternary)."""
        pk = lambda a: None if a is None else pack_ternary(a)
        return cls(router, [pk(g) for g in gate], gate_scales, [pk(u) for u in up], up_scales,
                   [pk(d) for d in down], down_scales, hidden, inter, top_k, use_gelu, device)

    @classmethod
    def from_fp32(cls, router, gate, up, down, hidden, inter, top_k=2, use_gelu=False,
                  device=None):
        """Experts from fp32 matrices (gate/up [inter, hidden], down [hidden, inter];
        None for experts another rank holds), quantized on the device per matrix as
        TernaryExpert::from_fp32 does (src/model/cpu_moe.rs:33-37) -- the load path of
        src/model/checkpoint.rs:387-400."""
        self = cls.__new__(cls)
        self.ctx = get_context(device)
        E = len(gate)
        if not (len(up) == len(down) == E):
            raise ShapeError("per-expert lists must have equal lengths")
        r = _host(router, np.float32)
        if r.size != E * hidden:
            raise ShapeError("router must be [n_experts * hidden] fp32")
        keep = [r]

        def arr(lst):
            ptrs = []
            for a in lst:
                if a is None:
                    ptrs.append(None)
                    continue
                a = _host(a, np.float32)
                if a.size != hidden * inter:
                    raise ShapeError("expert matrix must hold hidden * inter floats")
                keep.append(a)
                ptrs.append(a.ctypes.data)
            return (C.c_void_p * E)(*ptrs)

        h = C.c_void_p()
        call("ft_moe_create_f32", self.ctx.handle, E, hidden, inter, top_k, int(use_gelu),
             r.ctypes.data_as(C.c_void_p), arr(gate), arr(up), arr(down), C.byref(h))
        self.handle = h
        self.n_experts, self.hidden_dim, self.intermediate_dim = E, hidden, inter
        self.top_k, self.use_gelu = top_k, use_gelu
        return self

    def forward_device(self, x: torch.Tensor, probs: bool = False, stream=None):
        """x [T, H] float32 or bfloat16 CUDA tensor -> y [T, H] float32 (and softmax probs)."""
        if x.dim() != 2 or x.shape[1] != self.hidden_dim:
            raise ShapeError(f"x must be [T, {self.hidden_dim}]")
        if x.dtype not in (torch.float32, torch.bfloat16):
            raise ShapeError("x must be float32 or bfloat16")
        T = x.shape[0]
        y = torch.empty(T, self.hidden_dim, dtype=torch.float32, device=x.device)
        p = torch.empty(T, self.n_experts, dtype=torch.float32, device=x.device) if probs else None
        call("ft_moe_forward", self.ctx.handle, self.handle, T, _dptr(x),
             int(x.dtype == torch.bfloat16), _dptr(y), _dptr(p) if p is not None else None,
             _stream_ptr(stream))
        return (y, p) if probs else y

    def decode_device(self, x: torch.Tensor, probs: bool = False, stream=None):
        """Fused decode step (ft_moe_decode) for 1..8 tokens: x [T, H] float32 or
        bfloat16 CUDA tensor -> (y [T, H] float32, topk_idx [T, K], topk_w [T, K]
        [, probs [T, E]]), one kernel launch, no host synchronisation."""
        if x.dim() != 2 or x.shape[1] != self.hidden_dim:
            raise ShapeError(f"x must be [T, {self.hidden_dim}]")
        if x.dtype not in (torch.float32, torch.bfloat16):
            raise ShapeError("x must be float32 or bfloat16")
        T = x.shape[0]
        y = torch.empty(T, self.hidden_dim, dtype=torch.float32, device=x.device)
        idx = torch.empty(T, self.top_k, dtype=torch.int32, device=x.device)
        w = torch.empty(T, self.top_k, dtype=torch.float32, device=x.device)
        p = torch.empty(T, self.n_experts, dtype=torch.float32, device=x.device) if probs else None
        call("ft_moe_decode", self.ctx.handle, self.handle, T, _dptr(x),
             int(x.dtype == torch.bfloat16), _dptr(y), _dptr(idx), _dptr(w),
             _dptr(p) if p is not None else None, _stream_ptr(stream))
        return (y, idx, w, p) if probs else (y, idx, w)

    def forward(self, input, seq: int):
        """src/model/ternary_moe.rs:145: host fp32 [seq * H] in, host fp32 out."""
        x = _host(input, np.float32)
        if x.size != seq * self.hidden_dim:
            raise ShapeError("input must be [seq * hidden_dim]")
        y = np.empty(seq * self.hidden_dim, np.float32)
        call("ft_moe_forward_host", self.ctx.handle, self.handle, x.ctypes.data_as(C.c_void_p),
             int(seq), y.ctypes.data_as(C.c_void_p))
        return y

    def close(self):
        if getattr(self, "handle", None):
            from ._lib import lib
            lib().ft_moe_destroy(self.handle)
            self.handle = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass
