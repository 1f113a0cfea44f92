"""Loader for libferris_ternary.so (the CUDA sm_100a library) and its C ABI.

There is no fallback: if the shared library is missing or cannot be loaded,
importing the compute entry points raises.  Status codes are mapped onto the
exception hierarchy that mirrors the reference's ``FerrisResError``
(src/error.rs:3-36).
"""
from __future__ import annotations

import ctypes as C
import os
import threading

HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(HERE, "libferris_ternary.so")


class FerrisResError(RuntimeError):
    """Base error (reference: ``FerrisResError``)."""


class ShapeError(FerrisResError):
    """``FerrisResError::Shape``."""


class GpuError(FerrisResError):
    """``FerrisResError::Gpu``."""


class OOMError(FerrisResError):
    """``FerrisResError::OOM``."""


class UnsupportedError(FerrisResError):
    """``FerrisResError::Unsupported``."""


class CommTimeoutError(FerrisResError):
    """A collective or bounded wait timed out."""


class DeviceError(FerrisResError):
    """``FerrisResError::Device``."""


_STATUS = {1: ShapeError, 2: GpuError, 3: OOMError, 4: UnsupportedError, 5: CommTimeoutError,
           6: DeviceError}

_lib = None
_lock = threading.Lock()

_p = C.c_void_p
_i64 = C.c_int64
_u32 = C.c_uint32
_sz = C.c_size_t
_i = C.c_int

# name -> argtypes (all return int status unless listed in _RESTYPE)
SIGNATURES = {
    "ft_version": [],
    "ft_last_error_string": [],
    "ft_launch_counter": [],
    "ft_ctx_create": [_i, _p],
    "ft_ctx_destroy": [_p],
    "ft_ctx_check": [_p],
    "ft_weight_upload_packed_u8": [_p, _p, _i64, _i64, _p, _p],
    "ft_weight_upload_packed_u32": [_p, _p, _i64, _i64, _p, _p],
    "ft_weight_from_device_u32": [_p, _p, _i64, _i64, _p, _p, _p],
    "ft_weight_destroy": [_p],
    "ft_weight_export_packed_u8": [_p, _p, _p],
    "ft_sparse_upload_host": [_p, _p, _p, _i64, _i64, _p, _p],
    "ft_sparse_upload_wgsl": [_p, _p, _i64, _i64, _p, _p],
    "ft_gpu_sparse_ternary_matmul": [_p, _p, C.c_float, _p, _sz, _sz, _sz, _p],
    "ft_weight_info": [_p, _p, _p, _p],
    "ft_ternary_matmul_f32": [_p, _p, _i64, _p, _p, _p],
    "ft_ternary_matmul_bf16": [_p, _p, _i64, _p, _p, _p],
    "ft_ternary_matmul_f32_grouped": [_p, _i, _p, _i64, _p, _p, _p],
    "ft_ternary_matmul_i8_grouped": [_p, _i, _p, _i64, _p, _p, _p, _p],
    "ft_ternary_matmul_f32_noalloc": [_p, _p, _i64, _p, _p, _p],
    "ft_ternary_matmul_blocked_f32": [_p, _p, _i64, _p, _p, _i64, _p, _p],
    "ft_weight_upload_index_lists": [_p, _i64, _i64, _p, _p, _p, _p, _p, _p],
    "ft_weight_quantize_f32": [_p, _p, _i64, _i64, _p, _p],
    "ft_weight_requantize": [_p, _p, _p, _i, C.c_float, _p],
    "ft_shadow_alpha": [_p, _i, _p, _p, _i, _p],
    "ft_moe_create_f32": [_p, _i64, _i64, _i64, _i, _i, _p, _p, _p, _p, _p],
    "ft_quantize_absmax_i8_f32": [_p, _i64, _i64, _p, _p, _p, _p],
    "ft_quantize_absmax_i8_bf16": [_p, _i64, _i64, _p, _p, _p, _p],
    "ft_ternary_matmul_i8": [_p, _p, _i64, _p, _p, _p, _p],
    "ft_ternary_matmul_op_dispatch": [_p, _p, _p, _p, _p, _u32, _u32, _u32, _p],
    "ft_gpu_ternary_matmul": [_p, _p, _p, _p, _sz, _sz, _sz, _p],
    "ft_gpu_ternary_matmul_vram": [_p, _p, _p, _sz, _sz, _sz, _p],
    "ft_moe_create": [_p, _i64, _i64, _i64, _i, _i, _p, _p, _p, _p, _p, _p, _p, _p],
    "ft_moe_destroy": [_p],
    "ft_moe_forward": [_p, _p, _i64, _p, _i, _p, _p, _p],
    "ft_moe_forward_host": [_p, _p, _p, _sz, _p],
    "ft_moe_decode": [_p, _p, _i64, _p, _i, _p, _p, _p, _p, _p],
    "ft_moe_route": [_p, _p, _i64, _p, _i, _p, _p, _p, _p, _p],
    "ft_moe_dispatch_layout": [_p, _p, _i64, _p, _p, _p, _p, _p, _p, _p],
    "ft_moe_gather_rows": [_p, _p, _i, _i64, _p, _i64, _p, _p],
    "ft_moe_expert_ffn": [_p, _p, _i, _p, _p, _p, _i, _p, _p],
    "ft_moe_combine": [_p, _p, _i64, _p, _p, _p, _p, _p],
    "ft_kv3_create": [_p, _i64, _i64, _i64, _i64, _p],
    "ft_kv3_create_mode": [_p, _i64, _i64, _i64, _i64, _i, C.c_uint64, _p],
    "ft_kv3_signs": [_p, _p],
    "ft_kv3_destroy": [_p],
    "ft_kv3_append": [_p, _p, _i64, _p, _p, _i, _p],
    "ft_kv3_append_packed": [_p, _p, _i64, _p, _p, _p, _p, _p],
    "ft_kv3_len": [_p, _p],
    "ft_kv3_capacity": [_p, _p],
    "ft_kv3_evict_front": [_p, _i64],
    "ft_kv3_reset": [_p],
    "ft_kv3_get_range": [_p, _p, _i64, _i64, _p, _p, _p],
    "ft_kv3_export_range": [_p, _p, _i64, _i64, _p, _p, _p, _p, _p],
    "ft_flash_decode_3bit": [_p, _p, _p, _i64, C.c_float, _p, _p],
    "ft_kvp_create": [_p, _i64, _i64, _i64, _i64, _i, C.c_uint64, _p],
    "ft_kvp_destroy": [_p],
    "ft_kvp_signs": [_p, _p],
    "ft_kvp_append": [_p, _p, _i64, _i64, _p, _i64, _p, _p, _p, _i, _p],
    "ft_kvp_append_packed": [_p, _p, _i64, _i64, _p, _i64, _p, _p, _p, _p, _p, _p],
    "ft_kvp_copy_pages": [_p, _p, _i64, _p, _p, _p],
    "ft_kvp_get_range": [_p, _p, _i64, _p, _i64, _i64, _i64, _p, _p, _p],
    "ft_kvp_export_range": [_p, _p, _i64, _p, _i64, _i64, _i64, _p, _p, _p, _p, _p],
    "ft_kvp_flash_decode": [_p, _p, _i64, _p, _i64, _p, _i64, _p, _i64, C.c_float, _p, _p],
}
_RESTYPE = {"ft_version": C.c_char_p, "ft_last_error_string": C.c_char_p,
            "ft_launch_counter": C.c_uint64}


def lib():
    """Load the library once; raise ImportError if it is not built."""
    global _lib
    if _lib is not None:
        return _lib
    with _lock:
        if _lib is None:
            if not os.path.exists(LIB_PATH):
                raise ImportError(
                    f"{LIB_PATH} is missing: build it with `python -m ferrisres_b200.build` "
                    "(there is no CPU fallback)")
            L = C.CDLL(LIB_PATH)
            for name, args in SIGNATURES.items():
                f = getattr(L, name)
                f.argtypes = args
                f.restype = _RESTYPE.get(name, C.c_int)
            _lib = L
    return _lib


def check(status: int) -> None:
    if status != 0:
        msg = lib().ft_last_error_string().decode(errors="replace")
        raise _STATUS.get(status, FerrisResError)(msg)


def call(name: str, *args) -> None:
    check(getattr(lib(), name)(*args))
