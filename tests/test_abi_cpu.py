"""CPU-only checks of the boundary: the CUDA library loads and exports every
symbol that include/*.h declares; the host-side packing mirrors agree with
the oracle; error paths behave without a GPU (no compute calls)."""
import ctypes as C
import glob
import os
import re

import numpy as np
import pytest

from ferrisres_b200 import _lib, ternary
from oracle import oracle as fo

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def declared_symbols():
    names = set()
    for h in glob.glob(os.path.join(ROOT, "include", "*.h")):
        src = open(h).read()
        src = re.sub(r"/\*.*?\*/", "", src, flags=re.S)
        names |= set(re.findall(r"\b(ft_[a-z0-9_]+)\s*\(", src))
    return names


def test_library_loads_and_exports_every_declared_symbol():
    L = _lib.lib()
    declared = declared_symbols()
    assert declared, "no declarations found in include/*.h"
    missing = [n for n in sorted(declared) if not hasattr(L, n)]
    assert not missing, f"declared but not exported: {missing}"


def test_python_signatures_cover_header():
    assert declared_symbols() <= set(_lib.SIGNATURES), \
        sorted(declared_symbols() - set(_lib.SIGNATURES))


def test_version_string():
    assert b"sm_100a" in _lib.lib().ft_version()


def test_null_arguments_are_shape_errors():
    L = _lib.lib()
    rc = L.ft_weight_upload_packed_u8(None, None, 4, 4, None, None)
    assert rc == 1
    assert b"null" in L.ft_last_error_string()
    with pytest.raises(_lib.ShapeError):
        _lib.check(rc)


@pytest.mark.skipif(os.path.exists("/dev/nvidia0"), reason="checks the no-GPU path")
def test_ctx_create_without_gpu_reports_device_error():
    h = C.c_void_p()
    rc = _lib.lib().ft_ctx_create(0, C.byref(h))
    assert rc == 6, _lib.lib().ft_last_error_string()


@pytest.mark.parametrize("n", [1, 3, 4, 17, 1024, 1027])
def test_host_pack_matches_oracle(n):
    rng = np.random.default_rng(n)
    v = rng.integers(-1, 2, size=n).astype(np.int8)
    p = ternary.pack_ternary(v)
    assert (p == fo.pack_ternary(v)).all()
    assert (ternary.unpack_ternary(p, n) == v).all()
    assert (ternary.pack_ternary_u32(p, n) == fo.pack_ternary_u32(p, n)).all()


def test_host_quantize_matches_oracle():
    rng = np.random.default_rng(1)
    w = (rng.standard_normal(4096) * 0.02).astype(np.float32)
    w[::97] = 0.0
    q1, a1 = ternary.quantize_ternary(w)
    q2, a2 = fo.quantize_ternary(w)
    assert a1 == a2 and (q1 == q2).all()


def test_rust_sys_crate_matches_header():
    """rust/ferris-ternary-sys declares every entry point of include/ferris_ternary.h with
    the same number of arguments (the crate cannot be compiled in this image)."""
    import re
    root = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
    h = open(os.path.join(root, "include", "ferris_ternary.h")).read()
    h = re.sub(r"/\*.*?\*/", "", h, flags=re.S)
    c = {n: len([a for a in args.split(",") if a.strip() and a.strip() != "void"])
         for n, args in re.findall(r"\b(ft_[a-z0-9_]+)\(([^)]*)\);", h, flags=re.S)}
    rs = open(os.path.join(root, "rust", "ferris-ternary-sys", "src", "lib.rs")).read()
    r = {n: len([a for a in args.split(",") if a.strip()])
         for n, args in re.findall(r"pub fn (ft_[a-z0-9_]+)\(([^)]*)\)", rs, flags=re.S)}
    assert c == r
