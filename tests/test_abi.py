"""CPU: the C-ABI library loads, exports every symbol include/kda_b200.h declares, and its
host-side validation returns the documented status codes (no device work is issued)."""
import ctypes
import os
import re

import pytest

from mlx_vit_b200 import _lib

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def header_symbols():
    syms = set()
    for fn in os.listdir(os.path.join(ROOT, "include")):
        if fn.endswith(".h"):
            txt = open(os.path.join(ROOT, "include", fn)).read()
            syms |= set(re.findall(r"KDA_API\s+[\w\s\*]+?\b(kda_\w+)\s*\(", txt))
    return syms


def test_library_exports_every_declared_symbol():
    L = _lib.lib()
    syms = header_symbols()
    assert {"kda_fwd", "kda_bwd", "kda_abi_version"} <= syms
    for s in syms:
        assert hasattr(L, s), s
    assert set(_lib.EXPORTS) >= syms


def test_abi_version_and_strerror():
    L = _lib.lib()
    assert L.kda_abi_version() == _lib.KDA_ABI_VERSION
    for code in _lib.STATUS:
        assert L.kda_strerror(code)
    assert b"unknown" in L.kda_strerror(12345)


def desc(**kw):
    d = dict(B=2, T=256, H=4, Dk=64, Dv=64, chunk=64, dtype_qkv=_lib.KDA_BF16,
             dtype_beta=_lib.KDA_BF16, flags=0, reserved=0)
    d.update(kw)
    return _lib.KdaDesc(**d)


@pytest.mark.parametrize("kw,status", [
    (dict(), 0),
    (dict(dtype_qkv=_lib.KDA_F32, dtype_beta=_lib.KDA_F32), 0),
    (dict(B=0), -1), (dict(T=-3), -1), (dict(chunk=0), -1),
    (dict(dtype_qkv=7), -3),
    (dict(Dv=32), -2), (dict(chunk=128), -2), (dict(Dk=256, Dv=256), -2),
    (dict(D=None) if False else dict(Dk=16, Dv=16, chunk=8), 0),
])
def test_check_desc_status(kw, status):
    L = _lib.lib()
    assert L.kda_check_desc(ctypes.byref(desc(**kw)), 0) == status


def test_negative_stride_rejected():
    L = _lib.lib()
    d = desc()
    d.q = _lib.KdaStrides(256 * 4 * 64, -4 * 64, 64)
    assert L.kda_check_desc(ctypes.byref(d), 0) == -1
    d.q = _lib.KdaStrides(256 * 4 * 64 * 3, 4 * 64 * 3, 64)  # a slice of a fused projection
    assert L.kda_check_desc(ctypes.byref(d), 0) == 0


def test_backward_head_dims_up_to_128():
    """Gradients exist for every head dim the forward takes (the fp32 kernels run D = 96 and
    D = 128 at a smaller internal chunk); beyond D = 128 both directions are refused."""
    L = _lib.lib()
    for D in (96, 128):
        d = desc(Dk=D, Dv=D, flags=_lib.KDA_FLAG_FORCE_GENERIC)
        assert L.kda_check_desc(ctypes.byref(d), 0) == 0
        assert L.kda_check_desc(ctypes.byref(d), 1) == 0
        assert L.kda_saved_bytes(ctypes.byref(d)) > 0
    d = desc(Dk=256, Dv=256)
    assert L.kda_check_desc(ctypes.byref(d), 1) == -2


def test_null_pointers_rejected_before_any_launch():
    L = _lib.lib()
    d = desc()
    z = ctypes.c_void_p(0)
    st = L.kda_fwd(ctypes.byref(d), *([z] * 9), z, 0, z)
    assert st == -1
    st = L.kda_bwd(ctypes.byref(d), *([z] * 15), z, 0, z)
    assert st == -1


def test_misaligned_pointer_rejected():
    L = _lib.lib()
    d = desc()
    a = ctypes.c_void_p(4096 + 4)
    ok = ctypes.c_void_p(8192)
    st = L.kda_fwd(ctypes.byref(d), a, ok, ok, ok, ok, ctypes.c_void_p(0), ok, ok,
                   ctypes.c_void_p(0), ctypes.c_void_p(0), 0, ctypes.c_void_p(0))
    assert st == -4


def test_workspace_query_is_consistent():
    L = _lib.lib()
    for bwd in (0, 1):
        assert L.kda_workspace_bytes(ctypes.byref(desc(B=0)), bwd) == 0
        n = L.kda_workspace_bytes(ctypes.byref(desc()), bwd)
        assert n >= 0
