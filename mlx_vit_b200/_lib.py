"""ctypes binding of libkda_b200.so (declarations: include/kda_b200.h).

The library is loaded from the package directory.  There is no fallback: if the shared
object is missing or does not export the expected ABI, ``lib()`` raises.
"""
from __future__ import annotations

import ctypes
import os
import threading

_HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(_HERE, "libkda_b200.so")

KDA_ABI_VERSION = 6
KDA_F32, KDA_BF16, KDA_F16 = 0, 1, 2
KDA_FLAG_FORCE_GENERIC = 0x1
KDA_FLAG_DEBUG_WAIT_TIMEOUT = 0x2

STATUS = {
    0: "KDA_OK", -1: "KDA_ERR_INVALID_ARG", -2: "KDA_ERR_UNSUPPORTED", -3: "KDA_ERR_DTYPE",
    -4: "KDA_ERR_MISALIGNED", -5: "KDA_ERR_WORKSPACE", -6: "KDA_ERR_CUDA", -7: "KDA_ERR_TIMEOUT",
    -8: "KDA_ERR_SCRATCH_LIMIT",
}
STATUS_CODE = {v: k for k, v in STATUS.items()}
KDA_NOALLOC_SCRATCH_BYTES = 32 << 20

# every symbol include/kda_b200.h declares
EXPORTS = ("kda_abi_version", "kda_strerror", "kda_check_desc", "kda_workspace_bytes",
           "kda_saved_bytes", "kda_launch_counter", "kda_device_status", "kda_fwd", "kda_bwd",
           "kda_bwd_noalloc", "kda_fwd_gated", "kda_bwd_gated", "kda_fwd_recurrent",
           "kda_l2norm_silu_fwd", "kda_l2norm_silu_bwd", "kda_gated_rmsnorm_fwd", "kda_gated_rmsnorm_bwd",
           "kda_conv_silu_fwd", "kda_conv_silu_bwd")


class KdaStrides(ctypes.Structure):
    """Element strides (b, t, h) of one input; all zero = dense (include/kda_b200.h)."""
    _fields_ = [("b", ctypes.c_int64), ("t", ctypes.c_int64), ("h", ctypes.c_int64)]


class KdaDesc(ctypes.Structure):
    _fields_ = [("B", ctypes.c_int64), ("T", ctypes.c_int64), ("H", ctypes.c_int64),
                ("Dk", ctypes.c_int64), ("Dv", ctypes.c_int64), ("chunk", ctypes.c_int64),
                ("dtype_qkv", ctypes.c_int32), ("dtype_beta", ctypes.c_int32),
                ("flags", ctypes.c_int32), ("reserved", ctypes.c_int32),
                ("q", KdaStrides), ("k", KdaStrides), ("v", KdaStrides), ("g", KdaStrides),
                ("beta", KdaStrides), ("dO", KdaStrides)]


class KdaGate(ctypes.Structure):
    """The layer's decay / write gate inputs (include/kda_b200.h, KdaGate)."""
    _fields_ = [("f", ctypes.c_void_p), ("A_log", ctypes.c_void_p), ("dt_bias", ctypes.c_void_p),
                ("b", ctypes.c_void_p), ("allow_neg_eigval", ctypes.c_int32), ("reserved", ctypes.c_int32)]


class KdaError(RuntimeError):
    def __init__(self, status: int, msg: str, where: str):
        super().__init__(f"{where}: {STATUS.get(status, status)} ({msg})")
        self.status = status


_lib = None
_lock = threading.Lock()


def _declare(L):
    P, S, I = ctypes.c_void_p, ctypes.c_size_t, ctypes.c_int
    D = ctypes.POINTER(KdaDesc)
    L.kda_abi_version.restype = I
    L.kda_abi_version.argtypes = []
    L.kda_strerror.restype = ctypes.c_char_p
    L.kda_strerror.argtypes = [I]
    L.kda_check_desc.restype = I
    L.kda_check_desc.argtypes = [D, I]
    L.kda_workspace_bytes.restype = S
    L.kda_workspace_bytes.argtypes = [D, I]
    L.kda_saved_bytes.restype = S
    L.kda_saved_bytes.argtypes = [D]
    L.kda_device_status.restype = I
    L.kda_device_status.argtypes = [I]
    L.kda_launch_counter.restype = ctypes.c_uint64
    L.kda_launch_counter.argtypes = []
    L.kda_fwd.restype = I
    L.kda_fwd.argtypes = [D] + [P] * 9 + [P, S, P]
    L.kda_bwd.restype = I
    L.kda_bwd.argtypes = [D] + [P] * 15 + [P, S, P]
    L.kda_bwd_noalloc.restype = I
    L.kda_bwd_noalloc.argtypes = [D] + [P] * 15 + [P]
    G = ctypes.POINTER(KdaGate)
    L.kda_fwd_gated.restype = I
    L.kda_fwd_gated.argtypes = [D, P, P, P, G, P, P, P, P, P, S, P]
    L.kda_bwd_gated.restype = I
    L.kda_bwd_gated.argtypes = [D, P, P, P, G] + [P] * 12 + [P, S, P]
    L.kda_fwd_recurrent.restype = I
    L.kda_fwd_recurrent.argtypes = [D] + [P] * 9
    i64, f32 = ctypes.c_int64, ctypes.c_float
    for n, a in (("kda_l2norm_silu_fwd", [i64, I, P, P, f32, P]),
                 ("kda_l2norm_silu_bwd", [i64, I, P, P, P, f32, P]),
                 ("kda_gated_rmsnorm_fwd", [i64, I, P, P, P, P, f32, P]),
                 ("kda_gated_rmsnorm_bwd", [i64, I, P, P, P, P, P, P, P, f32, P]),
                 ("kda_conv_silu_fwd", [i64, i64, I, I, P, P, P, P, I, f32, P]),
                 ("kda_conv_silu_bwd", [i64, i64, I, I, P, P, P, P, P, P, P, I, f32, P, P])):
        getattr(L, n).restype = I
        getattr(L, n).argtypes = a


def lib(path: str | None = None):
    """Load (once) and return the ctypes handle; raises if the library is unusable."""
    global _lib
    if _lib is not None and path is None:
        return _lib
    with _lock:
        if _lib is not None and path is None:
            return _lib
        p = path or LIB_PATH
        if not os.path.exists(p):
            raise RuntimeError(f"libkda_b200.so not built ({p} missing): run "
                               "`python -m mlx_vit_b200.build` (no fallback path exists)")
        L = ctypes.CDLL(p)
        for name in EXPORTS:
            if not hasattr(L, name):
                raise RuntimeError(f"{p} does not export {name}")
        _declare(L)
        v = L.kda_abi_version()
        if v != KDA_ABI_VERSION:
            raise RuntimeError(f"{p}: ABI version {v}, expected {KDA_ABI_VERSION}")
        if path is None:
            _lib = L
        return L


def check(status: int, where: str):
    if status != 0:
        raise KdaError(status, lib().kda_strerror(status).decode(), where)
