"""ctypes binding of libfmha_b200.so (the C ABI declared in include/fmha.h).

Loading fails loudly: there is no CPU or PyTorch fallback for any entry point.
"""
from __future__ import annotations

import ctypes
import os

PKG = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(PKG, "libfmha_b200.so")

FMHA_OK = 0
FMHA_ERR_INVALID_ARG = 1
FMHA_ERR_UNSUPPORTED = 2
FMHA_ERR_MISALIGNED = 3
FMHA_ERR_CUDA = 4
FMHA_ERR_DEVICE_TIMEOUT = 5

VARIANT_AUTO, VARIANT_BULK, VARIANT_LDG = 0, 1, 2
VARIANTS = {"auto": VARIANT_AUTO, "bulk": VARIANT_BULK, "ldg": VARIANT_LDG}

# Every symbol include/fmha.h declares, with (restype, argtypes).
_vp, _i, _i64, _u64, _u32 = ctypes.c_void_p, ctypes.c_int, ctypes.c_int64, ctypes.c_uint64, ctypes.c_uint32
SIGNATURES = {
    "fmha_forward": (_i, [_vp, _vp, _vp, _vp, _i, _i, _i, _i, _i, _vp]),
    "fmha_forward_variant": (_i, [_vp, _vp, _vp, _vp, _i, _i, _i, _i, _i, _i, _vp]),
    "fmha_forward_noalloc": (_i, [_vp, _vp, _vp, _vp, _i, _i, _i, _i, _i, _vp]),
    "fmha_forward_varlen": (_i, [_vp, _vp, _vp, _vp, _vp, _i, _i, _i, _i, _i, ctypes.c_float, _vp]),
    "fmha_forward_varlen_variant": (_i, [_vp, _vp, _vp, _vp, _vp, _i, _i, _i, _i, _i,
                                         ctypes.c_float, _i, _vp]),
    "fmha_forward_append": (_i, [_vp, _vp, _vp, _vp, _vp, _vp, _i, _i, _i, _i, _i, _i, _vp]),
    "fmha_status_string": (ctypes.c_char_p, [_i]),
    "fmha_device_error": (_i, [ctypes.POINTER(_i)]),
    "fmha_fill_normal_bf16": (_i, [_vp, _i64, _u64, _u32, _i64, _vp]),
    "fmha_version": (ctypes.c_char_p, []),
    "fmha_seqlens_poisson": (_i, [_i, _i, _u32, ctypes.c_double, _vp]),
    "fmha_test_inject_stall": (None, [_i]),
}

_lib = None


class FmhaError(RuntimeError):
    def __init__(self, status: int, what: str = ""):
        self.status = status
        msg = status_string(status) if _lib is not None else f"status {status}"
        super().__init__(f"{what}: {msg}" if what else msg)


def load(path: str | None = None) -> ctypes.CDLL:
    """Loads the CUDA library (built in-tree by fmha_b200.build)."""
    global _lib
    if _lib is not None:
        return _lib
    path = path or LIB_PATH
    if not os.path.exists(path):
        raise ImportError(
            f"{path} is missing: build it with `python -m fmha_b200.build` "
            "(fmha_b200 has no fallback implementation)")
    lib = ctypes.CDLL(path)
    for name, (res, args) in SIGNATURES.items():
        fn = getattr(lib, name)
        fn.restype, fn.argtypes = res, args
    _lib = lib
    return lib


def status_string(status: int) -> str:
    return load().fmha_status_string(int(status)).decode()


def check(status: int, what: str = "") -> None:
    if status != FMHA_OK:
        raise FmhaError(status, what)
