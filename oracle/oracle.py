"""ctypes bindings for the CPU checkers (test infrastructure only).

Only ``tests/``, ``__graft_entry__.smoke()`` and ``bench.py``'s CPU-baseline
and reference legs may import this module. It wraps:

* ``_build/libfmha_oracle.so`` -- the restatement of the reference's CPU
  attention (``fmha_host.cpp:158-244``) in the [B,H,S,D] layout and in the
  reference's packed layout, plus the seeded input generator;
* ``_ref/libfmha_ref.so`` (when it was built) -- the reference's own
  ``do_validation`` (``fmha_host.cpp:158-284``) and seqlen generator
  (``fmha_host.cpp:58-72``), compiled from the reference sources.

Arrays are numpy ``uint16`` bit patterns for bf16/fp16 and ``float32``.
"""
from __future__ import annotations

import ctypes
import os
import subprocess

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
ORACLE_SO = os.path.join(HERE, "_build", "libfmha_oracle.so")
REF_SO = os.path.join(HERE, "_ref", "libfmha_ref.so")

TENSOR_Q, TENSOR_K, TENSOR_V = 1, 2, 3

_u16p = np.ctypeslib.ndpointer(np.uint16, flags="C_CONTIGUOUS")
_f32p = np.ctypeslib.ndpointer(np.float32, flags="C_CONTIGUOUS")
_i32p = np.ctypeslib.ndpointer(np.int32, flags="C_CONTIGUOUS")
_i64, _int = ctypes.c_int64, ctypes.c_int


def build(ref_dir: str | None = None) -> None:
    """Compile the restatement, and the reference build when its sources exist
    (``ref_dir``, else $FMHA_REF_DIR; no built-in location)."""
    subprocess.check_call(["make", "-s", "-C", HERE, "all"])
    ref_dir = ref_dir or os.environ.get("FMHA_REF_DIR", "")
    if ref_dir and os.path.isfile(os.path.join(ref_dir, "fmha_host.cpp")):
        subprocess.check_call(["make", "-s", "-C", HERE, "ref", f"REF_DIR={ref_dir}"],
                              stderr=subprocess.DEVNULL)


_lib = None
_ref = None


def lib():
    global _lib
    if _lib is None:
        if not os.path.exists(ORACLE_SO):
            build()
        L = ctypes.CDLL(ORACLE_SO)
        L.fmha_oracle_gen_bf16.argtypes = [_u16p, _i64, ctypes.c_uint64, ctypes.c_uint32, _i64]
        L.fmha_oracle_gen_bf16.restype = None
        opt_f32 = ctypes.c_void_p
        L.fmha_oracle_decode_bhsd.argtypes = [_u16p, _u16p, _u16p, _i64, _int, _int, _int, _int,
                                              _int, opt_f32, opt_f32]
        L.fmha_oracle_decode_bhsd.restype = None
        L.fmha_oracle_decode_thd.argtypes = [_u16p, _u16p, _u16p, _i32p, _i64, _int, _int, _int,
                                             _int, opt_f32, opt_f32]
        L.fmha_oracle_decode_thd.restype = None
        L.fmha_oracle_threads.restype = _int
        L.fmha_oracle_set_threads.argtypes = [_int]
        _lib = L
    return _lib


def ref_available() -> bool:
    return os.path.exists(REF_SO)


def ref():
    """The reference's own CPU code (raises if it was never built here)."""
    global _ref
    if _ref is None:
        if not ref_available():
            raise FileNotFoundError(f"{REF_SO} was not built (reference sources absent)")
        R = ctypes.CDLL(REF_SO)
        R.fmha_ref_do_validation.argtypes = [_u16p, _u16p, _u16p, _i32p, _int, _int, _int, _int,
                                             _u16p, _u16p, _int, _int]
        R.fmha_ref_do_validation.restype = _int
        R.fmha_ref_generate_seqlens.argtypes = [_int, _int, _i32p]
        R.fmha_ref_generate_seqlens.restype = None
        R.fmha_ref_hardware_threads.restype = _int
        _ref = R
    return _ref


def _ptr(a):
    return None if a is None else a.ctypes.data


def gen_bf16(n: int, seed: int, tensor_id: int, offset: int = 0) -> np.ndarray:
    out = np.empty(int(n), dtype=np.uint16)
    lib().fmha_oracle_gen_bf16(out, int(n), seed, tensor_id, int(offset))
    return out


def make_inputs_bhsd(batch, hq, hkv, s, d, seed=0, batch_offset=0):
    """Seeded Q [B,Hq,D], K/V [B,Hkv,S,D] (bf16 bits) for batch rows
    [batch_offset, batch_offset+batch) of a larger job."""
    q = gen_bf16(batch * hq * d, seed, TENSOR_Q, batch_offset * hq * d)
    k = gen_bf16(batch * hkv * s * d, seed, TENSOR_K, batch_offset * hkv * s * d)
    v = gen_bf16(batch * hkv * s * d, seed, TENSOR_V, batch_offset * hkv * s * d)
    return q, k, v


def decode_bhsd(q, k, v, batch, hq, hkv, s, d, p_bf16=False, want_f32=True):
    """Returns (O_f32 or None, O_f16 bits)."""
    o32 = np.empty(batch * hq * d, dtype=np.float32) if want_f32 else None
    o16 = np.empty(batch * hq * d, dtype=np.uint16)
    lib().fmha_oracle_decode_bhsd(q, k, v, batch, hq, hkv, s, d, int(p_bf16), _ptr(o32), _ptr(o16))
    return o32, o16


def decode_thd(q, k, v, cu_seqlens, batch, hq, hkv, d, p_bf16=False, want_f32=True):
    o32 = np.empty(batch * hq * d, dtype=np.float32) if want_f32 else None
    o16 = np.empty(batch * hq * d, dtype=np.uint16)
    cu = np.ascontiguousarray(cu_seqlens, dtype=np.int32)
    lib().fmha_oracle_decode_thd(q, k, v, cu, batch, hq, hkv, d, int(p_bf16), _ptr(o32), _ptr(o16))
    return o32, o16


def ref_do_validation(q, k, v, seqlens, batch, hq, hkv, d, h_o=None, threads=1, quiet=True):
    """Run the reference's do_validation(); returns (passed, ref_O fp16 bits)."""
    ref_o = np.zeros(batch * hq * d, dtype=np.uint16)
    if h_o is None:
        h_o = np.zeros_like(ref_o)
    sl = np.ascontiguousarray(seqlens, dtype=np.int32)
    ok = ref().fmha_ref_do_validation(q, k, v, sl, batch, hq, hkv, d, ref_o,
                                      np.ascontiguousarray(h_o, dtype=np.uint16), threads, int(quiet))
    return bool(ok), ref_o


def ref_generate_seqlens(batch, max_seqlen_kv=16):
    out = np.empty(batch, dtype=np.int32)
    ref().fmha_ref_generate_seqlens(batch, max_seqlen_kv, out)
    return out


def bf16_to_f32(bits: np.ndarray) -> np.ndarray:
    return (bits.astype(np.uint32) << 16).view(np.float32)


def f16_to_f32(bits: np.ndarray) -> np.ndarray:
    return bits.view(np.float16).astype(np.float32)


def threads() -> int:
    return lib().fmha_oracle_threads()


def set_threads(n: int) -> None:
    lib().fmha_oracle_set_threads(int(n))
