"""CPU tests of the C boundary: the library loads, exports every entry point
include/fmha.h declares, and rejects bad arguments before touching CUDA (so
these calls need no GPU)."""
import ctypes

import numpy as np
import os
import re

import pytest

import fmha_b200
from fmha_b200 import _lib

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def declared_symbols():
    names = set()
    for h in os.listdir(os.path.join(ROOT, "include")):
        if h.endswith(".h"):
            src = open(os.path.join(ROOT, "include", h)).read()
            src = re.sub(r"/\*.*?\*/", "", src, flags=re.S)
            names |= set(re.findall(r"\b(fmha_\w+)\s*\(", src))
    return sorted(names)


def test_library_loads_and_exports_every_declared_symbol():
    lib = fmha_b200.load()
    names = declared_symbols()
    assert "fmha_forward" in names
    for n in names:
        assert hasattr(lib, n), n
        assert n in _lib.SIGNATURES, f"{n} has no ctypes signature"


def test_version():
    assert "sm_100a" in fmha_b200.version()


BASE = dict(q=16, k=32, v=48, o=64, batch=4, num_heads_q=16, num_heads_kv=16, seqlen_kv=16,
            head_dim=128)


def call(**kw):
    a = dict(BASE)
    a.update(kw)
    return fmha_b200.fmha_forward_ptr(a["q"], a["k"], a["v"], a["o"], a["batch"], a["num_heads_q"],
                                      a["num_heads_kv"], a["seqlen_kv"], a["head_dim"],
                                      variant=a.get("variant", "auto"))


@pytest.mark.parametrize("kw,status", [
    (dict(q=0), _lib.FMHA_ERR_INVALID_ARG),
    (dict(o=0), _lib.FMHA_ERR_INVALID_ARG),
    (dict(batch=-1), _lib.FMHA_ERR_INVALID_ARG),
    (dict(num_heads_q=0), _lib.FMHA_ERR_INVALID_ARG),
    (dict(num_heads_kv=0), _lib.FMHA_ERR_INVALID_ARG),
    (dict(num_heads_q=24, num_heads_kv=16), _lib.FMHA_ERR_INVALID_ARG),
    (dict(seqlen_kv=0), _lib.FMHA_ERR_INVALID_ARG),
    (dict(seqlen_kv=17), _lib.FMHA_ERR_UNSUPPORTED),
    (dict(head_dim=64), _lib.FMHA_ERR_UNSUPPORTED),
    (dict(head_dim=192), _lib.FMHA_ERR_UNSUPPORTED),
    (dict(num_heads_q=48, num_heads_kv=16), _lib.FMHA_ERR_UNSUPPORTED),   # 3 q heads per kv head
    (dict(num_heads_q=32, num_heads_kv=2), _lib.FMHA_ERR_UNSUPPORTED),    # 16 per kv head
    (dict(q=24), _lib.FMHA_ERR_MISALIGNED),
    (dict(v=8), _lib.FMHA_ERR_MISALIGNED),
    (dict(variant=7), _lib.FMHA_ERR_INVALID_ARG),
])
def test_rejected_before_any_cuda_call(kw, status):
    assert call(**kw) == status


def test_empty_batch_is_a_noop():
    assert call(batch=0, q=0, k=0, v=0, o=0) == _lib.FMHA_OK


def test_status_strings():
    for s in range(6):
        assert fmha_b200.status_string(s).startswith("FMHA_")
    assert "UNKNOWN" in fmha_b200.status_string(99)


def test_fill_rejects_bad_args():
    lib = fmha_b200.load()
    assert lib.fmha_fill_normal_bf16(None, 8, 0, 1, 0, None) == _lib.FMHA_ERR_INVALID_ARG
    assert lib.fmha_fill_normal_bf16(18, 8, 0, 1, 0, None) == _lib.FMHA_ERR_MISALIGNED
    assert lib.fmha_fill_normal_bf16(16, -1, 0, 1, 0, None) == _lib.FMHA_ERR_INVALID_ARG
    assert lib.fmha_fill_normal_bf16(16, 0, 0, 1, 0, None) == _lib.FMHA_OK


def test_device_error_needs_pointer():
    lib = fmha_b200.load()
    assert lib.fmha_device_error(ctypes.cast(0, ctypes.POINTER(ctypes.c_int))) == \
        _lib.FMHA_ERR_INVALID_ARG


def varlen(**kw):
    a = dict(q=16, k=32, v=48, o=64, cu=80, batch=4, hq=16, hkv=16, max_s=16, d=128, scale=0.0)
    a.update(kw)
    return fmha_b200.load().fmha_forward_varlen(a["q"], a["k"], a["v"], a["o"], a["cu"], a["batch"],
                                                a["hq"], a["hkv"], a["max_s"], a["d"], a["scale"],
                                                None)


@pytest.mark.parametrize("kw,status", [
    (dict(cu=None), _lib.FMHA_ERR_INVALID_ARG),
    (dict(cu=82), _lib.FMHA_ERR_MISALIGNED),
    (dict(scale=-1.0), _lib.FMHA_ERR_INVALID_ARG),
    (dict(scale=float("nan")), _lib.FMHA_ERR_INVALID_ARG),
    (dict(max_s=17), _lib.FMHA_ERR_UNSUPPORTED),
    (dict(max_s=0), _lib.FMHA_ERR_INVALID_ARG),
    (dict(d=64), _lib.FMHA_ERR_UNSUPPORTED),
    (dict(q=8), _lib.FMHA_ERR_MISALIGNED),
])
def test_varlen_rejected_before_any_cuda_call(kw, status):
    assert varlen(**kw) == status


def test_varlen_empty_batch_is_a_noop():
    assert varlen(batch=0, q=None, k=None, v=None, o=None, cu=None) == _lib.FMHA_OK


def test_seqlens_poisson_matches_reference_generator(oracle):
    """fmha_seqlens_poisson reproduces FMHAConfig::generate_seqlens_kv
    (fmha_host.cpp:58-72) -- the reference build's own output."""
    got = fmha_b200.seqlens_poisson(30720, 16)
    assert got.min() >= 2 and got.max() <= 16 and abs(got.mean() - 4.4) < 0.2
    if not oracle.ref_available():
        pytest.skip("reference build absent")
    assert np.array_equal(got, oracle.ref_generate_seqlens(30720, 16))
    assert np.array_equal(fmha_b200.seqlens_poisson(100, 8), oracle.ref_generate_seqlens(100, 8))


def test_compat_header_compiles_on_cpu(tmp_path):
    """include/fmha_compat.hpp is valid C++ for a host compiler (the reference
    call site's translation unit)."""
    import shutil
    import subprocess
    nvcc = shutil.which("nvcc") or "/usr/local/cuda/bin/nvcc"
    src = os.path.join(ROOT, "tests", "cpp", "compat_call.cpp")
    subprocess.check_call([nvcc, "-std=c++17", "-I" + os.path.join(ROOT, "include"), "-c", src,
                           "-o", str(tmp_path / "c.o")])


def test_oversized_unit_count_is_rejected():
    """More than 2**30 (batch, kv head) units is outside the kernels' int32
    chunk indexing: rejected up front, not truncated."""
    assert call(batch=1 << 26, num_heads_q=32, num_heads_kv=32) == _lib.FMHA_ERR_UNSUPPORTED


def test_append_rejects_bad_new_rows():
    lib = fmha_b200.load()
    args = [16, 32, 48, None, 80, 96, 2, 16, 16, 8, 8, 128, None]
    assert lib.fmha_forward_append(*args) == _lib.FMHA_ERR_INVALID_ARG
    args[3] = 72
    assert lib.fmha_forward_append(*args) == _lib.FMHA_ERR_MISALIGNED


@pytest.mark.parametrize("variant,status", [(7, _lib.FMHA_ERR_INVALID_ARG),
                                            (-1, _lib.FMHA_ERR_INVALID_ARG)])
def test_varlen_variant_rejects_unknown_kernel(variant, status):
    lib = fmha_b200.load()
    assert lib.fmha_forward_varlen_variant(16, 32, 48, 64, 80, 4, 16, 16, 16, 128, 0.0, variant,
                                           None) == status
    # the selector is checked before anything else, even for an empty batch
    assert lib.fmha_forward_varlen_variant(None, None, None, None, None, 0, 16, 16, 16, 128, 0.0,
                                           variant, None) == status


def test_varlen_negative_scale_is_rejected_not_defaulted():
    """softmax_scale == 0 selects 1/sqrt(head_dim); any negative value is an
    error, never silently the default."""
    for sc in (-1.0, -1e-30, float("-inf"), float("inf")):
        assert varlen(scale=sc) == _lib.FMHA_ERR_INVALID_ARG


@pytest.mark.parametrize("lam,max_s", [(1000.0, 16), (200.0, 16), (1e6, 2)])
def test_seqlens_poisson_rejects_lambda_far_from_range(lam, max_s):
    """A lambda whose draws practically never land in [2, max_seqlen_kv]
    returns FMHA_ERR_INVALID_ARG instead of looping for ever."""
    out = np.empty(64, dtype=np.int32)
    st = fmha_b200.load().fmha_seqlens_poisson(64, max_s, 42, lam, out.ctypes.data)
    assert st == _lib.FMHA_ERR_INVALID_ARG


def test_seqlens_poisson_redraw_cap_ends_the_loop():
    """lambda inside the accepted range but with almost no mass in [2, 3]:
    the per-row redraw cap ends the call with an error, in bounded time."""
    import time
    out = np.empty(4, dtype=np.int32)
    t0 = time.perf_counter()
    st = fmha_b200.load().fmha_seqlens_poisson(4, 3, 42, 60.0, out.ctypes.data)
    assert st == _lib.FMHA_ERR_INVALID_ARG
    assert time.perf_counter() - t0 < 30


@pytest.mark.parametrize("kw,status", [
    (dict(batch=1 << 26, num_heads_q=32, num_heads_kv=32), _lib.FMHA_ERR_UNSUPPORTED),
    (dict(head_dim=64), _lib.FMHA_ERR_UNSUPPORTED),
    (dict(seqlen_kv=17), _lib.FMHA_ERR_UNSUPPORTED),
    (dict(q=40), _lib.FMHA_ERR_MISALIGNED),
    (dict(o=0), _lib.FMHA_ERR_INVALID_ARG),
    (dict(num_heads_q=24, num_heads_kv=16), _lib.FMHA_ERR_INVALID_ARG),
])
def test_noalloc_rejected_before_any_cuda_call(kw, status):
    a = dict(BASE)
    a.update(kw)
    got = fmha_b200.load().fmha_forward_noalloc(a["q"], a["k"], a["v"], a["o"], a["batch"],
                                                a["num_heads_q"], a["num_heads_kv"],
                                                a["seqlen_kv"], a["head_dim"], None)
    assert got == status


def test_noalloc_empty_batch_is_a_noop():
    assert fmha_b200.load().fmha_forward_noalloc(None, None, None, None, 0, 16, 16, 16, 128,
                                                 None) == _lib.FMHA_OK
