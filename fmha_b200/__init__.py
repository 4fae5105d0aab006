"""fmha_b200 -- B200-native (sm_100a) batched flash-decode attention.

The product is the C ABI of ``libfmha_b200.so`` (``include/fmha.h``). This
module is its Python host-side mirror: ``fmha_forward`` takes the same
arguments as the C entry point (raw device pointers, or torch tensors for
convenience) and raises :class:`FmhaError` carrying the C status on failure.
There is no CPU or PyTorch fallback: if the library is missing, importing the
binding raises.

Layout (the reference's Q/O layout, with K/V in [B,H,S,D]):
  Q [B, Hq, 1, D] bf16, K/V [B, Hkv, S, D] bf16, O [B, Hq, 1, D] fp16.
"""
from __future__ import annotations

from ._lib import (FMHA_ERR_CUDA, FMHA_ERR_DEVICE_TIMEOUT, FMHA_ERR_INVALID_ARG,  # noqa: F401
                   FMHA_ERR_MISALIGNED, FMHA_ERR_UNSUPPORTED, FMHA_OK, VARIANT_AUTO,
                   VARIANT_BULK, VARIANT_LDG, VARIANTS, FmhaError, check, load, status_string)

__all__ = ["fmha_forward", "fmha_forward_ptr", "fmha_forward_varlen_ptr", "seqlens_poisson", "fill_normal_bf16", "device_error", "FmhaError",
           "load", "version"]

TENSOR_Q, TENSOR_K, TENSOR_V = 1, 2, 3


def _ptr(x) -> int:
    if x is None:
        return 0
    if isinstance(x, int):
        return x
    return x.data_ptr()


def _stream_handle(stream) -> int:
    if stream is None:
        try:
            import torch
            if torch.cuda.is_available():
                return torch.cuda.current_stream().cuda_stream
        except ImportError:
            pass
        return 0
    if isinstance(stream, int):
        return stream
    return stream.cuda_stream


def fmha_forward_ptr(q, k, v, o, batch, num_heads_q, num_heads_kv, seqlen_kv, head_dim,
                     stream=0, variant="auto") -> int:
    """Raw C call; returns the fmha_status_t (does not raise). Pointers are
    ints or tensors; stream is a cudaStream_t as int, a torch stream, or None
    for torch's current stream."""
    lib = load()
    var = VARIANTS[variant] if isinstance(variant, str) else int(variant)
    return lib.fmha_forward_variant(_ptr(q), _ptr(k), _ptr(v), _ptr(o), int(batch),
                                    int(num_heads_q), int(num_heads_kv), int(seqlen_kv),
                                    int(head_dim), var, _stream_handle(stream))


def fmha_forward(q, k, v, o=None, *, stream=None, variant="auto"):
    """Decode attention on torch tensors: q [B,Hq,1,D] (or [B,Hq,D]) bf16,
    k/v [B,Hkv,S,D] bf16 on the same CUDA device. Writes and returns o
    [B,Hq,1,D] fp16 (allocated if not given). Raises FmhaError on failure."""
    import torch
    if k.dim() != 4 or v.shape != k.shape:
        raise FmhaError(FMHA_ERR_INVALID_ARG, "k/v must be [B,Hkv,S,D] with equal shapes")
    b, hkv, s, d = k.shape
    hq = q.shape[1]
    if q.numel() != b * hq * d:
        raise FmhaError(FMHA_ERR_INVALID_ARG, "q must be [B,Hq,1,D]")
    for t in (q, k, v):
        if t.dtype != torch.bfloat16 or not t.is_contiguous() or not t.is_cuda:
            raise FmhaError(FMHA_ERR_INVALID_ARG, "q/k/v must be contiguous bf16 CUDA tensors")
    if o is None:
        o = torch.empty((b, hq, 1, d), dtype=torch.float16, device=q.device)
    elif o.dtype != torch.float16 or not o.is_contiguous() or o.numel() != b * hq * d:
        raise FmhaError(FMHA_ERR_INVALID_ARG, "o must be contiguous fp16 [B,Hq,1,D]")
    st = fmha_forward_ptr(q, k, v, o, b, hq, hkv, s, d, stream=_stream_handle(stream),
                          variant=variant)
    check(st, "fmha_forward")
    return o


def fill_normal_bf16(t, seed: int, tensor_id: int, offset: int = 0, stream=None):
    """Fills a contiguous bf16 CUDA tensor with the seeded generator."""
    st = load().fmha_fill_normal_bf16(t.data_ptr(), t.numel(), seed, tensor_id, offset,
                                      _stream_handle(stream))
    check(st, "fmha_fill_normal_bf16")
    return t


def seqlens_poisson(batch: int, max_seqlen_kv: int = 16, seed: int = 42, lam: float = 4.0):
    """The reference benchmark's KV lengths (Poisson(4) in [2, 16], seed 42)."""
    import numpy as np
    out = np.empty(batch, dtype=np.int32)
    check(load().fmha_seqlens_poisson(batch, max_seqlen_kv, seed, lam, out.ctypes.data),
          "fmha_seqlens_poisson")
    return out


VARLEN_KERNELS = {"auto": VARIANT_AUTO, "chunk": VARIANT_BULK, "ldg": VARIANT_LDG}


def fmha_forward_varlen_ptr(q, k, v, o, cu_seqlens, batch, num_heads_q, num_heads_kv,
                            max_seqlen_kv, head_dim, softmax_scale=0.0, stream=None,
                            kernel="auto") -> int:
    """Raw C call of fmha_forward_varlen (kernel "auto") or
    fmha_forward_varlen_variant ("chunk" or "ldg"); returns the status."""
    args = (_ptr(q), _ptr(k), _ptr(v), _ptr(o), _ptr(cu_seqlens), int(batch), int(num_heads_q),
            int(num_heads_kv), int(max_seqlen_kv), int(head_dim), float(softmax_scale))
    if kernel == "auto":
        return load().fmha_forward_varlen(*args, _stream_handle(stream))
    return load().fmha_forward_varlen_variant(*args, VARLEN_KERNELS[kernel],
                                              _stream_handle(stream))


def device_error() -> int:
    """Reads and clears the current device's error word (synchronises)."""
    import ctypes
    code = ctypes.c_int(0)
    check(load().fmha_device_error(ctypes.byref(code)), "fmha_device_error")
    return code.value


def version() -> str:
    return load().fmha_version().decode()
