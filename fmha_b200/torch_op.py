"""PyTorch custom op over the C ABI: ``torch.ops.fmha_b200.decode``.

``decode(q, k, v) -> o`` with q [B,Hq,1,D] bf16, k/v [B,Hkv,S,D] bf16 (CUDA,
contiguous), o [B,Hq,1,D] fp16, scale 1/sqrt(D) -- the same call as
``fmha_forward`` registered with ``torch.library`` so it composes with torch
code (and has a shape-only fake implementation for tracing). The CUDA kernel
of libfmha_b200 runs on the current stream; there is no fallback.
"""
from __future__ import annotations

import torch

from . import _lib, fmha_forward_ptr

_lib.load()


@torch.library.custom_op("fmha_b200::decode", mutates_args=())
def decode(q: torch.Tensor, k: torch.Tensor, v: torch.Tensor) -> torch.Tensor:
    if k.dim() != 4 or v.shape != k.shape or q.dim() != 4 or q.shape[2] != 1:
        raise ValueError("decode: q [B,Hq,1,D], k/v [B,Hkv,S,D]")
    b, hkv, s, d = k.shape
    hq = q.shape[1]
    q, k, v = q.contiguous(), k.contiguous(), v.contiguous()
    o = torch.empty((b, hq, 1, d), dtype=torch.float16, device=q.device)
    st = fmha_forward_ptr(q, k, v, o, b, hq, hkv, s, d,
                          stream=torch.cuda.current_stream(q.device).cuda_stream)
    _lib.check(st, "fmha_b200::decode")
    return o


@decode.register_fake
def _(q, k, v):
    return q.new_empty((q.shape[0], q.shape[1], 1, q.shape[3]), dtype=torch.float16)
