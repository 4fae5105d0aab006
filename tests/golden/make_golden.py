"""Generates the golden fixtures in this folder from the REFERENCE'S OWN CPU
code (HGLiu1998/fmha fmha_host.cpp do_validation, compiled from its sources by
oracle/Makefile into oracle/_ref/libfmha_ref.so).

Each fixture fixes a shape and a seed; the inputs are regenerated from the
seeded counter-based generator (fmha_oracle_gen_bf16 / fmha_fill_normal_bf16),
so only the reference's fp16 output bits (and the seqlens) are stored.

  thd_*.npz   packed varlen layout [sum S_b, H, D] with the reference's own
              Poisson(4) seqlens (fmha_host.cpp:58-72); K/V generated in
              that layout.
  bhsd_*.npz  fixed seqlen; K/V generated in [B,H,S,D] and handed to the
              reference transposed to its [B*S, H, D] packing, so ref_O is
              the reference's answer for the [B,H,S,D] problem.

The reference computes with bf16-rounded P (fmha_host.cpp:225); fixtures are
its output verbatim. Run: python tests/golden/make_golden.py
"""
from __future__ import annotations

import os
import sys

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, os.path.dirname(os.path.dirname(HERE)))
from oracle import oracle as O  # noqa: E402

THD_CASES = [  # (batch, heads, head_dim, seed)
    (10, 16, 128, 11),   # the reference's own "Testing" config, fmha_host.cpp:512
    (12, 32, 256, 12),
    (9, 16, 256, 13),
]
BHSD_CASES = [  # (batch, heads, seqlen, head_dim, seed)
    (6, 16, 1, 128, 21),
    (5, 16, 16, 128, 22),
    (4, 32, 16, 256, 23),
    (7, 16, 3, 256, 24),
    (3, 32, 8, 128, 25),
]


def checksum(*arrays):
    """Position-weighted sum of the input bits: pins the generator too."""
    tot = 0
    for a in arrays:
        w = np.arange(1, a.size + 1, dtype=np.uint64)
        tot = (tot + int((a.astype(np.uint64) * w).sum(dtype=np.uint64))) % (1 << 61)
    return np.int64(tot)


def thd_case(b, h, d, seed):
    sl = O.ref_generate_seqlens(b, 16)
    total = int(sl.sum())
    q = O.gen_bf16(b * h * d, seed, O.TENSOR_Q)
    k = O.gen_bf16(total * h * d, seed, O.TENSOR_K)
    v = O.gen_bf16(total * h * d, seed, O.TENSOR_V)
    _, ref_o = O.ref_do_validation(q, k, v, sl, b, h, h, d)
    return dict(input_checksum=checksum(q, k, v), kind="thd", batch=b, heads=h, head_dim=d, seed=seed, seqlens=sl, ref_o=ref_o)


def bhsd_to_packed(x, b, h, s, d):
    return np.ascontiguousarray(x.reshape(b, h, s, d).transpose(0, 2, 1, 3)).reshape(-1)


def bhsd_case(b, h, s, d, seed):
    q, k, v = O.make_inputs_bhsd(b, h, h, s, d, seed)
    sl = np.full(b, s, dtype=np.int32)
    _, ref_o = O.ref_do_validation(q, bhsd_to_packed(k, b, h, s, d), bhsd_to_packed(v, b, h, s, d),
                                   sl, b, h, h, d)
    return dict(input_checksum=checksum(q, k, v), kind="bhsd", batch=b, heads=h, seqlen=s, head_dim=d, seed=seed, ref_o=ref_o)


def main():
    for (b, h, d, seed) in THD_CASES:
        f = thd_case(b, h, d, seed)
        np.savez_compressed(os.path.join(HERE, f"thd_b{b}_h{h}_d{d}_s{seed}.npz"), **f)
    for (b, h, s, d, seed) in BHSD_CASES:
        f = bhsd_case(b, h, s, d, seed)
        np.savez_compressed(os.path.join(HERE, f"bhsd_b{b}_h{h}_s{s}_d{d}_seed{seed}.npz"), **f)
    print("wrote", sorted(x for x in os.listdir(HERE) if x.endswith(".npz")))


if __name__ == "__main__":
    main()
