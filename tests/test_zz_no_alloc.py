"""fmha_forward_noalloc: the dense call for callers that cannot allocate
device memory (an allocator hook, a plug-in whose host owns every
allocation, a fixed memory budget). Its only scratch is a static device
array inside the library, shared by every call. Called through the C ABI,
its output must match fmha_forward's (ldg family, the same kernels) within
the library tolerance, on two calls in a row: the second call reuses the
scratch the first one left behind. This file sorts last so that a run
stopping at the first failure has run every other test first."""
import ctypes

import numpy as np
import pytest

import fmha_b200

pytestmark = pytest.mark.gpu

ATOL, RTOL = 2e-3, 1e-2


def _close(a_bits, b_bits):
    a = a_bits.view(np.float16).astype(np.float32)
    b = b_bits.view(np.float16).astype(np.float32)
    err = np.abs(a - b)
    assert np.all(np.isfinite(a))
    assert np.all((err <= ATOL) | (err <= RTOL * np.abs(b))), f"max abs err {err.max():.3e}"


@pytest.mark.parametrize("b,hq,hkv,s,d", [(3840, 32, 32, 16, 256), (1000, 16, 16, 1, 128),
                                          (257, 32, 16, 7, 256), (33, 32, 4, 3, 128)])
def test_noalloc_matches_fmha_forward_twice(b, hq, hkv, s, d):
    import torch
    if not torch.cuda.is_available():
        pytest.fail("GPU test collected on a machine without CUDA")
    lib = fmha_b200.load()
    dev = torch.device("cuda", 0)
    Q = torch.empty(b * hq * d, dtype=torch.bfloat16, device=dev)
    K = torch.empty(b * hkv * s * d, dtype=torch.bfloat16, device=dev)
    V = torch.empty_like(K)
    for t, tid in ((Q, 1), (K, 2), (V, 3)):
        fmha_b200.fill_normal_bf16(t, seed=17, tensor_id=tid)
    ref = torch.empty(b * hq * d, dtype=torch.float16, device=dev)
    st = lib.fmha_forward_variant(Q.data_ptr(), K.data_ptr(), V.data_ptr(), ref.data_ptr(), b, hq,
                                  hkv, s, d, fmha_b200.VARIANT_LDG, None)
    assert st == 0, fmha_b200.status_string(st)
    torch.cuda.synchronize()
    want = ref.cpu().view(torch.int16).numpy().view(np.uint16)
    for call in range(2):
        O = torch.full((b * hq * d,), float("nan"), dtype=torch.float16, device=dev)
        st = lib.fmha_forward_noalloc(Q.data_ptr(), K.data_ptr(), V.data_ptr(), O.data_ptr(), b,
                                      hq, hkv, s, d, None)
        assert st == 0, f"call {call}: {fmha_b200.status_string(st)}"
        torch.cuda.synchronize()
        _close(O.cpu().view(torch.int16).numpy().view(np.uint16), want)
    assert fmha_b200.device_error() == 0
