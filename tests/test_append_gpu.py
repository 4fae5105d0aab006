"""fmha_forward_append: the fused KV-cache append + attend. The new rows land
in the cache at position seqlen-1 (nothing else changes) and the output
matches the oracle on the updated cache prefix."""
import numpy as np
import pytest

import fmha_b200
from tests.test_parity_gpu import check_close, to_dev

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize("b,hq,hkv,s,smax,d", [(7, 16, 16, 1, 4, 128), (9, 32, 16, 5, 16, 256),
                                               (33, 16, 16, 16, 16, 128), (5, 8, 1, 12, 20, 256),
                                               (64, 32, 32, 9, 32, 256)])
def test_append_then_attend(cuda, oracle, b, hq, hkv, s, smax, d):
    lib = fmha_b200.load()
    q = oracle.gen_bf16(b * hq * d, 5, 1)
    kc = oracle.gen_bf16(b * hkv * smax * d, 5, 2)
    vc = oracle.gen_bf16(b * hkv * smax * d, 5, 3)
    kn = oracle.gen_bf16(b * hkv * d, 5, 4)
    vn = oracle.gen_bf16(b * hkv * d, 5, 5)
    Q, KC, VC, KN, VN = (to_dev(cuda, x) for x in (q, kc, vc, kn, vn))
    O = cuda.empty(b * hq * d, dtype=cuda.int16, device="cuda")
    st = lib.fmha_forward_append(Q.data_ptr(), KC.data_ptr(), VC.data_ptr(), KN.data_ptr(),
                                 VN.data_ptr(), O.data_ptr(), b, hq, hkv, s, smax, d, None)
    assert st == 0, fmha_b200.status_string(st)
    cuda.cuda.synchronize()
    assert fmha_b200.device_error() == 0
    ek, ev = kc.reshape(b, hkv, smax, d).copy(), vc.reshape(b, hkv, smax, d).copy()
    ek[:, :, s - 1] = kn.reshape(b, hkv, d)
    ev[:, :, s - 1] = vn.reshape(b, hkv, d)
    assert np.array_equal(KC.cpu().numpy().view(np.uint16).reshape(ek.shape), ek)
    assert np.array_equal(VC.cpu().numpy().view(np.uint16).reshape(ev.shape), ev)
    kp = np.ascontiguousarray(ek[:, :, :s]).reshape(-1)
    vp = np.ascontiguousarray(ev[:, :, :s]).reshape(-1)
    ref32, _ = oracle.decode_bhsd(q, kp, vp, b, hq, hkv, s, d)
    check_close(O.cpu().numpy().view(np.uint16), ref32)


def test_append_rejects_short_cache():
    lib = fmha_b200.load()
    assert lib.fmha_forward_append(16, 32, 48, 64, 80, 96, 2, 16, 16, 9, 8, 128, None) == \
        fmha_b200.FMHA_ERR_INVALID_ARG
