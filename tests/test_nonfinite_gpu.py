"""Non-finite inputs: NaN and +/-inf in Q, K or V propagate exactly where the
reference's math (restated by the oracle, fmha_host.cpp:179-243: fmaxf max,
expf, divide) puts NaN/inf; all other elements stay within tolerance."""
import numpy as np
import pytest

import fmha_b200
from tests.test_parity_gpu import ATOL, RTOL, run_kernel
from tests.test_varlen_gpu import run_varlen

pytestmark = pytest.mark.gpu

NAN, PINF, NINF = 0x7FC0, 0x7F80, 0xFF80  # bf16 bit patterns


def poison(oracle, q, k, v, b, hq, hkv, s, d):
    q, k, v = q.copy(), k.copy(), v.copy()
    K = k.reshape(b, hkv, s, d)
    V = v.reshape(b, hkv, s, d)
    Q = q.reshape(b, hq, d)
    K[0, 0, s - 1, 3] = NAN           # a NaN score
    V[1, 0, 0, 7] = PINF              # inf in one value column
    Q[2, 0, :] = 0                    # zero query ...
    K[2, 0, :, 0] = NINF              # ... times -inf: 0 * -inf = NaN
    K[3, 0, :, :] = 0
    K[3, 0, 0, 0] = PINF              # +inf score beside finite ones
    Q[3, 0, 0] = 0x3F80               # q[0] = 1
    K[4, 0, :, :] = 0
    K[4, 0, :, 1] = NINF              # every score -inf
    Q[4, 0, 1] = 0x3F80
    return q, k, v


def compare(out_bits, ref32):
    o = out_bits.view(np.float16).astype(np.float32)
    assert np.array_equal(np.isnan(o), np.isnan(ref32))
    fin = np.isfinite(ref32)
    assert np.array_equal(np.isinf(o), np.isinf(ref32) & ~np.isnan(ref32))
    assert np.array_equal(o[np.isinf(o)], ref32[np.isinf(o)])
    err = np.abs(o[fin] - ref32[fin])
    assert np.all((err <= ATOL) | (err <= RTOL * np.abs(ref32[fin])))
    assert np.isnan(o).any()


@pytest.mark.parametrize("variant", ["bulk", "ldg"])
@pytest.mark.parametrize("s,d", [(16, 256), (5, 128), (16, 128), (2, 256)])
def test_nonfinite_dense(cuda, oracle, variant, s, d):
    b, hq, hkv = 6, 16, 16
    q, k, v = oracle.make_inputs_bhsd(b, hq, hkv, s, d, seed=11)
    q, k, v = poison(oracle, q, k, v, b, hq, hkv, s, d)
    with np.errstate(all="ignore"):
        ref32, _ = oracle.decode_bhsd(q, k, v, b, hq, hkv, s, d)
    compare(run_kernel(cuda, q, k, v, b, hq, hkv, s, d, variant=variant), ref32)


def test_nonfinite_varlen(cuda, oracle):
    b, h, s, d = 6, 16, 4, 256
    q, k, v = oracle.make_inputs_bhsd(b, h, h, s, d, seed=12)
    q, k, v = poison(oracle, q, k, v, b, h, h, s, d)
    packed = lambda x: np.ascontiguousarray(x.reshape(b, h, s, d).transpose(0, 2, 1, 3)).reshape(-1)  # noqa
    out, err, cu = run_varlen(cuda, q, packed(k), packed(v), np.full(b, s, np.int32), b, h, h, d)
    assert err == 0
    ref32, _ = oracle.decode_thd(q, packed(k), packed(v), cu, b, h, h, d)
    compare(out, ref32)
