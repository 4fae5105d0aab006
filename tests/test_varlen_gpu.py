"""fmha_forward_varlen (the reference's packed K/V layout [sum S_b, Hkv, D] +
cu_seqlens_kv, fmha_host.cpp:143-157) against the oracle's packed-layout
restatement, the reference's own golden output and its Poisson(4) seqlens
(fmha_host.cpp:58-72). Every parity test runs both varlen kernels, selected
per call through fmha_forward_varlen_variant: the chunk ring (the default) and
the register-prefetch kernel."""
import glob
import os

import numpy as np
import pytest

import fmha_b200
from tests.test_parity_gpu import GUARD, POISON, check_close, to_dev

pytestmark = pytest.mark.gpu

KERNELS = ["chunk", "ldg"]


def seqlens(oracle, b, kind, rng):
    if kind == "poisson":
        if oracle.ref_available():
            return oracle.ref_generate_seqlens(b, 16)
        x = rng.poisson(4, size=4 * b + 64)
        return x[(x >= 2) & (x <= 16)][:b].astype(np.int32)
    if kind == "edge":
        return np.array([(0, 1, 16, 2, 15, 3, 8, 9, 4, 5, 7, 6, 10, 11, 12, 13, 14)[i % 17]
                         for i in range(b)], dtype=np.int32)
    return np.full(b, int(kind), dtype=np.int32)


def run_varlen(cuda, q, k, v, sl, b, hq, hkv, d, max_s=16, scale=0.0, kernel="chunk"):
    cu = np.concatenate([[0], np.cumsum(sl)]).astype(np.int32)
    n = b * hq * d
    Q, K, V = to_dev(cuda, q), to_dev(cuda, k), to_dev(cuda, v)
    CU = cuda.from_numpy(cu).cuda()
    buf = cuda.full((n + 2 * GUARD,), POISON, dtype=cuda.int16, device="cuda")
    O = buf[GUARD:GUARD + n]
    st = fmha_b200.fmha_forward_varlen_ptr(Q, K, V, O, CU, b, hq, hkv, max_s, d, scale, 0,
                                           kernel=kernel)
    assert st == 0, fmha_b200.status_string(st)
    cuda.cuda.synchronize()
    err = fmha_b200.device_error()
    out = buf.cpu().numpy().view(np.uint16)
    assert np.all(out[:GUARD] == POISON) and np.all(out[GUARD + n:] == POISON)
    return out[GUARD:GUARD + n].copy(), err, cu


CASES = [(b, hq, hkv, d, kind) for d in (128, 256) for (b, hq, hkv) in ((37, 16, 16), (20, 32, 32),
                                                                       (9, 32, 16), (6, 8, 1))
         for kind in ("poisson", "edge", "1", "3", "16")]


@pytest.mark.parametrize("kernel", KERNELS)
@pytest.mark.parametrize("b,hq,hkv,d,kind", CASES, ids=str)
def test_varlen_vs_oracle(cuda, oracle, b, hq, hkv, d, kind, kernel):
    rng = np.random.default_rng(b * 7 + d)
    sl = seqlens(oracle, b, kind, rng)
    t = int(sl.sum())
    q = oracle.gen_bf16(b * hq * d, 31, 1)
    k = oracle.gen_bf16(t * hkv * d, 31, 2)
    v = oracle.gen_bf16(t * hkv * d, 31, 3)
    out, err, cu = run_varlen(cuda, q, k, v, sl, b, hq, hkv, d, kernel=kernel)
    assert err == 0
    ref32, _ = oracle.decode_thd(q, k, v, cu, b, hq, hkv, d)
    check_close(out, ref32)


GOLDEN = sorted(glob.glob(os.path.join(os.path.dirname(__file__), "golden", "thd_*.npz")))


@pytest.mark.parametrize("kernel", KERNELS)
@pytest.mark.parametrize("path", GOLDEN, ids=os.path.basename)
def test_varlen_vs_reference_golden(cuda, oracle, path, kernel):
    """The reference's own output on its own layout and seqlens, under its
    own tolerance (fmha_host.cpp:260)."""
    f = np.load(path)
    b, h, d, seed = (int(f[x]) for x in ("batch", "heads", "head_dim", "seed"))
    sl = f["seqlens"].astype(np.int32)
    t = int(sl.sum())
    q = oracle.gen_bf16(b * h * d, seed, 1)
    k = oracle.gen_bf16(t * h * d, seed, 2)
    v = oracle.gen_bf16(t * h * d, seed, 3)
    out, err, _ = run_varlen(cuda, q, k, v, sl, b, h, h, d, kernel=kernel)
    assert err == 0
    o = out.view(np.float16).astype(np.float32)
    r = f["ref_o"].view(np.float16).astype(np.float32)
    assert np.all(np.abs(o - r) <= 1e-2 + 1e-2 * np.abs(r))


@pytest.mark.parametrize("kernel", KERNELS)
def test_varlen_uniform_matches_dense(cuda, oracle, kernel):
    b, h, s, d = 64, 16, 5, 256
    q, k, v = oracle.make_inputs_bhsd(b, h, h, s, d, seed=8)
    packed = lambda x: np.ascontiguousarray(x.reshape(b, h, s, d).transpose(0, 2, 1, 3)).reshape(-1)  # noqa
    out, err, _ = run_varlen(cuda, q, packed(k), packed(v), np.full(b, s, np.int32), b, h, h, d,
                             kernel=kernel)
    assert err == 0
    from tests.test_parity_gpu import run_kernel
    dense = run_kernel(cuda, q, k, v, b, h, h, s, d)
    a = out.view(np.float16).astype(np.float32)
    c = dense.view(np.float16).astype(np.float32)
    assert np.abs(a - c).max() <= 2e-3


@pytest.mark.parametrize("kernel", KERNELS)
def test_varlen_explicit_scale(cuda, oracle, kernel):
    b, h, d = 5, 16, 128
    sl = np.array([4, 4, 4, 4, 4], np.int32)
    q = oracle.gen_bf16(b * h * d, 3, 1)
    k = oracle.gen_bf16(20 * h * d, 3, 2)
    v = oracle.gen_bf16(20 * h * d, 3, 3)
    a, _, _ = run_varlen(cuda, q, k, v, sl, b, h, h, d, scale=0.0, kernel=kernel)
    c, _, _ = run_varlen(cuda, q, k, v, sl, b, h, h, d, scale=1.0 / np.sqrt(d), kernel=kernel)
    assert np.array_equal(a, c)
    e, _, _ = run_varlen(cuda, q, k, v, sl, b, h, h, d, scale=0.5, kernel=kernel)
    assert not np.array_equal(a, e)


@pytest.mark.parametrize("kernel", KERNELS)
def test_varlen_rejects_long_row_on_device(cuda, oracle, kernel):
    """A row longer than max_seqlen_kv is skipped and flagged in the device
    error word; the other rows are still computed."""
    b, h, d = 4, 16, 128
    sl = np.array([3, 9, 2, 5], np.int32)
    t = int(sl.sum())
    q = oracle.gen_bf16(b * h * d, 4, 1)
    k = oracle.gen_bf16(t * h * d, 4, 2)
    v = oracle.gen_bf16(t * h * d, 4, 3)
    out, err, cu = run_varlen(cuda, q, k, v, sl, b, h, h, d, max_s=8, kernel=kernel)
    assert err & 0xff == fmha_b200.FMHA_ERR_INVALID_ARG and (err >> 8) == 5
    ref32, _ = oracle.decode_thd(q, k, v, cu, b, h, h, d)
    n = h * d
    for r in (0, 2, 3):
        check_close(out[r * n:(r + 1) * n], ref32[r * n:(r + 1) * n])
    assert np.all(out[n:2 * n] == POISON)


@pytest.mark.slow
@pytest.mark.parametrize("kernel", KERNELS)
@pytest.mark.parametrize("hq,d", [(16, 128), (32, 256)])
def test_varlen_full_size_reference_seqlens(cuda, oracle, hq, d, kernel):
    """batch 30720 with the reference's own Poisson seqlens, inputs generated
    on the device: every row against the oracle."""
    B = 30720
    sl = seqlens(oracle, B, "poisson", np.random.default_rng(0))
    cu = np.concatenate([[0], np.cumsum(sl)]).astype(np.int32)
    t = int(cu[-1])
    Q = cuda.empty(B * hq * d, dtype=cuda.bfloat16, device="cuda")
    K = cuda.empty(t * hq * d, dtype=cuda.bfloat16, device="cuda")
    V = cuda.empty_like(K)
    for x, tid in ((Q, 1), (K, 2), (V, 3)):
        fmha_b200.fill_normal_bf16(x, seed=0, tensor_id=tid)
    O = cuda.empty(B * hq * d, dtype=cuda.float16, device="cuda")
    CU = cuda.from_numpy(cu).cuda()
    assert fmha_b200.fmha_forward_varlen_ptr(Q, K, V, O, CU, B, hq, hq, 16, d, 0.0, 0,
                                             kernel=kernel) == 0
    cuda.cuda.synchronize()
    assert fmha_b200.device_error() == 0
    oracle.set_threads(os.cpu_count() or 1)
    bits = lambda x: x.cpu().view(cuda.int16).numpy().view(np.uint16)  # noqa: E731
    ref32, _ = oracle.decode_thd(bits(Q), bits(K), bits(V), cu, B, hq, hq, d)
    check_close(bits(O), ref32)


PLAN_CASES = [  # (hq, hkv, d, chunk byte limit or 0 for the default, max_seqlen_kv)
    (16, 16, 128, 0, 16),
    (16, 16, 128, 20480, 16),   # most rows split into head groups
    (32, 16, 256, 0, 16),       # GQA
    (32, 16, 256, 40960, 12),   # splits + rows longer than max_seqlen_kv mid-window
    (4, 4, 128, 0, 16),         # tiny rows: the 8-rows-per-chunk limit binds
    (8, 1, 128, 0, 16),         # one kv head: many chunks, descriptor slots recycle fast
]


@pytest.mark.parametrize("kernel", KERNELS)
@pytest.mark.parametrize("hq,hkv,d,chunk,max_s", PLAN_CASES, ids=str)
def test_varlen_chunk_planning_all_rows(cuda, oracle, monkeypatch, hq, hkv, d, chunk, max_s,
                                        kernel):
    """Enough rows that every CTA plans several 32-row windows, packs rows into
    chunks and wraps its ring many times; lengths mix Poisson(4) with 0, 1,
    16 and (when max_seqlen_kv < 16) rows that must be flagged and skipped.
    Every row is checked against the oracle."""
    if chunk:
        monkeypatch.setenv("FMHA_VARLEN_CHUNK", str(chunk))
    b = 148 * (40 if d == 128 else 33)
    rng = np.random.default_rng(hq * 1000 + hkv * 10 + d + chunk)
    x = rng.poisson(4, size=4 * b)
    sl = x[(x >= 2) & (x <= 16)][:b].astype(np.int32)
    pos = rng.choice(b, size=b // 10, replace=False)
    sl[pos] = rng.choice(np.array([0, 1, 16, 16], np.int32), size=pos.size)
    t = int(sl.sum())
    q = oracle.gen_bf16(b * hq * d, 77, 1)
    k = oracle.gen_bf16(t * hkv * d, 77, 2)
    v = oracle.gen_bf16(t * hkv * d, 77, 3)
    out, err, cu = run_varlen(cuda, q, k, v, sl, b, hq, hkv, d, max_s=max_s, kernel=kernel)
    bad = sl > max_s
    if bad.any():
        assert err & 0xff == fmha_b200.FMHA_ERR_INVALID_ARG and (err >> 8) == 5
    else:
        assert err == 0
    ref32, _ = oracle.decode_thd(q, k, v, cu, b, hq, hkv, d)
    n = hq * d
    rows_ok = np.repeat(~bad, n)
    check_close(out[rows_ok], ref32[rows_ok])
    assert np.all(out[~rows_ok] == POISON)


@pytest.mark.parametrize("kernel", KERNELS)
def test_varlen_negative_lengths_cover_every_valid_row(cuda, oracle, kernel):
    """cu_seqlens that is not monotonic (a few negative lengths) makes the
    byte-balanced CTA ranges irregular; every valid row must still be
    computed (no gaps), invalid rows flagged and left untouched."""
    b, hq, hkv, d = 148 * 12, 16, 16, 128
    rng = np.random.default_rng(5)
    x = rng.poisson(4, size=4 * b)
    sl = x[(x >= 2) & (x <= 16)][:b].astype(np.int32)
    neg = rng.choice(np.arange(10, b), size=20, replace=False)
    sl[neg] = -3
    cu = np.concatenate([[0], np.cumsum(sl)]).astype(np.int32)
    assert cu.min() >= 0
    t = int(cu.max())
    q = oracle.gen_bf16(b * hq * d, 9, 1)
    k = oracle.gen_bf16(t * hkv * d, 9, 2)
    v = oracle.gen_bf16(t * hkv * d, 9, 3)
    n = b * hq * d
    Q, K, V = to_dev(cuda, q), to_dev(cuda, k), to_dev(cuda, v)
    CU = cuda.from_numpy(cu).cuda()
    buf = cuda.full((n + 2 * GUARD,), POISON, dtype=cuda.int16, device="cuda")
    st = fmha_b200.fmha_forward_varlen_ptr(Q, K, V, buf[GUARD:GUARD + n], CU, b, hq, hkv, 16, d,
                                           0.0, 0, kernel=kernel)
    assert st == 0
    cuda.cuda.synchronize()
    err = fmha_b200.device_error()
    assert err & 0xff == fmha_b200.FMHA_ERR_INVALID_ARG and (err >> 8) == 5
    out = buf.cpu().numpy().view(np.uint16)
    assert np.all(out[:GUARD] == POISON) and np.all(out[GUARD + n:] == POISON)
    out = out[GUARD:GUARD + n]
    m = hq * d
    kv_row = hkv * d
    for r in range(b):
        got = out[r * m:(r + 1) * m]
        if sl[r] < 0:
            assert np.all(got == POISON)
            continue
        c0, c1 = int(cu[r]), int(cu[r + 1])
        ref32, _ = oracle.decode_thd(q[r * m:(r + 1) * m], k[c0 * kv_row:c1 * kv_row],
                                     v[c0 * kv_row:c1 * kv_row], np.array([0, c1 - c0], np.int32),
                                     1, hq, hkv, d)
        check_close(got, ref32)
