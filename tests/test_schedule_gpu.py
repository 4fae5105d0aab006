"""The ldg family's dynamic tail (decode_common.cuh sched_join): warps take
~90 % of their steps statically and claim the rest from a per-launch schedule
word. These tests check that the tail never changes results: dynamic and fully
static schedules give the same bits, launches that contend for one word on
concurrent streams (FMHA_SCHED_SLOTS=1) stay correct, and launches captured in
a CUDA graph (static schedule) replay correctly."""
import numpy as np
import pytest

import fmha_b200
from tests.test_parity_gpu import check_close, to_dev

pytestmark = pytest.mark.gpu


def make(cuda, oracle, b, h, s, d, seed):
    q, k, v = oracle.make_inputs_bhsd(b, h, h, s, d, seed=seed)
    ref32, _ = oracle.decode_bhsd(q, k, v, b, h, h, s, d)
    return to_dev(cuda, q), to_dev(cuda, k), to_dev(cuda, v), ref32


@pytest.mark.parametrize("b,h,s,d", [(3840, 32, 16, 256), (1000, 16, 1, 128), (5, 32, 16, 256),
                                     (777, 16, 3, 256)])
def test_dynamic_tail_equals_static(cuda, oracle, monkeypatch, b, h, s, d):
    Q, K, V, ref32 = make(cuda, oracle, b, h, s, d, seed=11)
    outs = []
    for static in ("0", "1"):
        monkeypatch.setenv("FMHA_STATIC_SCHEDULE", static)
        O = cuda.empty(b * h * d, dtype=cuda.int16, device="cuda")
        for _ in range(3):  # repeated launches reuse schedule slots
            assert fmha_b200.fmha_forward_ptr(Q, K, V, O, b, h, h, s, d, stream=0,
                                              variant="ldg") == 0
        cuda.cuda.synchronize()
        assert fmha_b200.device_error() == 0
        outs.append(O.cpu().numpy().view(np.uint16))
    assert np.array_equal(outs[0], outs[1])
    check_close(outs[0], ref32)


def test_contended_schedule_word_stays_correct(cuda, oracle, monkeypatch):
    """One schedule slot for everything, launches on four streams at once:
    launches that find the word held by another run statically, the others
    share nothing they should not."""
    monkeypatch.setenv("FMHA_SCHED_SLOTS", "1")
    b, h, s, d = 2048, 32, 16, 256
    Q, K, V, ref32 = make(cuda, oracle, b, h, s, d, seed=12)
    streams = [cuda.cuda.Stream() for _ in range(4)]
    outs = [cuda.full((b * h * d,), 0x7BAD, dtype=cuda.int16, device="cuda") for _ in streams]
    cuda.cuda.synchronize()
    for rep in range(8):
        for st, O in zip(streams, outs):
            assert fmha_b200.fmha_forward_ptr(Q, K, V, O, b, h, h, s, d, stream=st.cuda_stream,
                                              variant="ldg") == 0
    cuda.cuda.synchronize()
    assert fmha_b200.device_error() == 0
    for O in outs:
        check_close(O.cpu().numpy().view(np.uint16), ref32)


def test_graph_captured_launch_replays(cuda, oracle):
    b, h, s, d = 1500, 32, 16, 256
    Q, K, V, ref32 = make(cuda, oracle, b, h, s, d, seed=13)
    O = cuda.empty(b * h * d, dtype=cuda.int16, device="cuda")
    st = cuda.cuda.Stream()
    # warm-up outside capture (first-call set-up queries must not be captured)
    with cuda.cuda.stream(st):
        assert fmha_b200.fmha_forward_ptr(Q, K, V, O, b, h, h, s, d, stream=st.cuda_stream,
                                          variant="ldg") == 0
    st.synchronize()
    g = cuda.cuda.CUDAGraph()
    with cuda.cuda.graph(g, stream=st):
        assert fmha_b200.fmha_forward_ptr(Q, K, V, O, b, h, h, s, d,
                                          stream=cuda.cuda.current_stream().cuda_stream,
                                          variant="ldg") == 0
    for _ in range(5):
        O.fill_(0x7BAD)
        g.replay()
        cuda.cuda.synchronize()
        check_close(O.cpu().numpy().view(np.uint16), ref32)
    assert fmha_b200.device_error() == 0
