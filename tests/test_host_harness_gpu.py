"""The C++ benchmark/validation host (fmha_b200/bin/fmha_host) on a GPU: the
reference's "testing" config and a GQA config validate on the CPU and report
sane metrics."""
import json
import os
import subprocess

import pytest

pytestmark = pytest.mark.gpu

BIN = os.path.join(os.path.dirname(os.path.dirname(os.path.abspath(__file__))), "fmha_b200", "bin",
                   "fmha_host")


@pytest.mark.parametrize("args", [["0"], ["5", "--seqlen", "7", "--validate-rows", "16"],
                                  ["0", "--variant", "bulk", "--seqlen", "1"],
                                  ["0", "--varlen"], ["4", "--varlen", "--validate-rows", "16"],
                                  ["5", "--varlen", "--validate-rows", "16"]])
def test_fmha_host_validates(cuda, args):
    if not os.path.exists(BIN):
        pytest.fail("fmha_host was not built (python -m fmha_b200.build)")
    r = subprocess.run([BIN] + args + ["--json", "--iters", "5"], capture_output=True, text=True,
                       timeout=600)
    assert r.returncode == 0, r.stderr
    line = json.loads(r.stdout.strip().splitlines()[-1])
    assert line["passed"] and line["bad"] == 0 and line["device_error"] == 0
    assert line["us_per_call"] > 0 and line["gbs"] > 0
    assert line["max_abs_err"] <= 2e-3 or line["max_rel_err"] <= 1e-2


def test_fmha_host_reports_a_failed_shard(cuda):
    """Host-side fault injection: the shard on GPU 0 fails before launching
    anything; the driver reports it (and, with more GPUs, the others still
    finish) and exits non-zero instead of crashing or hanging."""
    env = dict(os.environ, FMHA_HOST_FAIL_SHARD="0")
    r = subprocess.run([BIN, "0", "--json", "--iters", "3"], capture_output=True, text=True,
                       timeout=300, env=env)
    assert r.returncode != 0
    assert "shard on GPU 0 failed: injected failure" in r.stderr
    line = json.loads(r.stdout.strip().splitlines()[-1])
    assert not line["passed"] and line["failed_shards"].startswith("0: injected failure")


def test_fmha_host_stuck_shard_returns_without_blocking(cuda):
    """The timed wait of shard 0 sees an event query stub that never
    completes (FMHA_HOST_STUCK_SHARD, a host-side hook: no kernel is stuck).
    After its 2 s deadline the shard reports the timeout and returns without
    freeing its buffers, and the driver exits non-zero promptly."""
    env = dict(os.environ, FMHA_HOST_STUCK_SHARD="0")
    r = subprocess.run([BIN, "0", "--json", "--iters", "3"], capture_output=True, text=True,
                       timeout=300, env=env)
    assert r.returncode != 0
    assert "shard on GPU 0 failed: timed out" in r.stderr


def test_fmha_host_reports_measured_traffic(cuda):
    """--traffic reads the committed ncu table and adds the DRAM bytes ncu
    measured for the config (scaled to its batch) and the bandwidth they give."""
    table = os.path.join(os.path.dirname(BIN), "..", "..", "profiles", "ncu_traffic.json")
    r = subprocess.run([BIN, "4", "--json", "--iters", "3", "--validate-rows", "8", "--traffic",
                        table], capture_output=True, text=True, timeout=600)
    assert r.returncode == 0, r.stderr
    line = json.loads(r.stdout.strip().splitlines()[-1])
    assert line["ncu_dram_bytes"] > 0.9 * 17.11e9
    assert 0.8 * line["gbs"] < line["ncu_gbs"] <= 1.01 * line["gbs"]
