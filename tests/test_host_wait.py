"""CPU test of the C++ benchmark host's bounded wait (fmha_b200/csrc/host_wait.hpp):
a shard whose event never completes returns after the deadline and releases
none of its device resources, so the thread cannot block behind stuck
kernels in cudaFree. Compiled with g++, no GPU or CUDA runtime needed."""
import os
import shutil
import subprocess

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def test_host_wait_policy(tmp_path):
    gxx = shutil.which("g++")
    if gxx is None:
        pytest.skip("g++ absent")
    exe = tmp_path / "host_wait_test"
    subprocess.check_call([gxx, "-std=c++17", "-O1", "-pthread",
                           "-I" + os.path.join(ROOT, "fmha_b200", "csrc"),
                           os.path.join(ROOT, "tests", "cpp", "host_wait_test.cpp"), "-o", str(exe)])
    r = subprocess.run([str(exe)], capture_output=True, text=True, timeout=60)
    assert r.returncode == 0, r.stdout + r.stderr
    assert "host_wait_test: ok" in r.stdout
