"""The reference's own call site compiles and runs unchanged against
include/fmha_compat.hpp (launch_fmha_mfma_4x4x4 -> fmha_forward_varlen), and
its output equals the direct C-ABI call bit for bit."""
import os
import shutil
import subprocess

import pytest

pytestmark = pytest.mark.gpu
ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def test_reference_call_site_through_compat_header(cuda, tmp_path):
    nvcc = shutil.which("nvcc") or "/usr/local/cuda/bin/nvcc"
    exe = str(tmp_path / "compat_call")
    subprocess.check_call([nvcc, "-std=c++17", "-I" + os.path.join(ROOT, "include"),
                           os.path.join(ROOT, "tests", "cpp", "compat_call.cpp"), "-o", exe,
                           "-L" + os.path.join(ROOT, "fmha_b200"), "-lfmha_b200",
                           "-Xlinker", "-rpath=" + os.path.join(ROOT, "fmha_b200")])
    r = subprocess.run([exe], capture_output=True, text=True, timeout=120)
    assert r.returncode == 0, r.stdout + r.stderr
