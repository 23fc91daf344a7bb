"""The device restatements of libm's expf, tanhf (through expm1f) and the graph
executor's fused Gelu (executor.cpp:232-242) in leaf_b200/csrc/libm_math.cuh,
compiled as host code (tests/host_math_check.cpp) and compared bit for bit
with this machine's libm over an evenly strided sample of all float bit
patterns (every 257th: all binades, both signs, infinities and NaNs).  The
GPU tests check the same functions as compiled for sm_100a inside the
kernels."""
import shutil
import subprocess
from pathlib import Path

import pytest

HERE = Path(__file__).resolve().parent


@pytest.mark.skipif(shutil.which("g++") is None, reason="no host C++ compiler")
def test_libm_restatements_match_host_libm(tmp_path):
    exe = tmp_path / "host_math_check"
    subprocess.run(["g++", "-std=c++17", "-O2", "-ffp-contract=off", "-fno-fast-math", "-o", str(exe),
                    str(HERE / "host_math_check.cpp"), "-lm"], check=True)
    out = subprocess.run([str(exe), "257"], check=True, capture_output=True, text=True).stdout.split()
    count, bad_exp, bad_tanh, bad_gelu = (int(v) for v in out)
    assert count > 16_000_000
    assert (bad_exp, bad_tanh, bad_gelu) == (0, 0, 0)
