"""The C++ mirror of the ISS GEMM interface (hotarubi_b200/host/).

CPU: invalid commands print the reference's Require message and abort,
as gemm_array_test.cpp:201-215 expects of ExecuteGemm (no GPU touched).
GPU: random commands through the mirror's ExecuteGemm match the C
restatement of ExecuteGemm bit for bit, and its access log matches the
reference's address formulas (tests/cpp/test_iss_gemm.cpp).
"""
import os
import subprocess

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
BIN = os.path.join(ROOT, "tests", "cpp", "_build", "test_iss_gemm")


@pytest.fixture(scope="module")
def binary():
    from hotarubi_b200 import build
    try:
        build.build_host()
        subprocess.run(["make", "-s", "-C", os.path.join(ROOT, "tests", "cpp")], check=True,
                       capture_output=True)
    except (RuntimeError, subprocess.CalledProcessError) as e:
        pytest.skip(f"cannot build the C++ test program: {e}")
    return BIN


@pytest.mark.parametrize("case,message", [
    ("m", "error: GEMM m = 40 is not a multiple of 32 from 32 to 992"),
    ("kb", "error: GEMM kb = 5 is not in [1, a_stride = 4]"),
    ("n8", "error: GEMM n8 = 0"),
])
def test_invalid_commands_abort_with_the_reference_message(binary, case, message):
    r = subprocess.run([binary, "--death", case], capture_output=True, text=True, timeout=60)
    assert r.returncode != 0
    assert r.returncode == -6 or r.returncode == 134  # SIGABRT
    assert message in r.stderr


@pytest.mark.gpu
def test_mirror_matches_the_oracle_on_random_commands(binary):
    r = subprocess.run([binary, "--parity"], capture_output=True, text=True, timeout=300)
    assert r.returncode == 0, r.stdout + r.stderr
    assert "0 of 40 commands differ" in r.stdout
