"""GEMM instructions through hotarubi's own Machine (tools/iss/machine.cpp),
compiled from the reference checkout with the one-branch B200 drop-in in
ExecuteGemm (oracle/iss_gpu_gemm.patch, built into oracle/_ref/iss_machine
by oracle/Makefile).

The driver (oracle/iss_machine.cpp) runs a stream of raw DMA loads, FP4 and
W8 (HI then LO) GEMMs, an accumulating GEMM over preloaded FBUF words, a GEMM
whose ABUF addresses wrap, a DMA store and HALT, and prints how the machine
stopped, its hazards, digests of the stored words and of FBUF, and a digest
of every instruction's access log as the machine's observer sees it.

CPU: the harness builds and runs the reference's CPU body to HALT.
GPU: with HOTARUBI_GPU_GEMM=1 the same stream runs its GEMMs through
libhrb_gemm.so (a CUDA context is then active) and every printed line equals
the CPU body's: FBUF, the stored DDR words and the access logs bit for bit.
"""
import os
import subprocess

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
EXE = os.path.join(ROOT, "oracle", "_ref", "iss_machine")


def run(seed: int, gpu: bool) -> tuple[list[str], int]:
    env = dict(os.environ)
    env.pop("HOTARUBI_GPU_GEMM", None)
    if gpu:
        env["HOTARUBI_GPU_GEMM"] = "1"
    r = subprocess.run([EXE, str(seed)], capture_output=True, text=True, timeout=120, env=env)
    assert r.returncode == 0, r.stdout + r.stderr
    lines = r.stdout.splitlines()
    ctx = int(lines[-1].split()[1])
    return lines[:-1], ctx


def needs_harness():
    if not os.path.exists(EXE):
        pytest.skip("oracle/_ref/iss_machine not built (no reference checkout)")


@pytest.mark.parametrize("seed", [1, 2])
def test_reference_machine_runs_the_stream_to_halt(seed):
    needs_harness()
    lines, _ = run(seed, gpu=False)
    assert lines[0] == "stop 2"          # Stop::kHalt
    assert lines[1] == "hazards 0"
    assert sum(1 for s in lines if s.startswith("log ")) == 11


@pytest.mark.gpu
@pytest.mark.parametrize("seed", [1, 2, 3])
def test_machine_gemms_on_the_gpu_equal_the_cpu_body(seed):
    needs_harness()
    torch = pytest.importorskip("torch")
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    cpu_lines, cpu_ctx = run(seed, gpu=False)
    gpu_lines, gpu_ctx = run(seed, gpu=True)
    assert gpu_ctx == 1, "the GPU branch did not run"
    assert cpu_ctx != 1
    assert gpu_lines == cpu_lines
