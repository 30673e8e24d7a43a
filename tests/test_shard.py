"""Column-sharded GEMMs across ranks (hotarubi_b200.shard), as child
processes launched with torch.distributed.run on 127.0.0.1.

CPU: two gloo ranks gather oracle-computed column slices (host logic of the
sharded path: column split, exchange order, slice interleave).
GPU: two NCCL ranks on two GPUs (skipped with fewer) run column-sharded
GEMMs whose epilogues store into every rank's C over NVLink.
"""
import os
import socket
import subprocess
import sys

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
WORKER = os.path.join(ROOT, "tests", "shard_worker.py")


def free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def launch(mode: str, nproc: int, timeout: int) -> subprocess.CompletedProcess:
    env = dict(os.environ, NCCL_NVLS_ENABLE="0", OMP_NUM_THREADS="1")
    cmd = [sys.executable, "-m", "torch.distributed.run", "--nnodes=1",
           f"--nproc-per-node={nproc}", "--master-addr=127.0.0.1",
           f"--master-port={free_port()}", WORKER, "--mode", mode]
    return subprocess.run(cmd, capture_output=True, text=True, timeout=timeout, env=env)


def test_gloo_ranks_gather_column_slices():
    pytest.importorskip("torch")
    from oracle import cpu
    if cpu.oracle() is None:
        pytest.skip("oracle not built")
    r = launch("cpu", 2, 240)
    assert r.returncode == 0, r.stdout[-2000:] + r.stderr[-4000:]


@pytest.mark.gpu
def test_two_gpus_fused_all_gather():
    torch = pytest.importorskip("torch")
    if torch.cuda.device_count() < 2:
        pytest.skip("needs two GPUs")
    r = launch("gpu", 2, 400)
    assert r.returncode == 0, r.stdout[-2000:] + r.stderr[-4000:]


@pytest.mark.gpu
def test_cpp_host_shards_on_two_gpus():
    """The C++ host side with no framework (tests/cpp/test_shard_host.cpp):
    forked ranks, communicator bootstrap through pipes, a column-sharded GEMM
    and a row-sharded convolution with the all-gather fused into their
    epilogues, and the communicator's all-gather, each bit for bit with the
    unsharded result."""
    torch = pytest.importorskip("torch")
    if torch.cuda.device_count() < 2:
        pytest.skip("needs two GPUs")
    exe = os.path.join(ROOT, "tests", "cpp", "_build", "test_shard_host")
    if not os.path.exists(exe):
        pytest.skip("tests/cpp not built")
    env = dict(os.environ, NCCL_NVLS_ENABLE="0")
    r = subprocess.run([exe, "2"], capture_output=True, text=True, timeout=300, env=env)
    assert r.returncode == 0, r.stdout[-2000:] + r.stderr[-4000:]
