"""Builds libhrb_gemm.so, the C-ABI library of the B200 GEMM backend.

    python -m hotarubi_b200.build        # or __graft_entry__.build()

Compiles every .cu file under csrc/ with nvcc for sm_100a only and links one
shared library into hotarubi_b200/lib/.  The CUDA runtime is linked
statically so that the library loads wherever the driver is present.
"""
from __future__ import annotations

import concurrent.futures
import hashlib
import os
import shutil
import subprocess
import sys

PKG = os.path.dirname(os.path.abspath(__file__))
CSRC = os.path.join(PKG, "csrc")
INCLUDE = os.path.join(os.path.dirname(PKG), "include")
LIBDIR = os.path.join(PKG, "lib")
OBJDIR = os.path.join(PKG, "_build")
LIB = os.path.join(LIBDIR, "libhrb_gemm.so")

ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]
NVCC_FLAGS = ARCH + ["-O3", "-lineinfo", "-std=c++17", "-Xcompiler", "-fPIC",
                     "-Xcompiler", "-fvisibility=hidden", "--expt-relaxed-constexpr",
                     "-Xptxas", "-warn-spills", "-I", INCLUDE, "-I", CSRC]


def nvcc() -> str:
    path = shutil.which("nvcc") or "/usr/local/cuda/bin/nvcc"
    if not os.path.exists(path):
        raise RuntimeError("nvcc not found")
    return path


def _key(cmd: list[str], files: list[str]) -> str:
    """What an output is built from: the command and the contents of its
    inputs (not their timestamps, which a clock step can make lie)."""
    h = hashlib.sha256("\0".join(cmd).encode())
    for f in files:
        with open(f, "rb") as fh:
            h.update(hashlib.sha256(fh.read()).digest())
    return h.hexdigest()


def _fresh(out: str, key: str) -> bool:
    try:
        with open(out + ".key") as fh:
            return os.path.exists(out) and fh.read() == key
    except OSError:
        return False


def _stamp(out: str, key: str) -> None:
    with open(out + ".key", "w") as fh:
        fh.write(key)


def _compile(src: str, verbose: bool) -> str:
    obj = os.path.join(OBJDIR, os.path.basename(src).replace(".cu", ".o"))
    deps = [src] + sorted(os.path.join(CSRC, f) for f in os.listdir(CSRC)
                          if f.endswith((".cuh", ".h"))) + [os.path.join(INCLUDE, "hrb_gemm.h")]
    cmd = [nvcc()] + NVCC_FLAGS + ["-c", src, "-o", obj]
    key = _key(cmd, deps)
    if _fresh(obj, key) and not verbose:
        return obj
    run = cmd[:-4] + (["-Xptxas", "-v"] if verbose else []) + cmd[-4:]
    r = subprocess.run(run, capture_output=True, text=True)
    if r.returncode != 0:
        raise RuntimeError(f"nvcc failed on {src}:\n{r.stdout}\n{r.stderr}")
    if verbose:
        sys.stderr.write(r.stderr)
    _stamp(obj, key)
    return obj


def build(verbose: bool = False) -> str:
    os.makedirs(LIBDIR, exist_ok=True)
    os.makedirs(OBJDIR, exist_ok=True)
    sources = sorted(os.path.join(CSRC, f) for f in os.listdir(CSRC) if f.endswith(".cu"))
    with concurrent.futures.ThreadPoolExecutor(max_workers=os.cpu_count() or 4) as pool:
        objs = list(pool.map(lambda s: _compile(s, verbose), sources))
    tmp = LIB + ".tmp"
    cmd = [nvcc()] + ARCH + ["-shared", "-cudart", "static", "-o", tmp] + objs + ["-ldl"]
    key = _key(cmd, objs)
    if _fresh(LIB, key):
        return LIB
    r = subprocess.run(cmd, capture_output=True, text=True)
    if r.returncode != 0:
        raise RuntimeError(f"link failed:\n{r.stdout}\n{r.stderr}")
    os.replace(tmp, LIB)
    _stamp(LIB, key)
    return LIB


HOST = os.path.join(PKG, "host")
HOST_LIB = os.path.join(LIBDIR, "libhrb_iss.so")


def build_host() -> str:
    """libhrb_iss.so: the C++ mirror of the ISS GEMM interface (host/),
    linked against libhrb_gemm.so (found next to it at run time)."""
    gemm = build()
    src = os.path.join(HOST, "gpu_gemm_array.cpp")
    deps = [src, os.path.join(HOST, "gpu_gemm_array.hpp"), os.path.join(INCLUDE, "hrb_gemm.h"), gemm]
    cxx = shutil.which("g++") or "c++"
    cmd = [cxx, "-std=c++20", "-O2", "-fPIC", "-shared", "-Wall", "-Wextra", "-I", INCLUDE,
           "-I", HOST, src, "-L", LIBDIR, "-lhrb_gemm", "-Wl,-rpath,$ORIGIN", "-o", HOST_LIB]
    key = _key(cmd, deps)
    if _fresh(HOST_LIB, key):
        return HOST_LIB
    r = subprocess.run(cmd, capture_output=True, text=True)
    if r.returncode != 0:
        raise RuntimeError(f"host library build failed:\n{r.stdout}\n{r.stderr}")
    _stamp(HOST_LIB, key)
    return HOST_LIB


if __name__ == "__main__":
    print(build(verbose="-v" in sys.argv))
    print(build_host())
