"""CPU-only checks of the C ABI library: it loads, exports every function the
header declares, and its host-only helpers (instruction decode, argument
checks, access log) agree with the reference.  No compute call needs a GPU
here."""
import ctypes
import os
import subprocess

import numpy as np
import pytest

from hotarubi_b200 import capi
from oracle import cpu

FIELDS = ("a_base", "a_stride", "kb", "m", "w_base", "w_stride", "n8", "c_base", "wmode",
          "acc")


@pytest.fixture(scope="module")
def lib():
    if not os.path.exists(capi.LIB_PATH):
        from hotarubi_b200 import build
        build.build()
    return capi.load()


def cmd_of(values):
    c = capi.GemmCmd()
    for name, v in zip(FIELDS, values):
        setattr(c, name, int(v))
    return c


def test_library_exports_every_declared_function(lib):
    names = capi.header_functions()
    assert len(names) >= 20
    out = subprocess.run(["nm", "-D", "--defined-only", capi.LIB_PATH], capture_output=True,
                         text=True, check=True).stdout
    exported = {line.split()[-1] for line in out.splitlines() if " T " in line}
    missing = [n for n in names if n not in exported]
    assert not missing, missing
    for n in names:
        assert hasattr(lib, n)


def test_build_targets_sm100a_only():
    from hotarubi_b200 import build
    assert build.ARCH == ["-gencode", "arch=compute_100a,code=sm_100a"]


def encode_gemm(f) -> bytes:
    """EncodeGemm (tools/compiler/isa.cpp:89-103) restated for the test:
    opcode 4 in bits 127:120, fields at isa.hpp:77-86."""
    word = 4 << 120
    for (lsb, width), v in zip(((92, 20), (82, 10), (72, 10), (62, 10), (42, 20), (32, 10),
                                (24, 8), (4, 20), (2, 2), (1, 1)), f):
        assert v < (1 << width)
        word |= v << lsb
    return word.to_bytes(16, "little")


def test_decode_matches_the_isa_field_map(lib):
    rng = np.random.default_rng(1)
    for _ in range(200):
        f = [int(rng.integers(0, 1 << w)) for w in (20, 10, 10, 10, 20, 10, 8, 20, 2, 1)]
        c = capi.gemm_decode(encode_gemm(f))
        assert [getattr(c, n) for n in FIELDS] == f


def test_check_mirrors_execute_gemm_requires(lib):
    assert capi.gemm_check(cmd_of([0, 1, 1, 32, 0, 1, 1, 0, 0, 0]))[0] == capi.HRB_OK
    for bad in ([0, 1, 1, 16, 0, 1, 1, 0, 0, 0], [0, 1, 1, 1024, 0, 1, 1, 0, 0, 0],
                [0, 1, 1, 40, 0, 1, 1, 0, 0, 0], [0, 1, 0, 32, 0, 1, 1, 0, 0, 0],
                [0, 1, 2, 32, 0, 1, 1, 0, 0, 0], [0, 1, 1, 32, 0, 1, 0, 0, 0, 0]):
        assert capi.gemm_check(cmd_of(bad))[0] == capi.HRB_EINVAL


def test_accesses_match_the_iss_log(lib, ref_lib):
    rng = np.random.default_rng(2)
    abuf = np.zeros((8192, 132), np.uint8)
    wbuf = np.zeros((2048, 144), np.uint8)
    fbuf = np.zeros((4096, 32), np.uint32)
    for t in range(20):
        kb = int(rng.integers(1, 30))
        f = [int(rng.integers(0, 1 << 20)), kb + int(rng.integers(0, 4)), kb,
             int(rng.integers(1, 31)) * 32, int(rng.integers(0, 1 << 20)),
             int(rng.integers(1, 40)), int(rng.integers(1, 256)), int(rng.integers(0, 1 << 20)),
             t % 4, t % 2]
        log = np.zeros(8192 + 2048 + 4096 + 4096, np.uint8)
        ref_lib.hrbref_execute_gemm(np.array(f, np.uint32), abuf.reshape(-1),
                                    wbuf.reshape(-1), fbuf.reshape(-1), log.ctypes.data)
        a, w, fr, fw = capi.gemm_accesses(cmd_of(f))
        assert (a == log[:8192]).all()
        assert (w == log[8192:10240]).all()
        assert (fr == log[10240:14336]).all()
        assert (fw == log[14336:]).all()


def test_accesses_on_golden_cases(lib, golden):
    case = golden("iss_unit.npz")
    for name in case["names"]:
        a, w, fr, fw = capi.gemm_accesses(cmd_of(case[f"{name}/cmd"]))
        assert (np.flatnonzero(a) == case[f"{name}/a_idx"]).all()
        assert (np.flatnonzero(w) == case[f"{name}/w_idx"]).all()
        assert (np.flatnonzero(fw) == case[f"{name}/c_idx"]).all()
        assert (np.flatnonzero(fr) == case[f"{name}/log_fbuf_read"]).all()


def test_create_without_a_device_fails_cleanly(lib):
    import torch
    if torch.cuda.is_available():
        pytest.skip("a device is present")
    h = ctypes.c_void_p()
    assert lib.hrb_create(0, ctypes.byref(h)) == capi.HRB_EINVAL
    assert not h.value


def test_workload_canonicalisation_matches_the_reference_restatement():
    from hotarubi_b200 import workloads
    rng = np.random.default_rng(3)
    code = rng.integers(0, 16, (40, 256)).astype(np.uint8)
    e = rng.integers(-10, -3, (40, 8))
    a = workloads.canonical_mxfp4(code, e)
    b = cpu.canonical_mxfp4(code, e)
    assert (a[0] == b[0]).all() and (a[1] == b[1]).all()


def test_ctypes_structs_match_the_header(tmp_path):
    """The ctypes mirrors of hrb_gemm_desc, hrb_conv_desc, hrb_gemm_cmd and hrb_ipc_handle
    have the C layout: a C program built against include/hrb_gemm.h prints
    every field's offset and the sizes."""
    import ctypes
    import shutil
    import subprocess

    from hotarubi_b200 import capi
    cc = shutil.which("gcc") or shutil.which("cc")
    if cc is None:
        pytest.skip("no C compiler")
    structs = {"hrb_gemm_desc": capi.GemmDesc, "hrb_gemm_cmd": capi.GemmCmd,
               "hrb_ipc_handle": capi.IpcHandle, "hrb_conv_desc": capi.ConvDesc,
               "hrb_gacc_desc": capi.GaccDesc}
    lines = ["#include <stddef.h>", "#include <stdio.h>", '#include "hrb_gemm.h"',
             "int main(void) {"]
    for cname, py in structs.items():
        lines.append(f'  printf("{cname} size %zu\\n", sizeof({cname}));')
        for f in py._fields_:
            lines.append(f'  printf("{cname} {f[0]} %zu\\n", offsetof({cname}, {f[0]}));')
    lines += ["  return 0;", "}"]
    src = tmp_path / "layout.c"
    src.write_text("\n".join(lines) + "\n")
    exe = tmp_path / "layout"
    include = os.path.join(os.path.dirname(os.path.dirname(os.path.abspath(__file__))), "include")
    subprocess.run([cc, "-I", include, str(src), "-o", str(exe)], check=True)
    out = subprocess.run([str(exe)], capture_output=True, text=True, check=True).stdout.split("\n")
    for line in filter(None, out):
        cname, field, value = line.split()
        py = structs[cname]
        got = ctypes.sizeof(py) if field == "size" else getattr(py, field).offset
        assert got == int(value), (cname, field, got, value)
