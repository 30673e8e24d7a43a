"""NPU-equivalent time: hrb_gemm_npu_cycles / hrb_dense_npu_cycles (the
library, no GPU needed) against the reference's cycle model,
CostModel::Gemm and GemmArrayCycles (tools/iss/timing.cpp:65-67,89-93),
compiled into oracle/_ref.
"""
import numpy as np
import pytest

from hotarubi_b200 import capi


def test_gemm_cost_known_answer():
    # CostModelTest.GemmCostIsTheArrayTimePlusTheFixedCost
    # (tools/iss/timing_test.cpp:76-94).
    fields = [0, 24, 24, 128, 0, 24, 32, 0, 0, 0]
    assert capi.npu_cycles(fields) == 32 * 4 * 24 * 8 + 51


def test_gemm_cycles_match_reference(ref_lib):
    rng = np.random.default_rng(4)
    for _ in range(200):
        kb = int(rng.integers(1, 1024))
        f = np.array([int(rng.integers(0, 8192)), kb, kb, 32 * int(rng.integers(1, 32)),
                      int(rng.integers(0, 2048)), kb, int(rng.integers(1, 256)),
                      int(rng.integers(0, 4096)), int(rng.integers(0, 4)),
                      int(rng.integers(0, 2))], np.uint32)
        assert capi.npu_cycles(f) == ref_lib.hrbref_gemm_cycles(f, None)


@pytest.mark.parametrize("wfmt,M,N,K", [
    (0, 64, 960, 2560), (1, 64, 2560, 960), (0, 4096, 4096, 4096), (0, 141, 2560, 960),
    (1, 1, 8, 32), (1, 992, 2048, 720), (0, 65536, 960, 2560), (1, 5, 320, 65504)])
def test_dense_cycles_match_reference_tiling(ref_lib, wfmt, M, N, K):
    planes = 2 if wfmt == capi.WFMT_W8 else 1
    assert capi.dense_npu_cycles(wfmt, M, N, K) == ref_lib.hrbref_dense_gemm_cycles(
        planes, M, N, (K + 31) // 32)


def test_dense_cycles_reject_what_has_no_instruction():
    assert capi.dense_npu_cycles(capi.WFMT_MXFP8, 64, 64, 64) == 0
    assert capi.dense_npu_cycles(capi.WFMT_MXFP4, 64, 12, 64) == 0
