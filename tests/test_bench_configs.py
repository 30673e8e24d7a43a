"""The bench's configurations against the shapes and counts the survey
fixes for them (flops, algorithmic bytes, the C3 stream's GEMMs), and the
reference CPU leg's row padding, on the CPU."""
import numpy as np
import pytest

import bench


def test_c1_c2_algorithmic_bytes_and_flops():
    c1, c2 = bench.WORKLOADS["c1"], bench.WORKLOADS["c2"]
    assert c1.flops == c2.flops == 314_572_800
    # A (FP32) + W + W scales + bias + C, no padding.
    assert c2.bytes_step() == 655_360 + 1_228_800 + 76_800 + 245_760
    assert c1.bytes_step() == 245_760 + 2_457_600 + 76_800 + 10_240 + 655_360


def test_c3_prefix_stream_shapes():
    pw = bench.PREFIX
    assert pw.M == 141 and pw.layers == 16
    shapes = {name: (wfmt, k, n) for name, wfmt, k, n, _ in pw.gemms}
    assert shapes == {"q": (1, 960, 960), "k": (1, 960, 320), "v": (1, 960, 320),
                      "o": (1, 960, 960), "gate": (0, 960, 2560), "up": (0, 960, 2560),
                      "down": (0, 2560, 960)}
    assert pw.flops == 16 * 2_772_172_800
    # Dependency groups: Q/K/V share an input, then O, gate/up, down.
    assert [g for *_, g in pw.gemms] == [0, 0, 0, 1, 2, 2, 3]


def test_reference_leg_pads_rows_to_the_iss_token_multiple():
    from oracle import cpu
    if cpu.ref() is None:
        pytest.skip("reference build oracle/_ref is not present")
    wl = bench.Workload("t", "t", "t 40x64x64", 0, 40, 64, 64, False, 1, "hbm")
    r = bench.cpu_reference(wl, min_seconds=0.01, max_reps=1)
    assert r["kind"] == "reference" and "padded to 64 rows" in r["sample"]
    assert np.isfinite(r["value"]) and r["value"] > 0


def test_c4_expert_job_shapes():
    ew = bench.EXPERT
    groups = ew.step_groups()
    # 3 head groups in, 16 layers x 4 groups, 1 head group out.
    assert len(groups) == 68
    self_gemms = [g for _, gm in ew.self_layer for g in gm]
    assert [(k, n) for _, k, n in self_gemms] == [(720, 960), (720, 320), (720, 320),
                                                 (960, 720), (720, 2048), (720, 2048),
                                                 (2048, 720)]
    cross_gemms = [g for _, gm in ew.cross_layer for g in gm]
    assert [name for name, _, _ in cross_gemms] == ["q", "o", "gate", "up", "down"]
    assert ew.rows(1) == (12800, 36096) and ew.rows(8) == (1600, 4512)
    # Strong scaling: the job's FLOPs do not depend on the GPU count.
    assert ew.flops(1) == ew.flops(2) == ew.flops(8)
    per_token_step = (8 * sum(2 * k * n for _, k, n in self_gemms)
                      + 8 * sum(2 * k * n for _, k, n in cross_gemms)
                      + 2 * (32 * 720 + 3 * 720 * 720 + 720 * 32))
    kv = 8 * 2 * 2 * 141 * 960 * 320 * 256
    assert ew.flops() == 10 * 12800 * per_token_step + kv


def test_c5_sweep_covers_27_gemms_and_both_convs():
    wls = bench.sweep_workloads()
    assert len(wls) == 27 and len({w.key for w in wls}) == 27
    assert {(w.M, w.K, w.N, w.wfmt) for w in wls} == {
        (m, k, n, f) for m in (256, 4096, 65536) for k, n in ((960, 2560), (2560, 960),
                                                              (4096, 4096)) for f in (0, 1, 2)}
    assert all(w.bias == (w.wfmt == 1) for w in wls)
    assert bench.CONV.wfmt == 1 and bench.CONV_MXFP4.wfmt == 0
    assert bench.CONV.M == 48 * 16 * 44 and bench.CONV.K == 9 * 256
