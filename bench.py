"""Benchmark of the quantized GEMM hot path on B200.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]
                    [--config c2|c1|c4|c5|c5conv|gacc] [--mode exact|fast] [--batch B]

Default workload (the MXFP4 GEMM the metric is
quoted on): C = A . W^T with A FP32 [64, 2560] ~ N(0,1) encoded to MXINT8 on
the device, W MXFP4 [960, 2560] (E2M1 codes, one E8M0 scale per 32-block,
exponent in [-10, -4], canonicalised as hotarubi's compiler does), FP32 C
[64, 960].  --config c1 runs BASELINE configs[0]'s W8 GEMM (64 x 960 -> 2560,
per-channel int8 weights placed as hotarubi's compiler places a float
matrix, with bias); --config c5 one large-M MXFP4 GEMM of the configs[4]
sweep (4096 x 4096 x 4096), tensor-bound; --config c5conv the configs[4]
conv (3x3, 256 -> 256 channels, 48 maps of 16 x 44) as an implicit GEMM;
--config gacc the DMA engine's gather-accumulate on SparseDrive's detection
head sampling.

One step = the hot path over one batch of B independent instances of the
GEMM, each with its own activations, weights and output (C2: B = 128, 282 MB
of operands, more than twice the 126 MB L2, so every step streams from HBM
and no L2 flush is needed).  Per rank the batch is fixed: weak scaling, no
collective on the data path (the GEMMs are independent).

Reported (one JSON line, rank 0):
  value       TFLOP/s (2*M*N*K per GEMM) over all ranks, operands resident
              in HBM, max over ranks of the device time of K steps.
  e2e         the same metric through the plan's host entry point
              (hrb_plan_run_host): every step copies each GEMM's FP32
              activations from pinned host memory, runs, and copies C back;
              weights stay resident, as a loaded model's do.
  roofline    of the dominant kernel (the GEMM): its algorithmic bytes (or
              flops) per launch over its CUDA-event duration, against the
              measured HBM copy bandwidth (or tensor peak).
  cpu_baseline  the reference's own ExecuteGemm (oracle/_ref) on the host's
              cores on a bounded sample, rank 0 only.

--impl reference times only the reference's CPU implementation of the path
(rank 0), in the same metric.
"""
from __future__ import annotations

import argparse
import dataclasses
import json
import os
import re
import statistics
import sys
import threading
import time

import numpy as np

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, ROOT)

FMT_NAMES = {0: "mxfp4", 1: "w8", 2: "mxfp8"}


@dataclasses.dataclass(frozen=True)
class Workload:
    key: str
    name: str        # config.workload
    label: str       # metric label
    wfmt: int        # hrb_wfmt
    M: int
    N: int
    K: int
    bias: bool
    batch: int       # GEMMs per step per GPU
    bound: str       # "hbm" or "tensor"

    @property
    def kb(self) -> int:
        return (self.K + 31) // 32

    @property
    def flops(self) -> int:
        return 2 * self.M * self.N * self.K

    def w_bytes(self) -> int:
        return self.N * self.K // 2 if self.wfmt == 0 else self.N * self.K

    def bytes_step(self) -> int:
        """Compulsory bytes of one GEMM from FP32 activations."""
        return (self.M * self.K * 4 + self.w_bytes() + self.N * self.kb
                + (self.N * 4 if self.bias else 0) + self.M * self.N * 4)

    def bytes_gemm(self) -> int:
        """... of the GEMM kernel alone, which reads MXINT8 activations."""
        return (self.M * self.K + self.M * self.kb + self.w_bytes() + self.N * self.kb
                + (self.N * 4 if self.bias else 0) + self.M * self.N * 4)

    def bytes_quant(self) -> int:
        return self.M * self.K * 4 + self.M * self.K + self.M * self.kb

    @property
    def metric(self) -> str:
        return f"{FMT_NAMES[self.wfmt].upper()} GEMM TFLOP/s ({self.label})"


WORKLOADS = {
    "c2": Workload("c2", "c2_mxfp4_64x2560x960", "C2 64x2560x960", 0, 64, 960, 2560, False, 128,
                   "hbm"),
    "c1": Workload("c1", "c1_w8_64x960x2560", "C1 64x960x2560", 1, 64, 2560, 960, True, 128, "hbm"),
    "c5": Workload("c5", "c5_mxfp4_4096x4096x4096", "C5 4096x4096x4096", 0, 4096, 4096, 4096,
                   False, 4, "tensor"),
    # C4's largest GEMM (the action expert's MLP 720 -> 2048, MXFP8) for one
    # GPU's share of the 256 requests at 8 GPUs: 32 requests x 50 tokens,
    # one GEMM per layer of a flow step (16).  The whole C4 job is --config c4.
    "c4gemm": Workload("c4gemm", "c4_mxfp8_1600x720x2048", "C4 1600x720x2048", 2, 1600, 2048,
                       720, False, 16, "tensor"),
}


@dataclasses.dataclass(frozen=True)
class ConvWorkload:
    """The C5 conv (ResNet-50 stage-3 3x3, 256 -> 256 channels,
    16 x 44 maps, 6 cameras x batch 8), bias, FP32 NHWC input; W8 weights as
    the config names them (per-channel int8 placed as MXINT8 blocks), or
    MXFP4."""
    key: str = "c5conv"
    name: str = "c5_conv3x3_48x16x44x256_w8"
    images: int = 48
    H: int = 16
    W: int = 44
    cin: int = 256
    cout: int = 256
    kh: int = 3
    stride: int = 1
    wfmt: int = 1
    instances: int = 3   # rotated per step: 3 x ~190 MB > 2 x L2

    @property
    def M(self) -> int:
        return self.images * (self.H // self.stride) * (self.W // self.stride)

    @property
    def K(self) -> int:
        return self.kh * self.kh * self.cin

    @property
    def flops(self) -> int:
        return 2 * self.M * self.cout * self.K

    @property
    def metric(self) -> str:
        return (f"{FMT_NAMES[self.wfmt].upper()} implicit-GEMM conv TFLOP/s "
                "(C5 conv 3x3 256->256, 48 x 16x44)")

    def w_bytes(self) -> int:
        return self.cout * self.K // 2 if self.wfmt == 0 else self.cout * self.K

    def bytes_step(self) -> int:
        return (self.images * self.H * self.W * self.cin * 4 + self.w_bytes()
                + self.cout * self.K // 32 + self.cout * 4 + self.M * self.cout * 4)


CONV = ConvWorkload()
CONV_MXFP4 = dataclasses.replace(CONV, key="c5conv_mxfp4", name="c5_conv3x3_48x16x44x256_mxfp4",
                                 wfmt=0)
CONVS = {c.key: c for c in (CONV, CONV_MXFP4)}


@dataclasses.dataclass(frozen=True)
class GaccWorkload:
    """SparseDrive's detection head deformable sampling as GACC runs it
    (tools/compiler/sparsedrive_head.cpp:1177-1196: 928 padded anchors, per
    camera one GACC of 56 slots (4 levels x 13 points, padded) x 4 corners,
    8 blocks = 256 channels, chained over the 6 cameras).  Feature rows: the
    6 cameras' 4 levels of a 256 x 704 input (64x176 ... 8x22), MXINT8 row
    format; entries uniformly random (corners are not made adjacent)."""
    key: str = "gacc"
    name: str = "gacc_sparsedrive_det_928x336x4x256"
    tokens: int = 928
    slots: int = 6 * 56
    corners: int = 4
    blocks: int = 8
    nrows: int = 6 * (64 * 176 + 32 * 88 + 16 * 44 + 8 * 22)
    instances: int = 6    # rotated per step: 6 x ~45 MB > 2 x L2

    @property
    def entries(self) -> int:
        return self.tokens * self.slots * self.corners

    @property
    def row_stride(self) -> int:
        return (2 * self.blocks + 1) * 16

    @property
    def gathered_bytes(self) -> int:
        return self.entries * self.blocks * 33

    @property
    def metric(self) -> str:
        return "GACC gathered-row throughput GB/s (SparseDrive det head, 928 x 6 cams x 56 x 4)"


GACC = GaccWorkload()


@dataclasses.dataclass(frozen=True)
class PrefixWorkload:
    """C3: the SmolVLA-shaped VLM prefix stream, 16 decoder layers over M =
    141 tokens (2 cameras x 64 image tokens + 12 language + 1 state), hidden
    960, 15 query / 5 KV heads of 64, SiLU-gated MLP of 2560; Q/K/V/O in W8,
    the MLP in MXFP4, no bias (the model's linears have none).  Per layer the
    GEMMs run in their dependency groups: Q, K, V (one input), O (the
    attention output), gate and up (one input), down (the gated product);
    the attention, RMSNorm and SiLU between them are outside the GEMM path,
    so each group's input is a seeded synthetic activation with the shape the
    model gives it (N(0,1) rows renormalised to RMS 1, as each layer's norm
    leaves them)."""
    key: str = "c3"
    name: str = "c3_smolvla_prefix_16x141"
    M: int = 141
    layers: int = 16
    # (name, wfmt, K, N, group)
    gemms: tuple = (("q", 1, 960, 960, 0), ("k", 1, 960, 320, 0), ("v", 1, 960, 320, 0),
                    ("o", 1, 960, 960, 1), ("gate", 0, 960, 2560, 2), ("up", 0, 960, 2560, 2),
                    ("down", 0, 2560, 960, 3))
    streams: int = 2   # independent prefix streams, alternated so no step finds its weights in L2

    @property
    def flops(self) -> int:
        return self.layers * sum(2 * self.M * n * k for _, _, k, n, _ in self.gemms)

    @property
    def metric(self) -> str:
        return "W8/MXFP4 GEMM TFLOP/s (C3 SmolVLA prefix stream, 16 layers x 141 tokens)"

    def gemm_bytes(self, wfmt: int, k: int, n: int) -> int:
        """Compulsory bytes of one GEMM kernel launch (MXINT8 activations)."""
        kb = (k + 31) // 32
        w = n * k // 2 if wfmt == 0 else n * k
        return self.M * k + self.M * kb + w + n * kb + self.M * n * 4


PREFIX = PrefixWorkload()


@dataclasses.dataclass(frozen=True)
class ExpertWorkload:
    """C4: the SmolVLA-shaped action expert over a batch of 256 independent
    requests (tools/compiler/smolvla_expert.cpp: 16 layers of width 720,
    MLP 2048, odd layers cross-attending to the 141-token prefix,
    :75,182-203,608-651; 15 query / 5 KV heads of 64, smolvla_parts.hpp:
    29-30), every GEMM MXFP8 as the config sets it.  One bench step is the
    whole job: the cross-attention K/V projections of the prefix (960 ->
    320, once per request), then 10 flow steps, each the suffix heads
    (action in 32 -> 720, the time MLP 720 -> 720 twice and 720 -> 720,
    action out 720 -> 32) around the 16 layers.  The requests' rows are
    batched into each GEMM (50 tokens a request); N GPUs take 256 / N
    requests each (strong scaling).  Attention, norms and SiLU between the
    GEMMs are outside the GEMM path, so each dependency group reads a seeded
    synthetic FP32 input of its shape (rows of RMS 1)."""
    key: str = "c4"
    name: str = "c4_smolvla_expert_256req_10steps"
    requests: int = 256
    tokens: int = 50
    prefix: int = 141
    steps: int = 10
    layers: int = 16
    wfmt: int = 2
    # (group, [(name, K, N)]) per layer kind; the input of a group is shared.
    self_layer: tuple = (("qkv", (("q", 720, 960), ("k", 720, 320), ("v", 720, 320))),
                         ("o", (("o", 960, 720),)),
                         ("gate_up", (("gate", 720, 2048), ("up", 720, 2048))),
                         ("down", (("down", 2048, 720),)))
    cross_layer: tuple = (("q", (("q", 720, 960),)),
                          ("o", (("o", 960, 720),)),
                          ("gate_up", (("gate", 720, 2048), ("up", 720, 2048))),
                          ("down", (("down", 2048, 720),)))
    heads_in: tuple = (("action_in", (("in", 32, 720),)),
                       ("time_mlp_in", (("mlp_in_action", 720, 720),
                                        ("mlp_in_time", 720, 720))),
                       ("time_mlp_out", (("mlp_out", 720, 720),)))
    heads_out: tuple = (("action_out", (("out", 720, 32),)),)
    cross_kv: tuple = (("k", 960, 320), ("v", 960, 320))

    def rows(self, world: int) -> tuple[int, int]:
        """(suffix rows, prefix rows) of one GPU's GEMMs."""
        r = self.requests // world
        return r * self.tokens, r * self.prefix

    def step_groups(self) -> list:
        """One flow step's dependency groups in launch order: (label, gemms)."""
        out = [(f"head.{g}", gm) for g, gm in self.heads_in]
        for layer in range(self.layers):
            kind = self.cross_layer if layer % 2 else self.self_layer
            out += [(f"L{layer}.{g}", gm) for g, gm in kind]
        out += [(f"head.{g}", gm) for g, gm in self.heads_out]
        return out

    def flops(self, world: int = 1) -> int:
        """All GPUs' FLOPs of one job."""
        m, mp = self.rows(world)
        step = sum(2 * m * k * n for _, gm in self.step_groups() for _, k, n in gm)
        kv = (self.layers // 2) * sum(2 * mp * k * n for _, k, n in self.cross_kv)
        return world * (self.steps * step + kv)

    @property
    def metric(self) -> str:
        return ("MXFP8 GEMM TFLOP/s (C4 SmolVLA action expert, 256 requests x 10 flow steps "
                "x 16 layers)")


EXPERT = ExpertWorkload()


def peaks() -> dict:
    p = os.path.join(ROOT, "MEASURED_PEAKS.json")
    if os.path.exists(p):
        with open(p) as f:
            d = json.load(f)
        return {"hbm_gbs": d["hbm_gbs"], "bf16_tflops": d["bf16_tflops"],
                "bf16_tflops_sustained": d.get("bf16_tflops_sustained", d["bf16_tflops"]),
                "source": "measured"}
    return {"hbm_gbs": 6650.0, "bf16_tflops": 1590.0, "bf16_tflops_sustained": 1400.0,
            "source": "fallback"}


class ClockSampler:
    """SM clock and clock-event (throttle) reasons sampled through NVML every
    millisecond while the timed region runs (reads only; nothing is set).
    nvidia-smi's 200 ms sampling would miss a timed region of a few ms."""

    REASONS = {0x8: "hw_slowdown", 0x40: "hw_thermal_slowdown",
               0x20: "sw_thermal_slowdown", 0x4: "sw_power_cap", 0x80: "hw_power_brake"}

    def __init__(self, device: int):
        self.device = device
        self.samples: list[tuple[float, int]] = []
        self.max_mhz = None
        self.stop = threading.Event()
        self.nvml = None

    def __enter__(self):
        try:
            import pynvml
            pynvml.nvmlInit()
            self.nvml = pynvml
            self.h = pynvml.nvmlDeviceGetHandleByIndex(self.device)
            self.max_mhz = float(pynvml.nvmlDeviceGetMaxClockInfo(self.h, pynvml.NVML_CLOCK_SM))
            self.thread = threading.Thread(target=self._poll, daemon=True)
            self.thread.start()
        except Exception:
            self.nvml = None
        return self

    def _poll(self):
        p = self.nvml
        while not self.stop.is_set():
            try:
                mhz = p.nvmlDeviceGetClockInfo(self.h, p.NVML_CLOCK_SM)
                reasons = p.nvmlDeviceGetCurrentClocksEventReasons(self.h)
                self.samples.append((float(mhz), int(reasons)))
            except Exception:
                break
            time.sleep(0.001)

    def __exit__(self, *exc):
        self.stop.set()
        if self.nvml is not None:
            self.thread.join(timeout=5)

    def summary(self) -> dict:
        sm = [s[0] for s in self.samples]
        reasons = set()
        for _, bits in self.samples:
            for bit, name in self.REASONS.items():
                if bits & bit:
                    reasons.add(name)
        return {"sm_mhz": statistics.median(sm) if sm else None, "sm_max_mhz": self.max_mhz,
                "reasons": sorted(reasons), "samples": len(sm), "source": "nvml"}


# ---------------------------------------------------------------------------
# Synthetic operands (seeded; the survey's distributions)

def host_operands(wl: Workload, i: int, place=None):
    """Distinct operand set i: FP32 activations, weights and scales in the
    dense formats of include/hrb_gemm.h, bias (or None).  `place` encodes a
    float W8 matrix (default: this library's device encoder)."""
    from hotarubi_b200 import workloads
    x = workloads.activations(100 + i, wl.M, wl.K)
    b = workloads.bias(300 + i, wl.N) if wl.bias else None
    kp = wl.kb * 32  # the dense formats store K padded to whole blocks
    if wl.wfmt == 0:
        w, ws = workloads.mxfp4_weights(200 + i, wl.N, kp)
        if kp != wl.K:
            w[:, wl.K // 2:] = 0
    elif wl.wfmt == 1:
        q, s = workloads.w8_per_channel(200 + i, wl.N, wl.K)
        w, ws = (place or place_w8)(workloads.dequantize_per_channel(q, s))
    else:
        w, ws = workloads.mxfp8_weights(200 + i, wl.N, kp)
        w[:, wl.K:] = 0
    return x, w, ws, b


def place_w8(wf: np.ndarray):
    """A float weight matrix placed as W8 the way hotarubi's compiler does
    (PlaceW8: EncodeMxint8, then the HI/LO split the W8 format implies), with
    this library's own device encoder."""
    import torch

    from hotarubi_b200 import capi
    n, k = wf.shape
    kb = (k + 31) // 32
    lib = capi.Library(torch.cuda.current_device())
    x = torch.from_numpy(np.ascontiguousarray(wf)).cuda()
    q = torch.zeros((n, kb * 32), dtype=torch.int8, device="cuda")
    s = torch.zeros((n, kb), dtype=torch.uint8, device="cuda")
    torch.cuda.synchronize()  # the fills (torch's stream) before the encoder (the library's)
    lib.quantize(x, n, k, q, s)
    lib.sync()
    out = q.cpu().numpy().view(np.uint8), s.cpu().numpy()
    lib.close()
    return out


# ---------------------------------------------------------------------------
# The reference's CPU implementation (test infrastructure, timed only)

def cpu_reference(wl: Workload, min_seconds: float = 2.0, max_reps: int = 50,
                  columns: bool = False) -> dict:
    """hotarubi's ExecuteGemm, compiled from the reference sources
    (oracle/_ref), tiled into legal GEMM instructions over all host threads,
    on GEMMs of the workload until ~min_seconds of wall time; rows of large-M
    workloads are sampled (rows are independent)."""
    from oracle import cpu
    ref = cpu.ref()
    threads = os.cpu_count() or 1

    def place_cpu(wf):  # the same placement on the host (EncodeMxint8)
        q, s = cpu.encode_mxint8(wf.view(np.uint32))
        return q.view(np.uint8), s

    x, w, ws, _ = host_operands(wl, 0, place_cpu)
    rows = min(wl.M, 256)
    q, s = cpu.encode_mxint8(x[:rows].view(np.uint32))
    sample_flops = 2 * rows * wl.N * wl.K
    label = f"{wl.label}" + ("" if rows == wl.M else f", first {rows} of {wl.M} rows")
    if ref is None or wl.wfmt == 2:
        # No reference build (or MXFP8, which the reference lacks): the C
        # restatement stands in.
        t0 = time.perf_counter()
        reps = 0
        while reps < 1 or time.perf_counter() - t0 < min_seconds / 4:
            cpu.gemm_dense(wl.wfmt, q, s, w, ws, wl.N)
            reps += 1
        dt = time.perf_counter() - t0
        return {"value": reps * sample_flops / dt / 1e12, "unit": "TFLOP/s", "cores": 1,
                "kind": "port", "sample": f"{reps} x {label} on 1 thread", "seconds": dt}
    # The ISS runs tokens in multiples of 32 (GemmCommand.m): pad with zero
    # rows (scale byte 127) as a runtime would; the flops counted stay the
    # real rows'.
    prow = (rows + 31) // 32 * 32
    if prow != rows:
        q = np.concatenate([q, np.zeros((prow - rows, q.shape[1]), q.dtype)])
        s = np.concatenate([s, np.full((prow - rows, s.shape[1]), 127, s.dtype)])
        label += f", padded to {prow} rows"
    a_words = cpu.pack_abuf(q, s).reshape(-1)
    kp = wl.kb * 32
    if wl.wfmt == 0:
        codes = np.zeros((wl.N, kp), np.uint8)
        codes[:, 0::2] = w & 0xF
        codes[:, 1::2] = w >> 4
        planes = cpu.pack_wbuf(codes, ws).reshape(-1)
        nplanes = 1
    else:
        hi, lo = cpu.split_w8(w.view(np.int8))
        planes = np.concatenate([cpu.pack_wbuf(hi, ws).reshape(-1),
                                 cpu.pack_wbuf(lo, ws).reshape(-1)])
        nplanes = 2
    c = np.zeros((prow, wl.N), np.uint32)
    ref.hrbref_dense_gemm_iss(nplanes, prow, wl.N, wl.kb, a_words, planes, c, threads, 0, prow)
    t0 = time.perf_counter()
    reps = 0
    while reps < max_reps and (reps < 1 or time.perf_counter() - t0 < min_seconds):
        ref.hrbref_dense_gemm_iss(nplanes, prow, wl.N, wl.kb, a_words, planes, c, threads, 0,
                                  prow)
        reps += 1
    dt = time.perf_counter() - t0
    out = {"value": reps * sample_flops / dt / 1e12, "unit": "TFLOP/s", "cores": threads,
           "kind": "reference",
           "sample": f"{reps} x {label} through ExecuteGemm tiles on {threads} threads",
           "seconds": dt}
    if columns:
        out["columns"] = cpu_columns(ref, nplanes, prow, wl, a_words, planes, c, sample_flops,
                                     min_seconds / 2)
    return out


def cpu_columns(ref, nplanes, rows, wl, a_words, planes, c, flops, min_seconds):
    """The other CPU columns of the metric ("vs gemm_ref CPU"): the same
    sample through ExecuteGemm on one thread, and through tb/gemm_ref's
    ReferenceGemm (tb/gemm_ref.cpp:47-68, the model the RTL is checked
    against) on one thread and on all host threads."""
    import ctypes

    f = ref.hrbref_dense_gemm_tb
    f.restype = ctypes.c_int
    f.argtypes = [ctypes.c_uint32] * 4 + [np.ctypeslib.ndpointer(np.uint8),
                                          np.ctypeslib.ndpointer(np.uint8),
                                          np.ctypeslib.ndpointer(np.uint32), ctypes.c_uint32]
    threads = os.cpu_count() or 1

    def timed(run):
        run()
        t0 = time.perf_counter()
        reps = 0
        while reps < 1 or time.perf_counter() - t0 < min_seconds:
            run()
            reps += 1
        return reps * flops / (time.perf_counter() - t0) / 1e12

    return {
        "execute_gemm_1_thread": timed(lambda: ref.hrbref_dense_gemm_iss(
            nplanes, rows, wl.N, wl.kb, a_words, planes, c, 1, 0, rows)),
        "gemm_ref_1_thread": timed(lambda: f(nplanes, rows, wl.N, wl.kb, a_words, planes, c, 1)),
        f"gemm_ref_{threads}_threads": timed(lambda: f(nplanes, rows, wl.N, wl.kb, a_words,
                                                         planes, c, threads)),
        "unit": "TFLOP/s",
    }


def trial_stats(ms: list[float]) -> dict:
    """Per-step device times of the timed region (each step a trial)."""
    v = sorted(ms)
    return {"n": len(v), "median_ms": statistics.median(v), "min_ms": v[0], "max_ms": v[-1],
            "spread": (v[-1] - v[0]) / statistics.median(v) if v else 0.0}


def tensor_fracs(tflops: float, pk: dict, wfmt: int) -> dict:
    """A tensor-bound rate against (i) the dense peak of the MMA kind the
    kernel issues (kind::mxf4 4x, kind::mxf8f6f4 2x the measured dense BF16
    rate: NVIDIA's dense ratios) and (ii) the 8-bit dense peak (2x BF16)."""
    kind, mult = ("kind::mxf8f6f4", 2.0) if wfmt == 2 else ("kind::mxf4", 4.0)
    return {"mma_kind": kind,
            "frac_of_kind_dense_peak": tflops / (mult * pk["bf16_tflops"]),
            "frac_of_8bit_dense_peak": tflops / (2.0 * pk["bf16_tflops"])}


def run_reference(args, wl: Workload, rank: int, world: int) -> None:
    if rank != 0:
        return
    steps = []
    for i in range(args.warmup + args.steps):
        r = cpu_reference(wl, min_seconds=0.25, max_reps=20)
        if i >= args.warmup:
            steps.append(r)
    value = statistics.median(r["value"] for r in steps)
    secs = statistics.median(r["seconds"] for r in steps)
    base = steps[-1]
    line = {
        "impl": "reference", "metric": wl.metric,
        "value": value, "unit": "TFLOP/s", "n_gpus": args.gpus, "steps": args.steps,
        "warmup": args.warmup, "ms_per_step": secs * 1e3, "higher_is_better": True,
        "scaling": "weak", "vs_baseline": None, "dtype": "int8 block dot + fp32 accumulate",
        "data": "synthetic",
        "config": {"workload": wl.name, "M": wl.M, "N": wl.N, "K": wl.K,
                   "format": FMT_NAMES[wl.wfmt], "sample": base["sample"]},
        "cpu_baseline": {"value": value, "unit": "TFLOP/s", "cores": base["cores"],
                         "kind": base["kind"], "sample": base["sample"]},
        "e2e": {"value": value, "unit": "TFLOP/s", "h2d_bytes_per_step": 0,
                "d2h_bytes_per_step": 0},
    }
    print(json.dumps(line), flush=True)


# ---------------------------------------------------------------------------
# Our implementation

def build_batch(torch, lib, capi, wl: Workload, batch: int, mode: int, distinct: int = 4,
                w8_kernel: int = 0):
    """B instances on the device: `distinct` seeded operand sets copied into
    B separate buffers (distinct memory, so every instance streams)."""
    sets = [host_operands(wl, i) for i in range(min(distinct, batch))]
    # Activations and outputs of the batch are one allocation each (a batch
    # of requests arrives and leaves as one block); weights are separate.
    a_all = torch.empty((batch, wl.M, wl.K), dtype=torch.float32, device="cuda")
    c_all = torch.zeros((batch, wl.M, wl.N), dtype=torch.float32, device="cuda")
    inst = []
    for b in range(batch):
        x, w, ws, bias = sets[b % len(sets)]
        a_all[b].copy_(torch.from_numpy(x))
        inst.append(dict(
            a=a_all[b], w=torch.from_numpy(w).cuda(), ws=torch.from_numpy(ws).cuda(),
            bias=None if bias is None else torch.from_numpy(bias).cuda(), c=c_all[b]))
    descs = [capi.Library.desc(wl.wfmt, wl.M, wl.N, wl.K, a=d["a"], w=d["w"], wscale=d["ws"],
                               bias=d["bias"], c=d["c"], mode=mode, w8_kernel=w8_kernel)
             for d in inst]
    torch.cuda.synchronize()
    return inst, lib.plan(descs), sets


_E2M1 = np.array([0, 0.5, 1, 1.5, 2, 3, 4, 6], np.float64)


def dequant_weights(wfmt: int, w: np.ndarray, ws: np.ndarray, n: int, kp: int) -> np.ndarray:
    """[N][kp] float64 values of the dense weight formats (include/hrb_gemm.h)."""
    sc = np.repeat(np.ldexp(1.0, ws.astype(np.int64) - 127), 32, axis=1)
    if wfmt == 0:
        codes = np.zeros((n, kp), np.uint8)
        codes[:, 0::2] = w & 0xF
        codes[:, 1::2] = w >> 4
        return _E2M1[codes & 7] * np.where(codes & 8, -1.0, 1.0) * sc
    if wfmt == 1:
        return w.view(np.int8).astype(np.float64) * sc * 2.0**-6
    e = ((w >> 3) & 0xF).astype(np.int64)
    m = (w & 7).astype(np.float64)
    v = np.where(e == 0, m / 8 * 2.0**-6, (1 + m / 8) * np.ldexp(1.0, e - 7))
    return np.where(w & 0x80, -v, v) * sc


def fast_parity(torch, lib, wl: Workload, x, w, ws, bias, c_dev, rows: int = 64,
                tail: bool = False) -> dict:
    """GEMM 0's fast-mode output on its first rows (with `tail`, half of them
    the last rows: the last token tile) against the float64 dot product of
    its dequantized operands (activation codes from the library's own MXINT8
    encoder): the max relative error, the stated bound (K/16 + 4) 2^-23
    sum|a w| per output, and the ulp histogram against that product rounded
    to FP32."""
    m = min(rows, wl.M)
    sel = np.arange(m)
    if tail and wl.M > m:
        sel = np.concatenate([np.arange(m // 2), np.arange(wl.M - (m - m // 2), wl.M)])
    kb, kp = wl.kb, wl.kb * 32
    xd = torch.from_numpy(np.ascontiguousarray(x[sel])).cuda()
    q = torch.zeros((m, kp), dtype=torch.int8, device="cuda")
    s = torch.zeros((m, kb), dtype=torch.uint8, device="cuda")
    torch.cuda.synchronize()  # the fills (torch's stream) before the encoder (the library's)
    lib.quantize(xd, m, wl.K, q, s)
    lib.sync()
    a = q.cpu().numpy().astype(np.float64) * np.repeat(
        np.ldexp(1.0, s.cpu().numpy().astype(np.int64) - 133), 32, axis=1)
    wd = dequant_weights(wl.wfmt, w, ws, wl.N, kp)
    ref = a @ wd.T
    absref = np.abs(a) @ np.abs(wd).T
    if bias is not None:
        ref += bias.astype(np.float64)
        absref += np.abs(bias.astype(np.float64))
    got = c_dev[torch.from_numpy(sel).to(c_dev.device)].cpu().numpy()
    err = np.abs(got.astype(np.float64) - ref)
    bound = (kp / 16 + 4) * 2.0**-23 * absref + 1e-30
    rel = err / (absref + 1e-30)

    def ordered(v):
        i = v.view(np.int32).astype(np.int64)
        return np.where(i < 0, -(i & 0x7FFFFFFF), i)
    d = np.abs(ordered(got.astype(np.float32)) - ordered(ref.astype(np.float32)))
    worst = np.unravel_index(int(np.argmax(rel)), rel.shape)
    return {"reference": "float64 dot of the dequantized operands (library MXINT8 encoder)",
            "rows": m if not tail or wl.M <= m else f"first {m // 2} and last {m - m // 2}",
            "outputs": int(err.size), "max_rel_err": float(rel.max()),
            "worst_at": [int(sel[worst[0]]), int(worst[1])],
            "outside_bound": int((err > bound).sum()),
            "bound": "(K/16 + 4) * 2^-23 * sum|a w| per output",
            "within_bound": bool((err <= bound).all()),
            "ulp_hist_vs_fp32_rounded": {"0": int((d == 0).sum()), "1": int((d == 1).sum()),
                                         "2-3": int(((d >= 2) & (d < 4)).sum()),
                                         "4-15": int(((d >= 4) & (d < 16)).sum()),
                                         ">=16": int((d >= 16).sum())}}


def traffic_from_profiles(kernel: str, wl: Workload):
    """DRAM bytes per GEMM of `kernel` on this workload, as summarised from an
    ncu capture in profiles/dram_traffic.txt (lines: kernel workload bytes)."""
    path = os.path.join(ROOT, "profiles", "dram_traffic.txt")
    if not os.path.exists(path):
        return None
    for line in open(path):
        parts = line.split()
        if len(parts) >= 3 and parts[0] == kernel and parts[1] == wl.name:
            return float(parts[2])
    return None


def time_e2e(torch, plan, wl: Workload, sets, batch: int, steps: int, warmup: int,
             stream) -> dict:
    """hrb_plan_run_host over the batch: every GEMM's FP32 activations from
    pinned host memory to the device, the plan, C back to pinned memory."""
    a_all = torch.empty((batch, wl.M, wl.K), dtype=torch.float32).pin_memory()
    for b in range(batch):
        a_all[b].copy_(torch.from_numpy(sets[b % len(sets)][0]))
    c_all = torch.zeros((batch, wl.M, wl.N), dtype=torch.float32).pin_memory()
    a_host = [a_all[b] for b in range(batch)]
    c_host = [c_all[b] for b in range(batch)]
    for _ in range(warmup):
        plan.run_host(a_host, c_host, stream=stream.cuda_stream)
    stream.synchronize()
    t0 = time.perf_counter()
    for _ in range(steps):
        plan.run_host(a_host, c_host, stream=stream.cuda_stream)
        stream.synchronize()
    dt = (time.perf_counter() - t0) / steps
    return {"value": batch * wl.flops / dt / 1e12, "unit": "TFLOP/s",
            "h2d_bytes_per_step": batch * wl.M * wl.K * 4,
            "d2h_bytes_per_step": batch * wl.M * wl.N * 4, "ms_per_step": dt * 1e3,
            "entry_point": "hrb_plan_run_host (weights resident)"}


def run_ours(args, wl: Workload, rank: int, world: int, local_rank: int) -> None:
    import torch

    from hotarubi_b200 import capi
    torch.cuda.set_device(local_rank)
    dist = None
    if world > 1:
        import datetime

        import torch.distributed as dist
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=120),
                                device_id=torch.device("cuda", local_rank))
    lib = capi.Library(local_rank)
    mode = capi.MODE_FAST if args.mode == "fast" else capi.MODE_EXACT
    stream = torch.cuda.Stream()
    lib.set_stream(stream.cuda_stream)
    batch = args.batch or wl.batch
    w8_bf16 = args.w8_kernel == "bf16" and wl.wfmt == capi.WFMT_W8 and wl.M <= 64
    inst, plan_full, sets = build_batch(torch, lib, capi, wl, batch, mode,
                                        w8_kernel=capi.W8_BF16 if w8_bf16 else capi.W8_DIGIT_PLANES)

    # Per-kernel device times (the dominant kernel's roofline): each launch
    # of the plan repeated back to back between two events (not the timed
    # region).
    kernel_ms = plan_full.profile(reps=20, stream=stream.cuda_stream)
    quant_ms, gemm_ms = kernel_ms[0], sum(kernel_ms[1:])

    if dist is not None:
        dist.barrier()
    torch.cuda.synchronize()
    with ClockSampler(local_rank) as clocks:
        for _ in range(args.warmup):
            plan_full.run(stream.cuda_stream)
        stream.synchronize()
        if dist is not None:
            dist.barrier()
        torch.cuda.synchronize()
        # One event after every step as well: each step is a timing trial.
        marks = [torch.cuda.Event(enable_timing=True) for _ in range(args.steps + 1)]
        marks[0].record(stream)
        launches = 0
        for i in range(args.steps):
            launches += plan_full.run(stream.cuda_stream)
            marks[i + 1].record(stream)
        marks[-1].synchronize()
        torch.cuda.synchronize()
        if dist is not None:
            dist.barrier()
    lib.sync()
    ms = marks[0].elapsed_time(marks[-1]) / args.steps
    trials = trial_stats([marks[i].elapsed_time(marks[i + 1]) for i in range(args.steps)])
    if dist is not None:
        t = torch.tensor([ms], device="cuda")
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        ms = float(t.item())
    parity = None
    if rank == 0 and mode == capi.MODE_FAST:
        x0, w0, ws0, b0 = sets[0]
        parity = fast_parity(torch, lib, wl, x0, w0, ws0, b0, inst[0]["c"])

    e2e = None
    if not args.no_e2e:
        e2e = time_e2e(torch, plan_full, wl, sets, batch, max(1, min(args.steps, 10)), 2, stream)
    if dist is not None and e2e is not None:
        t = torch.tensor([e2e["ms_per_step"]], device="cuda")
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        e2e["ms_per_step"] = float(t.item())
        e2e["value"] = world * batch * wl.flops / (e2e["ms_per_step"] / 1e3) / 1e12
        e2e["h2d_bytes_per_step"] *= world
        e2e["d2h_bytes_per_step"] *= world

    if rank == 0:
        pk = peaks()
        fast = mode == capi.MODE_FAST
        kname = ("k_gemm_w8bf" if w8_bf16 else "k_gemm_mxf4") if fast else exact_kernel(wl.wfmt)
        qname = "k_quantize_planes" if fast else "k_quantize"
        gemm_gbs = batch * wl.bytes_gemm() / (gemm_ms / 1e3) / 1e9
        quant_gbs = batch * wl.bytes_quant() / (quant_ms / 1e3) / 1e9
        per_gemm_traffic = traffic_from_profiles(kname, wl) if fast else None
        per_quant_traffic = traffic_from_profiles(qname, wl) if fast else None
        step_gbs = batch * wl.bytes_step() / (ms / 1e3) / 1e9
        if wl.bound == "hbm":
            roof = {"bound": "hbm", "kernel": kname, "achieved": gemm_gbs, "peak": pk["hbm_gbs"],
                    "unit": "GB/s", "frac": gemm_gbs / pk["hbm_gbs"],
                    "peak_source": pk["source"] + " (HBM copy)",
                    "alg_bytes_per_launch": batch * wl.bytes_gemm()}
        else:
            tflops = batch * wl.flops / (gemm_ms / 1e3) / 1e12
            if not fast and exact_kernel(wl.wfmt) == "k_exact_tc":
                # k_exact_tc: one kind::i8 MMA per block product (2x the dense
                # BF16 rate), W8 two (its HI and LO nibble planes).
                peak = pk["bf16_tflops"] * 2.0 / (1.0 if wl.wfmt == 0 else 2.0)
                how = (" (cuBLAS BF16 x 2: the int8 MMA rate)" if wl.wfmt == 0
                       else " (cuBLAS BF16 x 2 / 2: the int8 MMA rate over two nibble planes)")
            elif wl.wfmt == 2:
                # MXFP8 runs kind::mxf8f6f4 at 2x the dense BF16 rate, with two
                # E4M3 digit planes per exact product: the BF16 peak.
                peak, how = pk["bf16_tflops"], " (cuBLAS BF16: FP8 MMA rate over two digit planes)"
            else:
                # kind::mxf4 runs at 4x the dense BF16 rate (nominal 9 vs
                # 2.25 PFLOP/s); each exact MXINT8 x E2M1 product takes three
                # of its MMAs (the activation digit planes; W8 weights add
                # three planes more), so the useful ceiling is a third (a
                # ninth) of that.
                peak = pk["bf16_tflops"] * 4.0 / (3.0 if wl.wfmt == 0 else 9.0)
                how = (" (cuBLAS BF16 x 4/3: FP4 MMA rate over three digit planes)"
                       if wl.wfmt == 0 else " (cuBLAS BF16 x 4/9: FP4 MMA rate over 3 x 3 planes)")
            roof = {"bound": "tensor", "kernel": kname, "achieved": tflops,
                    "peak": pk["bf16_tflops"], "unit": "TFLOP/s",
                    "frac": tflops / pk["bf16_tflops"],
                    "peak_source": pk["source"] + " (cuBLAS BF16 dense)",
                    **tensor_fracs(tflops, pk, wl.wfmt),
                    "useful_ceiling": {"peak": peak, "frac": tflops / peak,
                                       "how": pk["source"] + how},
                    "alg_flops_per_launch": batch * wl.flops}
        roof.update({"traffic": (None if per_gemm_traffic is None
                                 else per_gemm_traffic * batch),
                     "launch_ms": gemm_ms})
        total_gemms = world * batch
        line = {
            "metric": wl.metric,
            "value": total_gemms * wl.flops / (ms / 1e3) / 1e12,
            "unit": "TFLOP/s", "n_gpus": world, "steps": args.steps, "warmup": args.warmup,
            "ms_per_step": ms, "higher_is_better": True, "scaling": "weak",
            "vs_baseline": None, "dtype": "int8 block dot + fp32 accumulate",
            "data": "synthetic",
            "config": {"workload": wl.name, "batch_per_gpu": batch,
                       "M": wl.M, "N": wl.N, "K": wl.K, "format": FMT_NAMES[wl.wfmt],
                       "bias": wl.bias, "mode": args.mode,
                       **({"w8_kernel": args.w8_kernel} if wl.wfmt == capi.WFMT_W8 else {}),
                       "activations": "fp32, encoded to mxint8 on device each step",
                       "l2": f"working set {batch * wl.bytes_step() / 1e6:.0f} MB per GPU"
                             + (" > 2 x 126 MB L2, no flush" if batch * wl.bytes_step() > 252e6
                                else ""),
                       "parallelism": f"replicas x{world} (independent GEMMs)"},
            "step_hbm_gbs": step_gbs,
            "step_hbm_frac": step_gbs / pk["hbm_gbs"],
            "trials": trials,
            "roofline": roof,
            "encoder": {"kernel": qname, "launch_ms": quant_ms, "achieved_gbs": quant_gbs,
                        "frac": quant_gbs / pk["hbm_gbs"],
                        "alg_bytes_per_launch": batch * wl.bytes_quant(),
                        "traffic": (None if per_quant_traffic is None
                                    else per_quant_traffic * batch)},
            "e2e": e2e, "gpu_launches": launches,
            "clocks": clocks.summary(),
        }
        if parity is not None:
            line["parity"] = parity
        # The same batch on hotarubi's NPU, by the ISS cycle model of its GEMM
        # instructions at the 250 MHz PL clock (none for MXFP8).
        npu = capi.dense_npu_cycles(wl.wfmt, wl.M, wl.N, wl.K)
        if npu:
            npu_ms = batch * npu / capi.NPU_CLOCK_HZ * 1e3
            line["npu_equivalent"] = {"cycles_per_gemm": npu, "ms_per_step": npu_ms,
                                      "per_gpu_speedup": npu_ms / ms,
                                      "model": "CostModel::Gemm over the GEMM instructions "
                                               "of a tiled run, 250 MHz"}
        if not args.no_cpu_baseline:
            line["cpu_baseline"] = {k: v for k, v in cpu_reference(wl, columns=True).items()
                                    if k != "seconds"}
        print(json.dumps(line), flush=True)
    plan_full.close()
    lib.close()
    if dist is not None:
        dist.barrier()
        dist.destroy_process_group()


def exact_kernel(wfmt: int) -> str:
    """The kernel of an exact-mode GEMM: k_exact_tc (int8 tensor-core block
    dots) for MXFP4 and W8 unless HRB_EXACT_TC=0, else k_dense_exact."""
    tc = os.environ.get("HRB_EXACT_TC", "1") != "0"
    return "k_exact_tc" if tc and wfmt in (0, 1) else "k_dense_exact"


def conv_operands(cw: ConvWorkload, i: int, place=None):
    """FP32 NHWC map, weights [cout][9 x cin] (tap-major) in the dense format,
    bias.  W8: per-channel int8 placed as MXINT8 blocks (`place`, default
    this library's device encoder)."""
    from hotarubi_b200 import workloads
    x = workloads.activations(500 + i, cw.images * cw.H * cw.W, cw.cin)
    if cw.wfmt == 1:
        q, sc = workloads.w8_per_channel(600 + i, cw.cout, cw.K)
        w, ws = (place or place_w8)(workloads.dequantize_per_channel(q, sc))
    else:
        w, ws = workloads.mxfp4_weights(600 + i, cw.cout, cw.K)
    b = workloads.bias(700 + i, cw.cout)
    return x, w, ws, b


def conv_cpu_reference(cw: ConvWorkload, min_seconds: float = 2.0) -> dict:
    """The conv lowered as ConvEmitter lowers it and run on the reference's
    own DMA engine and ExecuteGemm (oracle/_ref hrbref_conv_iss, one thread),
    on one image of the batch."""
    from oracle import cpu
    ref = cpu.ref()

    def place_cpu(wf):  # W8 placement on the host (EncodeMxint8)
        q, s = cpu.encode_mxint8(wf.view(np.uint32))
        return q.view(np.uint8), s

    x, w, ws, b = conv_operands(cw, 0, place_cpu)
    hw = cw.H * cw.W
    # One image, x-major as the compiler's maps are (the conv is the same).
    img = x[:hw].reshape(cw.H, cw.W, cw.cin).transpose(1, 0, 2).reshape(hw, cw.cin)
    q, s = cpu.encode_mxint8(np.ascontiguousarray(img).view(np.uint32))
    if cw.wfmt == 0:
        codes = np.zeros((cw.cout, cw.K), np.uint8)
        codes[:, 0::2] = w & 0xF
        codes[:, 1::2] = w >> 4
    else:
        hi, lo = cpu.split_w8(w.view(np.int8))
    e = ws.astype(np.int32) - 127
    flops = 2 * hw // (cw.stride * cw.stride) * cw.cout * cw.K
    c = np.zeros((hw // (cw.stride * cw.stride), cw.cout), np.uint32)
    if ref is None:
        t0 = time.perf_counter()
        cpu.conv_dense(cw.wfmt, q, s, 1, cw.H, cw.W, cw.cin, cw.cout, cw.kh, cw.stride, w, ws,
                       bias_bits=b.view(np.uint32))
        dt = time.perf_counter() - t0
        return {"value": flops / dt / 1e12, "unit": "TFLOP/s", "cores": 1, "kind": "port",
                "sample": "1 of 48 images on 1 thread", "seconds": dt}
    t0 = time.perf_counter()
    reps = 0
    while reps < 1 or time.perf_counter() - t0 < min_seconds:
        if cw.wfmt == 0:
            ref.hrbref_conv_iss(cw.H, cw.W, cw.cin, cw.cout, cw.kh, cw.stride, q.ravel(),
                                s.ravel(), codes.ravel(), e.ravel(), b.view(np.uint32), None, 0,
                                c.ravel())
        else:
            ref.hrbref_conv_iss_w8(cw.H, cw.W, cw.cin, cw.cout, cw.kh, cw.stride, q.ravel(),
                                   s.ravel(), hi.ravel(), lo.ravel(), e.ravel(),
                                   b.view(np.uint32), None, 0, c.ravel())
        reps += 1
    dt = time.perf_counter() - t0
    return {"value": reps * flops / dt / 1e12, "unit": "TFLOP/s", "cores": 1,
            "kind": "reference",
            "sample": f"{reps} x 1 of 48 images through the reference's DMA gathers and "
                      "ExecuteGemm on 1 thread", "seconds": dt}


def run_conv(args, rank: int, world: int, local_rank: int) -> None:
    """--config c5conv: the C5 conv through hrb_conv_plan_* (fast mode:
    the FP32 map encoded once into operand blocks, the 3x3 taps' blocks
    gathered per output row, the tcgen05 GEMM over K = 9 x 256).  One step = one conv over the 48 images; the
    instances rotate so no step finds its operands in L2.  Replicas for
    N > 1 (weak scaling)."""
    import torch

    from hotarubi_b200 import capi
    cw = CONVS[args.config]
    if args.impl == "reference":
        if rank != 0:
            return
        runs = [conv_cpu_reference(cw, 0.5) for _ in range(args.warmup + args.steps)]
        runs = runs[args.warmup:]
        value = statistics.median(r["value"] for r in runs)
        base = runs[-1]
        print(json.dumps({
            "impl": "reference", "metric": cw.metric, "value": value, "unit": "TFLOP/s",
            "n_gpus": args.gpus, "steps": args.steps, "warmup": args.warmup,
            "ms_per_step": statistics.median(r["seconds"] for r in runs) * 1e3,
            "higher_is_better": True, "scaling": "weak", "vs_baseline": None,
            "dtype": "int8 block dot + fp32 accumulate", "data": "synthetic",
            "config": {"workload": cw.name, "sample": base["sample"]},
            "cpu_baseline": {k: v for k, v in base.items() if k != "seconds"} | {"value": value},
            "e2e": {"value": value, "unit": "TFLOP/s", "h2d_bytes_per_step": 0,
                    "d2h_bytes_per_step": 0}}), flush=True)
        return
    torch.cuda.set_device(local_rank)
    dist = None
    if world > 1:
        import datetime

        import torch.distributed as dist
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=120),
                                device_id=torch.device("cuda", local_rank))
    lib = capi.Library(local_rank)
    mode = capi.MODE_FAST if args.mode == "fast" else capi.MODE_EXACT
    stream = torch.cuda.Stream()
    lib.set_stream(stream.cuda_stream)
    inst = []
    for i in range(cw.instances):
        x, w, ws, b = conv_operands(cw, i)
        t = {"x": torch.from_numpy(x).cuda(), "w": torch.from_numpy(w).cuda(),
             "ws": torch.from_numpy(ws).cuda(), "b": torch.from_numpy(b).cuda(),
             "c": torch.zeros((cw.M, cw.cout), dtype=torch.float32, device="cuda")}
        d = capi.conv_desc(cw.wfmt, cw.images, cw.H, cw.W, cw.cin, cw.cout, cw.kh, cw.stride,
                           order=capi.CONV_YMAJOR, a=t["x"], w=t["w"], wscale=t["ws"],
                           bias=t["b"], c=t["c"], mode=mode)
        t["plan"] = lib.conv_plan(d)
        inst.append(t)
    torch.cuda.synchronize()
    kernel_ms = inst[0]["plan"].profile(reps=10, stream=stream.cuda_stream)
    gemm_ms = kernel_ms[-1] if mode == capi.MODE_FAST else max(kernel_ms)
    prep_ms = sum(kernel_ms) - gemm_ms
    if dist is not None:
        dist.barrier()
    with ClockSampler(local_rank) as clocks:
        for i in range(args.warmup):
            inst[i % cw.instances]["plan"].run(stream.cuda_stream)
        stream.synchronize()
        if dist is not None:
            dist.barrier()
        torch.cuda.synchronize()
        start = torch.cuda.Event(enable_timing=True)
        end = torch.cuda.Event(enable_timing=True)
        start.record(stream)
        launches = 0
        for i in range(args.steps):
            launches += inst[i % cw.instances]["plan"].run(stream.cuda_stream)
        end.record(stream)
        end.synchronize()
        if dist is not None:
            dist.barrier()
    lib.sync()
    ms = start.elapsed_time(end) / args.steps
    if dist is not None:
        t = torch.tensor([ms], device="cuda")
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        ms = float(t.item())
    # End to end: the FP32 map from pinned host memory, the conv, C back.
    e2e = None
    if not args.no_e2e:
        xh = torch.from_numpy(conv_operands(cw, 0)[0]).pin_memory()
        ch = torch.empty((cw.M, cw.cout), dtype=torch.float32).pin_memory()
        t0 = inst[0]
        n_e2e = max(1, min(args.steps, 10))
        for k in range(2 + n_e2e):
            if k == 2:
                stream.synchronize()
                w0 = time.perf_counter()
            with torch.cuda.stream(stream):
                t0["x"].copy_(xh, non_blocking=True)
                t0["plan"].run(stream.cuda_stream)
                ch.copy_(t0["c"], non_blocking=True)
            stream.synchronize()
        dt = (time.perf_counter() - w0) / n_e2e
        e2e = {"value": world * cw.flops / dt / 1e12, "unit": "TFLOP/s",
               "h2d_bytes_per_step": world * xh.numel() * 4,
               "d2h_bytes_per_step": world * ch.numel() * 4, "ms_per_step": dt * 1e3,
               "entry_point": "pinned copies + hrb_conv_plan_run (weights resident)"}
    if rank == 0:
        pk = peaks()
        tflops = cw.flops / (gemm_ms / 1e3) / 1e12
        peak = pk["bf16_tflops"] * 4.0 / (3.0 if cw.wfmt == 0 else 9.0)
        line = {
            "metric": cw.metric, "value": world * cw.flops / (ms / 1e3) / 1e12,
            "unit": "TFLOP/s", "n_gpus": world, "steps": args.steps, "warmup": args.warmup,
            "ms_per_step": ms, "higher_is_better": True, "scaling": "weak", "vs_baseline": None,
            "dtype": "int8 block dot + fp32 accumulate", "data": "synthetic",
            "config": {"workload": cw.name, "M": cw.M, "N": cw.cout, "K": cw.K,
                       "images": cw.images, "map": f"{cw.H}x{cw.W}x{cw.cin}",
                       "kernel": f"{cw.kh}x{cw.kh}", "format": FMT_NAMES[cw.wfmt], "bias": True,
                       "mode": args.mode, "activations": "fp32 NHWC map, encoded and gathered "
                                                         "on device each step",
                       "l2": f"{cw.instances} instances rotated, ~"
                             f"{cw.instances * (cw.bytes_step() + cw.M * cw.K * 1.5) / 1e6:.0f}"
                             " MB > 2 x 126 MB L2",
                       "parallelism": f"replicas x{world}"},
            "roofline": {"bound": "tensor", "kernel": "k_gemm_mxf4" if mode == capi.MODE_FAST
                         else exact_kernel(cw.wfmt), "achieved": tflops, "peak": pk["bf16_tflops"],
                         "unit": "TFLOP/s", "frac": tflops / pk["bf16_tflops"],
                         "peak_source": pk["source"] + " (cuBLAS BF16 dense)",
                         **tensor_fracs(tflops, pk, cw.wfmt),
                         "useful_ceiling": {"peak": peak, "frac": tflops / peak,
                                            "how": "cuBLAS BF16 x 4/3: FP4 MMA rate over three "
                                                   "digit planes" if cw.wfmt == 0 else
                                                   "cuBLAS BF16 x 4/9: FP4 MMA rate over 3 x 3 "
                                                   "digit planes"},
                         "alg_flops_per_launch": cw.flops, "traffic": None,
                         "launch_ms": gemm_ms},
            "encoder": {"kernels": ("k_quantize_planes (map; the GEMM gathers its blocks)"
                                    if cw.wfmt == 0 else
                                    "k_quantize_planes (map) + k_conv_gather_tiles")
                                   if mode == capi.MODE_FAST else "encoder + im2col",
                        "launch_ms": prep_ms, "per_kernel_ms": kernel_ms},
            "e2e": e2e, "gpu_launches": launches, "clocks": clocks.summary(),
        }
        if not args.no_cpu_baseline:
            line["cpu_baseline"] = {k: v for k, v in conv_cpu_reference(cw).items()
                                    if k != "seconds"}
        print(json.dumps(line), flush=True)
    for t in inst:
        t["plan"].close()
    lib.close()
    if dist is not None:
        dist.barrier()
        dist.destroy_process_group()


def prefix_operands(pw: PrefixWorkload, stream_id: int):
    """Per layer and GEMM: weights in the dense formats (W8 placed from
    per-channel int8 the way hotarubi's compiler places it, MXFP4 through
    CanonicalMxfp4) and per group one FP32 input of RMS-1 rows."""
    from hotarubi_b200 import workloads
    layers = []
    for layer in range(pw.layers):
        seed = 10000 * (stream_id + 1) + 100 * layer
        gemms = []
        for j, (name, wfmt, k, n, group) in enumerate(pw.gemms):
            if wfmt == 1:
                q, sc = workloads.w8_per_channel(seed + j, n, k)
                w, ws = place_w8(workloads.dequantize_per_channel(q, sc))
            else:
                w, ws = workloads.mxfp4_weights(seed + j, n, k)
            gemms.append((name, wfmt, k, n, group, w, ws))
        inputs = {}
        for _, _, k, _, group in pw.gemms:
            if group not in inputs:
                x = workloads.activations(seed + 50 + group, pw.M, k)
                x /= np.sqrt(np.mean(x.astype(np.float64) ** 2, axis=1, keepdims=True)).astype(
                    np.float32)
                inputs[group] = x
        layers.append((gemms, inputs))
    return layers


def prefix_cpu_reference(pw: PrefixWorkload, min_seconds: float = 1.0) -> dict:
    """The reference's ExecuteGemm (oracle/_ref) on one layer's seven GEMM
    shapes at M = 141 (cpu_reference per shape); the stream's rate is its
    flops over the summed per-shape times (all layers have the same shapes)."""
    total_s = 0.0
    layer_flops = 0
    parts = []
    for name, wfmt, k, n, _ in pw.gemms:
        wl = Workload(f"c3{name}", f"c3_{name}", f"C3 {name} {pw.M}x{k}x{n}", wfmt, pw.M, n, k,
                      False, 1, "hbm")
        r = cpu_reference(wl, min_seconds=min_seconds, max_reps=20)
        flops = 2 * pw.M * n * k
        total_s += flops / (r["value"] * 1e12)
        layer_flops += flops
        parts.append(r)
    return {"value": layer_flops / total_s / 1e12, "unit": "TFLOP/s", "cores": parts[0]["cores"],
            "kind": parts[0]["kind"],
            "sample": f"one layer's 7 GEMMs ({pw.M} rows) through ExecuteGemm tiles on "
                      f"{parts[0]['cores']} threads, each timed >= {min_seconds} s",
            "seconds": total_s}


def run_prefix(args, rank: int, world: int, local_rank: int) -> None:
    """--config c3: the 16-layer prefix stream as 64 dependent plan runs (one
    plan per layer and group) captured in a CUDA graph; one step = one
    stream.  Two independent streams alternate so that no step finds its
    weights (about 118 MB) in L2.  Replicas for N > 1 (weak scaling)."""
    import torch

    from hotarubi_b200 import capi
    pw = PREFIX
    if args.impl == "reference":
        if rank != 0:
            return
        # Each run times the seven shapes (about 2 s of CPU work): a few runs.
        warm, timed = min(args.warmup, 1), max(1, min(args.steps, 5))
        runs = [prefix_cpu_reference(pw, 0.25) for _ in range(warm + timed)]
        runs = runs[warm:]
        value = statistics.median(r["value"] for r in runs)
        base = runs[-1]
        print(json.dumps({
            "impl": "reference", "metric": pw.metric, "value": value, "unit": "TFLOP/s",
            "n_gpus": args.gpus, "steps": args.steps, "warmup": args.warmup,
            "ms_per_step": pw.flops / (value * 1e12) * 1e3,
            "higher_is_better": True, "scaling": "weak", "vs_baseline": None,
            "dtype": "int8 block dot + fp32 accumulate", "data": "synthetic",
            "config": {"workload": pw.name, "sample": base["sample"]},
            "cpu_baseline": {k: v for k, v in base.items() if k != "seconds"} | {"value": value},
            "e2e": {"value": value, "unit": "TFLOP/s", "h2d_bytes_per_step": 0,
                    "d2h_bytes_per_step": 0}}), flush=True)
        return
    torch.cuda.set_device(local_rank)
    dist = None
    if world > 1:
        import datetime

        import torch.distributed as dist
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=120),
                                device_id=torch.device("cuda", local_rank))
    lib = capi.Library(local_rank)
    mode = capi.MODE_FAST if args.mode == "fast" else capi.MODE_EXACT
    stream = torch.cuda.Stream()
    lib.set_stream(stream.cuda_stream)
    streams = []
    keep = []
    for sid in range(pw.streams):
        plans, first_x, last_c = [], None, None
        for gemms, inputs in prefix_operands(pw, sid):
            xs = {g: torch.from_numpy(x).cuda() for g, x in inputs.items()}
            keep.append(xs)
            for group in range(4):
                descs = []
                for name, wfmt, k, n, g, w, ws in gemms:
                    if g != group:
                        continue
                    t = {"w": torch.from_numpy(w).cuda(), "ws": torch.from_numpy(ws).cuda(),
                         "c": torch.zeros((pw.M, n), dtype=torch.float32, device="cuda")}
                    keep.append(t)
                    descs.append(capi.Library.desc(wfmt, pw.M, n, k, a=xs[group], w=t["w"],
                                                   wscale=t["ws"], c=t["c"], mode=mode))
                    last_c = t["c"]
                plans.append(lib.plan(descs))
            if first_x is None:
                first_x = xs[0]
        streams.append({"plans": plans, "x0": first_x, "c_last": last_c})
    torch.cuda.synchronize()
    # Warm-up outside the graph (kernel attributes are set on first launch),
    # then one graph per stream.
    launches_per_step = 0
    for st in streams:
        launches_per_step = sum(pl.run(stream.cuda_stream) for pl in st["plans"])
    stream.synchronize()
    graphs = []
    for st in streams:
        g = torch.cuda.CUDAGraph()
        with torch.cuda.graph(g, stream=stream):
            for pl in st["plans"]:
                pl.run(stream.cuda_stream)
        graphs.append(g)
    torch.cuda.synchronize()
    # The heaviest launch: the MLP's gate + up GEMMs (group 2), profiled alone.
    per_plan = streams[0]["plans"][2].profile(reps=20, stream=stream.cuda_stream)
    gemm_ms = per_plan[-1] if mode == capi.MODE_FAST else max(per_plan)
    if dist is not None:
        dist.barrier()
    with ClockSampler(local_rank) as clocks:
        with torch.cuda.stream(stream):
            for i in range(args.warmup):
                graphs[i % pw.streams].replay()
        stream.synchronize()
        if dist is not None:
            dist.barrier()
        torch.cuda.synchronize()
        start = torch.cuda.Event(enable_timing=True)
        end = torch.cuda.Event(enable_timing=True)
        with torch.cuda.stream(stream):
            start.record(stream)
            for i in range(args.steps):
                graphs[i % pw.streams].replay()
            end.record(stream)
        end.synchronize()
        if dist is not None:
            dist.barrier()
    lib.sync()
    ms = start.elapsed_time(end) / args.steps
    if dist is not None:
        t = torch.tensor([ms], device="cuda")
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        ms = float(t.item())
    # End to end: the first layer's input from pinned host memory, the
    # stream, the last GEMM's output back.
    e2e = None
    if not args.no_e2e:
        st = streams[0]
        xh = st["x0"].cpu().pin_memory()
        ch = torch.empty(tuple(st["c_last"].shape), dtype=torch.float32).pin_memory()
        n_e2e = max(1, min(args.steps, 10))
        for k in range(2 + n_e2e):
            if k == 2:
                stream.synchronize()
                w0 = time.perf_counter()
            with torch.cuda.stream(stream):
                st["x0"].copy_(xh, non_blocking=True)
                graphs[0].replay()
                ch.copy_(st["c_last"], non_blocking=True)
            stream.synchronize()
        dt = (time.perf_counter() - w0) / n_e2e
        e2e = {"value": world * pw.flops / dt / 1e12, "unit": "TFLOP/s",
               "h2d_bytes_per_step": world * xh.numel() * 4,
               "d2h_bytes_per_step": world * ch.numel() * 4, "ms_per_step": dt * 1e3,
               "entry_point": "pinned copies + the stream's hrb_plan_run calls in a CUDA graph "
                              "(weights resident)"}
    if rank == 0:
        pk = peaks()
        mlp_bytes = sum(pw.gemm_bytes(wfmt, k, n) for _, wfmt, k, n, g in pw.gemms if g == 2)
        achieved = mlp_bytes / (gemm_ms / 1e3) / 1e9
        w_bytes = pw.layers * sum((n * k // 2 if wfmt == 0 else n * k) + n * ((k + 31) // 32)
                                  for _, wfmt, k, n, _ in pw.gemms)
        line = {
            "metric": pw.metric, "value": world * pw.flops / (ms / 1e3) / 1e12,
            "unit": "TFLOP/s", "n_gpus": world, "steps": args.steps, "warmup": args.warmup,
            "ms_per_step": ms, "higher_is_better": True, "scaling": "weak", "vs_baseline": None,
            "dtype": "int8 block dot + fp32 accumulate", "data": "synthetic",
            "config": {"workload": pw.name, "M": pw.M, "layers": pw.layers,
                       "gemms_per_layer": "q k v (w8) | o (w8) | gate up (mxfp4) | down (mxfp4)",
                       "formats": "w8 + mxfp4", "bias": False, "mode": args.mode,
                       "activations": "fp32 per group, encoded on device each step",
                       "l2": f"{pw.streams} streams alternated, {w_bytes / 1e6:.0f} MB of "
                             "weights each",
                       "parallelism": f"replicas x{world}",
                       "launch": f"{pw.layers * 4} dependent plan runs in a CUDA graph"},
            "roofline": {"bound": "hbm", "kernel": "k_gemm_mxf4 (gate + up, one launch)"
                         if mode == capi.MODE_FAST else exact_kernel(0),
                         "achieved": achieved, "peak": pk["hbm_gbs"], "unit": "GB/s",
                         "frac": achieved / pk["hbm_gbs"], "peak_source": pk["source"] +
                         " (HBM copy)", "alg_bytes_per_launch": mlp_bytes, "traffic": None,
                         "launch_ms": gemm_ms},
            "e2e": e2e, "gpu_launches": launches_per_step * args.steps,
            "clocks": clocks.summary(),
        }
        if not args.no_cpu_baseline:
            line["cpu_baseline"] = {k: v for k, v in prefix_cpu_reference(pw).items()
                                    if k != "seconds"}
        print(json.dumps(line), flush=True)
    del graphs
    for st in streams:
        for pl in st["plans"]:
            pl.close()
    lib.close()
    if dist is not None:
        dist.barrier()
        dist.destroy_process_group()


def gacc_operands(gw: GaccWorkload, i: int):
    rng = np.random.default_rng(800 + i)
    rows = rng.integers(0, 256, (gw.nrows, gw.row_stride), dtype=np.uint8)
    rows[:, 32 * gw.blocks:33 * gw.blocks] = rng.integers(118, 134, (gw.nrows, gw.blocks))
    idx = rng.integers(0, gw.nrows, (gw.tokens, gw.slots, gw.corners)).astype(np.uint64)
    idx[:, 52::56, :] = 0xFFFFFFFF      # the 4 padding slots of each camera are null
    idx[:, 53::56, :] = 0xFFFFFFFF
    idx[:, 54::56, :] = 0xFFFFFFFF
    idx[:, 55::56, :] = 0xFFFFFFFF
    bw = (rng.random((gw.tokens, gw.slots, gw.corners)).astype(np.float32) * 0.25)
    w = rng.random((gw.tokens, gw.slots, gw.blocks)).astype(np.float32) / 52.0
    entries = idx | (bw.view(np.uint32).astype(np.uint64) << np.uint64(32))
    return entries, w, rows


def run_gacc(args, rank: int, world: int, local_rank: int) -> None:
    """--config gacc: hrb_gacc_dense on the SparseDrive detection head's
    sampling (replicas for N > 1, weak scaling).  The metric is the gathered
    feature-row bytes per second; the FP32 chain adds 2 flops per gathered
    code."""
    import torch

    from hotarubi_b200 import capi
    gw = GACC
    live = gw.entries - gw.tokens * 6 * 4 * gw.corners   # null padding slots excluded
    def cpu_sample(reps: int, warm: int):
        """The C restatement on 1 thread over 16 of the tokens (GB/s, s)."""
        from oracle import cpu
        e, w, rows = gacc_operands(gw, 0)
        sample = 16
        runs = []
        for _ in range(warm + reps):
            t0 = time.perf_counter()
            cpu.gacc_dense(e[:sample], w[:sample].view(np.uint32), rows, gw.blocks)
            runs.append(time.perf_counter() - t0)
        dt = statistics.median(runs[warm:])
        return (live * sample / gw.tokens * gw.blocks * 33 / dt / 1e9, dt,
                f"{sample} of {gw.tokens} tokens through the C restatement on 1 thread")

    if args.impl == "reference":
        if rank != 0:
            return
        value, dt, desc = cpu_sample(args.steps, args.warmup)
        print(json.dumps({
            "impl": "reference", "metric": gw.metric, "value": value, "unit": "GB/s",
            "n_gpus": args.gpus, "steps": args.steps, "warmup": args.warmup,
            "ms_per_step": dt * 1e3, "higher_is_better": True, "scaling": "weak",
            "vs_baseline": None, "dtype": "fp32 chain over int8 rows", "data": "synthetic",
            "config": {"workload": gw.name, "sample": desc},
            "cpu_baseline": {"value": value, "unit": "GB/s", "cores": 1, "kind": "port",
                             "sample": desc},
            "e2e": {"value": value, "unit": "GB/s", "h2d_bytes_per_step": 0,
                    "d2h_bytes_per_step": 0}}), flush=True)
        return
    torch.cuda.set_device(local_rank)
    dist = None
    if world > 1:
        import datetime

        import torch.distributed as dist
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=120),
                                device_id=torch.device("cuda", local_rank))
    lib = capi.Library(local_rank)
    stream = torch.cuda.Stream()
    lib.set_stream(stream.cuda_stream)
    inst = []
    for i in range(gw.instances):
        e, w, rows = gacc_operands(gw, i)
        inst.append({"e": torch.from_numpy(e.view(np.int64)).cuda(),
                     "w": torch.from_numpy(w).cuda(), "rows": torch.from_numpy(rows).cuda(),
                     "out": torch.zeros((gw.tokens, gw.blocks * 32), device="cuda")})

    def launch(t):
        lib.gacc(t["e"], t["w"], t["rows"], t["out"], tokens=gw.tokens, slots=gw.slots,
                 corners=gw.corners, blocks=gw.blocks, row_stride=gw.row_stride,
                 nrows=gw.nrows, stream=stream.cuda_stream)

    torch.cuda.synchronize()
    if dist is not None:
        dist.barrier()
    with ClockSampler(local_rank) as clocks:
        for i in range(args.warmup):
            launch(inst[i % gw.instances])
        stream.synchronize()
        if dist is not None:
            dist.barrier()
        start = torch.cuda.Event(enable_timing=True)
        end = torch.cuda.Event(enable_timing=True)
        start.record(stream)
        for i in range(args.steps):
            launch(inst[i % gw.instances])
        end.record(stream)
        end.synchronize()
        if dist is not None:
            dist.barrier()
    lib.sync()
    ms = start.elapsed_time(end) / args.steps
    if dist is not None:
        t = torch.tensor([ms], device="cuda")
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        ms = float(t.item())
    e2e = None
    if not args.no_e2e:
        e, w, _ = gacc_operands(gw, 0)
        eh = torch.from_numpy(e.view(np.int64)).pin_memory()
        wh = torch.from_numpy(w).pin_memory()
        oh = torch.empty((gw.tokens, gw.blocks * 32)).pin_memory()
        t0 = inst[0]
        n_e2e = max(1, min(args.steps, 10))
        for k in range(2 + n_e2e):
            if k == 2:
                stream.synchronize()
                w0 = time.perf_counter()
            with torch.cuda.stream(stream):
                t0["e"].copy_(eh, non_blocking=True)
                t0["w"].copy_(wh, non_blocking=True)
                launch(t0)
                oh.copy_(t0["out"], non_blocking=True)
            stream.synchronize()
        dt = (time.perf_counter() - w0) / n_e2e
        e2e = {"value": world * live * gw.blocks * 33 / dt / 1e9, "unit": "GB/s",
               "h2d_bytes_per_step": world * (eh.numel() * 8 + wh.numel() * 4),
               "d2h_bytes_per_step": world * oh.numel() * 4, "ms_per_step": dt * 1e3,
               "entry_point": "pinned copies of entries and coefficients + hrb_gacc_dense "
                              "(feature rows resident)"}
    if rank == 0:
        pk = peaks()
        gbs = world * live * gw.blocks * 33 / (ms / 1e3) / 1e9
        per_gpu = live * gw.blocks * 33 / (ms / 1e3) / 1e9
        line = {
            "metric": gw.metric, "value": gbs, "unit": "GB/s", "n_gpus": world,
            "steps": args.steps, "warmup": args.warmup, "ms_per_step": ms,
            "higher_is_better": True, "scaling": "weak", "vs_baseline": None,
            "dtype": "fp32 chain over int8 rows (bit-exact)", "data": "synthetic",
            "config": {"workload": gw.name, "tokens": gw.tokens, "slots": gw.slots,
                       "corners": gw.corners, "channels": gw.blocks * 32,
                       "feature_rows": gw.nrows, "live_entries": live,
                       "l2": f"{gw.instances} instances rotated (> 2 x 126 MB L2)",
                       "parallelism": f"replicas x{world}"},
            "roofline": {"bound": "hbm", "kernel": "k_gacc", "achieved": per_gpu,
                         "peak": pk["hbm_gbs"], "unit": "GB/s", "frac": per_gpu / pk["hbm_gbs"],
                         "peak_source": pk["source"] + " (HBM copy; a 24 MB row table is "
                                                       "gathered mostly from L2)",
                         "alg_bytes_per_launch": live * gw.blocks * 33, "traffic": None,
                         "launch_ms": ms},
            "gflops": live * gw.blocks * 32 * 2 / (ms / 1e3) / 1e9,
            "e2e": e2e, "gpu_launches": args.steps, "clocks": clocks.summary(),
        }
        if not args.no_cpu_baseline:
            value, _, desc = cpu_sample(3, 1)
            line["cpu_baseline"] = {"value": value, "unit": "GB/s", "cores": 1, "kind": "port",
                                    "sample": desc}
        print(json.dumps(line), flush=True)
    lib.close()
    if dist is not None:
        dist.barrier()
        dist.destroy_process_group()


def run_shard(args, wl: Workload, rank: int, world: int, local_rank: int) -> None:
    """--shard: the batch's GEMMs split along N over the ranks (strong
    scaling: the total work is fixed); every rank's kernel also stores its
    outputs into all other ranks' C over NVLink (the all-gather fused into
    the GEMM), and a step ends when every rank holds all of C."""
    import datetime

    import torch
    import torch.distributed as dist

    from hotarubi_b200 import capi, shard
    torch.cuda.set_device(local_rank)
    dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=120),
                            device_id=torch.device("cuda", local_rank))
    lib = capi.Library(local_rank)
    stream = torch.cuda.Stream()
    lib.set_stream(stream.cuda_stream)
    group = shard.Group(lib)   # the library's communicator (NCCL through the C ABI)
    batch = args.batch or wl.batch
    n0, n1 = shard.columns(wl.N)
    mx = args.gather == "mxint8"
    kpn = (wl.N + 31) // 32 * 32
    # --gather mxint8: each GEMM keeps only its MXINT8 copy (1 + 1/32 bytes an
    # output, the next layer's activation format), written in the full
    # matrix's layout (ldcq) into every rank's buffer.
    out = (shard.PeerOutput(lib, group, (1,), mx_shape=(batch * wl.M, kpn)) if mx
           else shard.PeerOutput(lib, group, (batch, wl.M, wl.N)))
    sets = [host_operands(wl, i) for i in range(min(4, batch))]
    keep, descs = [], []
    a_all = torch.empty((batch, wl.M, wl.K), dtype=torch.float32, device="cuda")
    for b in range(batch):
        x, w, ws, bias = sets[b % len(sets)]
        a_all[b].copy_(torch.from_numpy(x))
        t = [torch.from_numpy(w[n0:n1].copy()).cuda(), torch.from_numpy(ws[n0:n1].copy()).cuda(),
             None if bias is None else torch.from_numpy(bias[n0:n1].copy()).cuda()]
        keep += t
        if n1 > n0 and mx:
            rows = slice(b * wl.M, (b + 1) * wl.M)
            descs.append(capi.Library.desc(wl.wfmt, wl.M, n1 - n0, wl.K, a=a_all[b], w=t[0],
                                           wscale=t[1], bias=t[2], c=None,
                                           cq=out.q[rows].data_ptr() + n0,
                                           cscale=out.s[rows].data_ptr() + n0 // 32,
                                           ldcq=kpn, mode=capi.MODE_FAST))
        elif n1 > n0:
            descs.append(capi.Library.desc(wl.wfmt, wl.M, n1 - n0, wl.K, a=a_all[b], w=t[0],
                                           wscale=t[1], bias=t[2],
                                           c=out.tensor[b].data_ptr() + 4 * n0, ldc=wl.N,
                                           mode=capi.MODE_FAST))
    plan = lib.plan(descs) if descs else None
    if plan is not None:
        plan.set_peers(out.ptr, out.peer_bases)
    torch.cuda.synchronize()

    def step():
        if plan is not None:
            plan.run(stream.cuda_stream)
        group.fence(stream.cuda_stream)  # the step ends when every rank's stores are done

    dist.barrier()
    with ClockSampler(local_rank) as clocks:
        for _ in range(args.warmup):
            step()
        stream.synchronize()
        dist.barrier()
        start = torch.cuda.Event(enable_timing=True)
        end = torch.cuda.Event(enable_timing=True)
        start.record(stream)
        for _ in range(args.steps):
            step()
        end.record(stream)
        end.synchronize()
        dist.barrier()
    ms = start.elapsed_time(end) / args.steps
    t = torch.tensor([ms], device="cuda")
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    ms = float(t.item())
    if rank == 0:
        pk = peaks()
        per_out = (1 + 1 / 32) if mx else 4                       # bytes an output crosses
        nvlink = (world - 1) * batch * wl.M * wl.N * per_out / world  # each rank to its peers
        line = {
            "metric": wl.metric, "value": batch * wl.flops / (ms / 1e3) / 1e12,
            "unit": "TFLOP/s", "n_gpus": world, "steps": args.steps, "warmup": args.warmup,
            "ms_per_step": ms, "higher_is_better": True, "scaling": "strong",
            "vs_baseline": None, "dtype": "int8 block dot + fp32 accumulate",
            "data": "synthetic",
            "config": {"workload": wl.name, "batch": batch, "M": wl.M, "N": wl.N, "K": wl.K,
                       "format": FMT_NAMES[wl.wfmt], "mode": "fast",
                       "gather": ("MXINT8 copy (1 + 1/32 B an output, the FP32 output "
                                  "not kept)" if mx else "FP32 output"),
                       "parallelism": f"N-sharded x{world}, all-gather fused into the GEMM "
                                      "epilogue (NVLink peer stores)"},
            "nvlink": {"bytes_per_rank_per_step": nvlink,
                       "gbs_per_rank": nvlink / (ms / 1e3) / 1e9},
            **{"per_gpu_" + k: v for k, v in tensor_fracs(
                batch * wl.flops / world / (ms / 1e3) / 1e12, pk, wl.wfmt).items()},
            "gpu_launches": 2 * args.steps if plan is not None else 0,
            "e2e": None, "clocks": clocks.summary(),
        }
        print(json.dumps(line), flush=True)
    dist.barrier()
    if plan is not None:
        plan.close()
    torch.cuda.synchronize()
    dist.barrier()
    out.close()
    group.close()
    lib.close()
    dist.destroy_process_group()


def run_conv_shard(args, rank: int, world: int, local_rank: int) -> None:
    """--config c5conv --shard: the C5 conv's 48 images split over the ranks
    (shard.rows; strong scaling, the total work is fixed).  Each rank's conv
    plan covers its images and its epilogue stores every output row into all
    ranks' C over NVLink (the all-gather along M fused into the kernel,
    ConvPlan.set_peers); a step ends when every rank holds all 33,792 rows
    (Group.fence)."""
    import datetime

    import torch
    import torch.distributed as dist

    from hotarubi_b200 import capi, shard
    cw = CONVS[args.config]
    torch.cuda.set_device(local_rank)
    dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=120),
                            device_id=torch.device("cuda", local_rank))
    lib = capi.Library(local_rank)
    stream = torch.cuda.Stream()
    lib.set_stream(stream.cuda_stream)
    group = shard.Group(lib)
    per = (cw.H // cw.stride) * (cw.W // cw.stride)
    i0, i1 = shard.rows(cw.images)
    x, w, ws, b = conv_operands(cw, 0)
    hw = cw.H * cw.W
    out = shard.PeerOutput(lib, group, (cw.M, cw.cout))
    t = {"x": torch.from_numpy(x[i0 * hw:i1 * hw].copy()).cuda(), "w": torch.from_numpy(w).cuda(),
         "ws": torch.from_numpy(ws).cuda(), "b": torch.from_numpy(b).cuda()}
    plan = None
    if i1 > i0:
        d = capi.conv_desc(cw.wfmt, i1 - i0, cw.H, cw.W, cw.cin, cw.cout, cw.kh, cw.stride,
                           order=capi.CONV_YMAJOR, a=t["x"], w=t["w"], wscale=t["ws"],
                           bias=t["b"], c=out.tensor[i0 * per:i1 * per], mode=capi.MODE_FAST)
        plan = lib.conv_plan(d)
        plan.set_peers(out.ptr, out.peer_bases)
    torch.cuda.synchronize()

    def step():
        n = plan.run(stream.cuda_stream) if plan is not None else 0
        group.fence(stream.cuda_stream)
        return n

    dist.barrier()
    with ClockSampler(local_rank) as clocks:
        for _ in range(args.warmup):
            step()
        stream.synchronize()
        dist.barrier()
        start = torch.cuda.Event(enable_timing=True)
        end = torch.cuda.Event(enable_timing=True)
        start.record(stream)
        launches = 0
        for _ in range(args.steps):
            launches += step()
        end.record(stream)
        end.synchronize()
        dist.barrier()
    ms = start.elapsed_time(end) / args.steps
    tm = torch.tensor([ms], device="cuda")
    dist.all_reduce(tm, op=dist.ReduceOp.MAX)
    ms = float(tm.item())
    if rank == 0:
        nvlink = (world - 1) * cw.M * cw.cout * 4 / world   # bytes each rank stores to peers
        print(json.dumps({
            "metric": cw.metric, "value": cw.flops / (ms / 1e3) / 1e12, "unit": "TFLOP/s",
            "n_gpus": world, "steps": args.steps, "warmup": args.warmup, "ms_per_step": ms,
            "higher_is_better": True, "scaling": "strong", "vs_baseline": None,
            "dtype": "int8 block dot + fp32 accumulate", "data": "synthetic",
            "config": {"workload": cw.name, "M": cw.M, "N": cw.cout, "K": cw.K,
                       "images": cw.images, "format": FMT_NAMES[cw.wfmt], "bias": True,
                       "mode": "fast",
                       "parallelism": f"M-sharded (images) x{world}, all-gather along M fused "
                                      "into the GEMM epilogue (NVLink peer stores)"},
            "nvlink": {"bytes_per_rank_per_step": nvlink,
                       "gbs_per_rank": nvlink / (ms / 1e3) / 1e9},
            "gpu_launches": launches, "e2e": None, "clocks": clocks.summary()}), flush=True)
    dist.barrier()
    if plan is not None:
        plan.close()
    torch.cuda.synchronize()
    dist.barrier()
    out.close()
    group.close()
    lib.close()
    dist.destroy_process_group()


# ---------------------------------------------------------------------------
# C4: the action expert's whole job

def expert_cpu_reference(ew: ExpertWorkload, min_seconds: float = 0.5) -> dict:
    """The reference has no MXFP8 path, so the oracle's C restatement (one
    thread) stands in: one request's self-attention layer (7 GEMMs at 50
    rows) and one cross-attention K/V pair (141 rows), each timed; the job's
    rate is its FLOPs over the time those shapes predict."""
    secs = {}
    parts = []
    for label, gm in list(ew.self_layer) + [("kv", ew.cross_kv)]:
        for name, k, n in gm:
            m = ew.prefix if label == "kv" else ew.tokens
            wl = Workload(f"c4{name}", f"c4_{name}", f"C4 {name} {m}x{k}x{n}", ew.wfmt, m, n, k,
                          False, 1, "tensor")
            r = cpu_reference(wl, min_seconds=min_seconds, max_reps=5)
            secs[(m, k, n)] = 2 * m * k * n / (r["value"] * 1e12)
            parts.append(r)

    def t(m, k, n):  # seconds for m rows of (k, n), scaled from the timed rows
        base = ew.prefix if (k, n) in [(kk, nn) for _, kk, nn in ew.cross_kv] else ew.tokens
        key = next((x for x in secs if x[0] == base and x[1:] == (k, n)), None)
        if key is None:  # the heads: the closest timed shape by MACs
            key = min(secs, key=lambda x: abs(x[1] * x[2] - k * n))
            return secs[key] * (m * k * n) / (key[0] * key[1] * key[2])
        return secs[key] * m / key[0]

    m, mp = ew.rows(1)
    total = ew.steps * sum(t(m, k, n) for _, gm in ew.step_groups() for _, k, n in gm)
    total += (ew.layers // 2) * sum(t(mp, k, n) for _, k, n in ew.cross_kv)
    return {"value": ew.flops() / total / 1e12, "unit": "TFLOP/s", "cores": 1, "kind": "port",
            "sample": "one request's self-attention layer (7 GEMMs, 50 rows) and one "
                      "cross K/V pair (141 rows) through the oracle's MXFP8 chain on 1 thread "
                      "(the reference has no MXFP8), scaled to the job's shapes",
            "seconds": total}


def run_expert(args, rank: int, world: int, local_rank: int) -> None:
    """--config c4: the action expert's job (ExpertWorkload) as one CUDA graph
    of plan runs: the cross K/V plan, then per flow step the 68 dependency
    groups in order.  The requests split over the ranks (strong scaling,
    no collective: requests are independent)."""
    import torch

    from hotarubi_b200 import capi, workloads
    ew = EXPERT
    if args.impl == "reference":
        if rank != 0:
            return
        warm, timed = min(args.warmup, 1), max(1, min(args.steps, 5))
        runs = [expert_cpu_reference(ew, 0.2) for _ in range(warm + timed)][warm:]
        value = statistics.median(r["value"] for r in runs)
        base = runs[-1]
        print(json.dumps({
            "impl": "reference", "metric": ew.metric, "value": value, "unit": "TFLOP/s",
            "n_gpus": args.gpus, "steps": args.steps, "warmup": args.warmup,
            "ms_per_step": ew.flops() / (value * 1e12) * 1e3,
            "higher_is_better": True, "scaling": "strong", "vs_baseline": None,
            "dtype": "e4m3 x int8 block dot + fp32 accumulate", "data": "synthetic",
            "config": {"workload": ew.name, "sample": base["sample"]},
            "cpu_baseline": {k: v for k, v in base.items() if k != "seconds"} | {"value": value},
            "e2e": {"value": value, "unit": "TFLOP/s", "h2d_bytes_per_step": 0,
                    "d2h_bytes_per_step": 0}}), flush=True)
        return
    torch.cuda.set_device(local_rank)
    dist = None
    if world > 1:
        import datetime

        import torch.distributed as dist
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=120),
                                device_id=torch.device("cuda", local_rank))
    lib = capi.Library(local_rank)
    mode = capi.MODE_FAST if args.mode == "fast" else capi.MODE_EXACT
    stream = torch.cuda.Stream()
    lib.set_stream(stream.cuda_stream)
    m, mp = ew.rows(world)
    gen = torch.Generator(device="cuda")

    def synthetic(seed, rows, k):
        gen.manual_seed(seed)
        x = torch.randn((rows, k), generator=gen, device="cuda", dtype=torch.float32)
        return x / x.pow(2).mean(dim=1, keepdim=True).sqrt()

    keep = []

    def group_plan(seed, rows, gemms, separate_inputs=False):
        """One plan over a dependency group's GEMMs (one shared input)."""
        x = None
        descs = []
        for j, (name, k, n) in enumerate(gemms):
            if x is None or separate_inputs:
                x = synthetic(seed + 97 * j, rows, k)
            kp = (k + 31) // 32 * 32
            w, ws = workloads.mxfp8_weights(seed + j, n, kp)
            w[:, k:] = 0
            t = {"x": x, "w": torch.from_numpy(w).cuda(), "ws": torch.from_numpy(ws).cuda(),
                 "c": torch.empty((rows, n), dtype=torch.float32, device="cuda")}
            keep.append(t)
            descs.append(capi.Library.desc(ew.wfmt, rows, n, k, a=t["x"], w=t["w"],
                                           wscale=t["ws"], c=t["c"], mode=mode))
        return lib.plan(descs)

    # Cross K/V of the prefix: the 8 cross layers' K and V projections in one
    # plan (independent GEMMs), each layer's prefix states its own input.
    kv_descs = []
    for layer in range(1, ew.layers, 2):
        for j, (name, k, n) in enumerate(ew.cross_kv):
            if j == 0:
                x = synthetic(50_000 + layer, mp, k)
            w, ws = workloads.mxfp8_weights(60_000 + 10 * layer + j, n, k)
            t = {"x": x, "w": torch.from_numpy(w).cuda(), "ws": torch.from_numpy(ws).cuda(),
                 "c": torch.empty((mp, n), dtype=torch.float32, device="cuda")}
            keep.append(t)
            kv_descs.append(capi.Library.desc(ew.wfmt, mp, n, k, a=t["x"], w=t["w"],
                                              wscale=t["ws"], c=t["c"], mode=mode))
    kv_plan = lib.plan(kv_descs)
    kv_inputs = [t["x"] for t in keep[::2]]
    plans = []
    labels = []
    for gi, (label, gemms) in enumerate(ew.step_groups()):
        plans.append(group_plan(1000 * (gi + 1), m, gemms,
                                separate_inputs=label == "head.time_mlp_in"))
        labels.append(label)
    x_noise = keep[len(kv_descs)]["x"]          # action_in's input (the noise x_t)
    v_out = keep[-1]["c"]                      # action_out's output (the velocity)
    torch.cuda.synchronize()

    def job(s):
        n = kv_plan.run(s)
        for _ in range(ew.steps):
            for pl in plans:
                n += pl.run(s)
        return n

    launches_per_job = job(stream.cuda_stream)   # warm (kernel attributes set)
    stream.synchronize()
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph, stream=stream):
        job(stream.cuda_stream)
    torch.cuda.synchronize()
    # The heaviest group: a layer's gate + up, profiled alone.
    gu = labels.index("L0.gate_up")
    per_plan = plans[gu].profile(reps=20, stream=stream.cuda_stream)
    gemm_ms = per_plan[-1] if mode == capi.MODE_FAST else max(per_plan)
    if dist is not None:
        dist.barrier()
    with ClockSampler(local_rank) as clocks:
        with torch.cuda.stream(stream):
            for _ in range(args.warmup):
                graph.replay()
        stream.synchronize()
        if dist is not None:
            dist.barrier()
        torch.cuda.synchronize()
        marks = [torch.cuda.Event(enable_timing=True) for _ in range(args.steps + 1)]
        with torch.cuda.stream(stream):
            marks[0].record(stream)
            for i in range(args.steps):
                graph.replay()
                marks[i + 1].record(stream)
        marks[-1].synchronize()
        if dist is not None:
            dist.barrier()
    lib.sync()
    ms = marks[0].elapsed_time(marks[-1]) / args.steps
    trials = trial_stats([marks[i].elapsed_time(marks[i + 1]) for i in range(args.steps)])
    if dist is not None:
        t = torch.tensor([ms], device="cuda")
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        ms = float(t.item())
    # End to end: the job's inputs from pinned host memory (the noise and the
    # 8 cross layers' prefix states), the graph, the velocity back.
    e2e = None
    if not args.no_e2e:
        hx = x_noise.cpu().pin_memory()
        hkv = [x.cpu().pin_memory() for x in kv_inputs]
        hv = torch.empty(tuple(v_out.shape), dtype=torch.float32).pin_memory()
        n_e2e = max(1, min(args.steps, 5))
        for k in range(1 + n_e2e):
            if k == 1:
                stream.synchronize()
                w0 = time.perf_counter()
            with torch.cuda.stream(stream):
                x_noise.copy_(hx, non_blocking=True)
                for d, h in zip(kv_inputs, hkv):
                    d.copy_(h, non_blocking=True)
                graph.replay()
                hv.copy_(v_out, non_blocking=True)
            stream.synchronize()
        dt = (time.perf_counter() - w0) / n_e2e
        if dist is not None:
            t = torch.tensor([dt], device="cuda")
            dist.all_reduce(t, op=dist.ReduceOp.MAX)
            dt = float(t.item())
        h2d = hx.numel() * 4 + sum(h.numel() * 4 for h in hkv)
        e2e = {"value": ew.flops(world) / dt / 1e12, "unit": "TFLOP/s",
               "h2d_bytes_per_step": world * h2d, "d2h_bytes_per_step": world * hv.numel() * 4,
               "ms_per_step": dt * 1e3,
               "entry_point": "pinned copies + the job's hrb_plan_run calls in a CUDA graph "
                              "(weights resident)"}
    if rank == 0:
        pk = peaks()
        gu_flops = sum(2 * m * k * n for _, k, n in ew.step_groups()[gu][1])
        tflops = gu_flops / (gemm_ms / 1e3) / 1e12
        w_bytes = sum(n * ((k + 31) // 32) * 33 for _, gm in ew.step_groups() for _, k, n in gm)
        line = {
            "metric": ew.metric, "value": ew.flops(world) / (ms / 1e3) / 1e12,
            "unit": "TFLOP/s", "n_gpus": world, "steps": args.steps, "warmup": args.warmup,
            "ms_per_step": ms, "higher_is_better": True, "scaling": "strong",
            "vs_baseline": None, "dtype": "e4m3 x int8 block dot + fp32 accumulate",
            "data": "synthetic",
            "config": {"workload": ew.name, "requests": ew.requests,
                       "requests_per_gpu": ew.requests // world, "rows_per_gemm": m,
                       "prefix_rows_per_gemm": mp, "flow_steps": ew.steps,
                       "layers": ew.layers, "format": "mxfp8", "bias": False,
                       "mode": args.mode,
                       "activations": "fp32 per dependency group (synthetic, RMS 1 rows), "
                                      "encoded on device by each plan run",
                       "l2": f"activations {m} rows per GEMM, {w_bytes * ew.layers / 1e6:.0f}"
                             " MB of weights per flow step; no flush (the job's own data "
                             "exceeds L2 many times)",
                       "parallelism": f"requests split x{world} (data parallel, no collective)",
                       "launch": f"{1 + ew.steps * len(plans)} plan runs in one CUDA graph"},
            "trials": trials,
            "roofline": {"bound": "tensor",
                         "kernel": "k_gemm_mxf4 (kind::mxf8f6f4; a layer's gate + up, one "
                                   "launch)" if mode == capi.MODE_FAST else "k_dense_exact",
                         "achieved": tflops, "peak": pk["bf16_tflops"], "unit": "TFLOP/s",
                         "frac": tflops / pk["bf16_tflops"],
                         "peak_source": pk["source"] + " (cuBLAS BF16 dense)",
                         **tensor_fracs(tflops, pk, ew.wfmt),
                         "alg_flops_per_launch": gu_flops, "traffic": None,
                         "launch_ms": gemm_ms,
                         # The job runs tens of ms a step, under the power cap: its own
                         # rate against the sustained dense rate of the MMA kind.
                         "job_frac_of_kind_sustained_peak":
                             ew.flops(world) / (ms / 1e3) / 1e12 / world
                             / (2.0 * pk["bf16_tflops_sustained"])},
            "e2e": e2e, "gpu_launches": launches_per_job * args.steps,
            "clocks": clocks.summary(),
        }
        if not args.no_cpu_baseline:
            line["cpu_baseline"] = {k: v for k, v in expert_cpu_reference(ew).items()
                                    if k != "seconds"}
        print(json.dumps(line), flush=True)
    del graph
    kv_plan.close()
    for pl in plans:
        pl.close()
    lib.close()
    if dist is not None:
        dist.barrier()
        dist.destroy_process_group()


# ---------------------------------------------------------------------------
# The C5 sweep: 27 GEMMs and the conv, one command

SWEEP_M = (256, 4096, 65536)
SWEEP_KN = ((960, 2560), (2560, 960), (4096, 4096))
SWEEP_FMTS = (1, 0, 2)   # W8, MXFP4, MXFP8


def sweep_workloads() -> list[Workload]:
    """M x (K, N) x format, each with its config's distributions
    (W8 as C1 with bias, MXFP4 as C2, MXFP8 as C4, no bias)."""
    out = []
    for k, n in SWEEP_KN:
        for m in SWEEP_M:
            for wfmt in SWEEP_FMTS:
                f = FMT_NAMES[wfmt]
                out.append(Workload(f"s_{f}_{m}_{k}_{n}", f"c5sweep_{f}_{m}x{k}x{n}",
                                    f"C5 sweep {m}x{k}x{n}", wfmt, m, n, k, wfmt == 1, 1,
                                    "tensor"))
    return out


def run_sweep(args, rank: int, world: int, local_rank: int) -> None:
    """--config c5sweep (one GPU): every GEMM of the sweep through a plan of B
    instances (B so that a step's operands exceed 2 x L2), W untimed steps,
    then K steps each bracketed by events (the median is the figure); the
    GEMM kernel alone timed over repeated launches (plan profile) for its
    tensor fractions; parity on the first and last rows; then both conv
    formats through run_conv.  Prints one JSON line holding every record and
    writes a markdown table with --summary-md."""
    import contextlib
    import io

    import torch

    from hotarubi_b200 import capi
    if world != 1 or args.impl == "reference":
        if rank == 0:
            print(json.dumps({"impl": args.impl, "config": "c5sweep",
                              "unavailable": "the sweep runs on one GPU through this library"}))
        return
    torch.cuda.set_device(local_rank)
    lib = capi.Library(local_rank)
    stream = torch.cuda.Stream()
    lib.set_stream(stream.cuda_stream)
    pk = peaks()
    records = []
    cpu_rates = {}
    x_cache = {}
    for wl0 in sweep_workloads():
        if args.sweep_filter and not re.search(args.sweep_filter, wl0.key):
            continue
        batch = max(1, -(-320_000_000 // wl0.bytes_step()))
        wl = dataclasses.replace(wl0, batch=batch)
        distinct = min(2, batch)
        sets = []
        for i in range(distinct):
            # The three formats of one shape share their activations.
            key = (wl.M, wl.K, i)
            if key not in x_cache:
                from hotarubi_b200 import workloads
                x_cache = {k2: v for k2, v in x_cache.items() if k2[:2] == key[:2]}
                x_cache[key] = workloads.activations(100 + i, wl.M, wl.K)
            _, w, ws, b = host_operands(dataclasses.replace(wl, M=1), i)
            sets.append((x_cache[key], w, ws, b))
        a_all = torch.empty((batch, wl.M, wl.K), dtype=torch.float32, device="cuda")
        c_all = torch.zeros((batch, wl.M, wl.N), dtype=torch.float32, device="cuda")
        keep = []
        descs = []
        for j in range(batch):
            x, w, ws, b = sets[j % distinct]
            a_all[j].copy_(torch.from_numpy(x))
            t = {"w": torch.from_numpy(w).cuda(), "ws": torch.from_numpy(ws).cuda(),
                 "b": None if b is None else torch.from_numpy(b).cuda()}
            keep.append(t)
            descs.append(capi.Library.desc(wl.wfmt, wl.M, wl.N, wl.K, a=a_all[j], w=t["w"],
                                           wscale=t["ws"], bias=t["b"], c=c_all[j],
                                           mode=capi.MODE_FAST))
        plan = lib.plan(descs)
        torch.cuda.synchronize()
        kernel_ms = plan.profile(reps=max(3, min(20, int(2e13 / (batch * wl.flops)))),
                                 stream=stream.cuda_stream)
        gemm_ms = sum(kernel_ms[1:])
        with ClockSampler(local_rank) as clocks:
            for _ in range(args.warmup):
                plan.run(stream.cuda_stream)
            marks = [torch.cuda.Event(enable_timing=True) for _ in range(args.steps + 1)]
            marks[0].record(stream)
            for i in range(args.steps):
                plan.run(stream.cuda_stream)
                marks[i + 1].record(stream)
            marks[-1].synchronize()
        trials = trial_stats([marks[i].elapsed_time(marks[i + 1]) for i in range(args.steps)])
        x0, w0, ws0, b0 = sets[0]
        par = fast_parity(torch, lib, wl, x0, w0, ws0, b0, c_all[0], rows=64, tail=True)
        if not par["within_bound"]:
            # Evidence for a miss: the same plan once more on the same inputs.
            plan.run(stream.cuda_stream)
            stream.synchronize()
            again = fast_parity(torch, lib, wl, x0, w0, ws0, b0, c_all[0], rows=64, tail=True)
            par["rerun"] = {k: again[k] for k in ("within_bound", "max_rel_err", "worst_at",
                                                  "outside_bound")}
        step_tf = batch * wl.flops / (trials["median_ms"] / 1e3) / 1e12
        gemm_tf = batch * wl.flops / (gemm_ms / 1e3) / 1e12
        rec = {"workload": wl.name, "format": FMT_NAMES[wl.wfmt], "M": wl.M, "K": wl.K,
               "N": wl.N, "batch": batch, "bias": wl.bias,
               "step_tflops": step_tf, "trials": trials,
               "gemm": {"kernel": "k_gemm_mxf4", "launch_ms": gemm_ms, "tflops": gemm_tf,
                        **tensor_fracs(gemm_tf, pk, wl.wfmt)},
               "encoder_ms": kernel_ms[0],
               "hbm_gbs_gemm": batch * wl.bytes_gemm() / (gemm_ms / 1e3) / 1e9,
               "parity": {k: par[k] for k in ("rows", "outputs", "max_rel_err", "within_bound",
                                              "worst_at", "outside_bound", "rerun")
                          if k in par},
               "clocks": clocks.summary()}
        if not args.no_cpu_baseline:
            ck = (wl.wfmt, wl.K, wl.N)
            if ck not in cpu_rates:
                r = cpu_reference(dataclasses.replace(wl, M=256), min_seconds=0.5, max_reps=5)
                cpu_rates[ck] = {k: v for k, v in r.items() if k != "seconds"}
            rec["cpu_baseline"] = cpu_rates[ck]
            rec["vs_cpu"] = step_tf / cpu_rates[ck]["value"]
        records.append(rec)
        print(f"# {wl.name}: step {step_tf:.1f} TFLOP/s, GEMM {gemm_tf:.1f} TFLOP/s "
              f"({rec['gemm']['frac_of_8bit_dense_peak']:.3f} of 8-bit dense), "
              f"parity {par['within_bound']}", file=sys.stderr, flush=True)
        plan.close()
        del a_all, c_all, keep, descs, sets
        torch.cuda.synchronize()
        torch.cuda.empty_cache()
    lib.close()
    conv = []
    for key in sorted(CONVS):
        if args.sweep_filter and not re.search(args.sweep_filter, key):
            continue
        sub = argparse.Namespace(**vars(args))
        sub.config = key
        sub.no_e2e = True
        buf = io.StringIO()
        with contextlib.redirect_stdout(buf):
            run_conv(sub, rank, world, local_rank)
        for line in buf.getvalue().splitlines():
            if line.startswith("{"):
                conv.append(json.loads(line))
    line = {"metric": "W8/MXFP4/MXFP8 GEMM TFLOP/s (C5 large-M sweep, 27 GEMMs + conv)",
            "unit": "TFLOP/s", "n_gpus": 1, "steps": args.steps, "warmup": args.warmup,
            "higher_is_better": True, "data": "synthetic",
            "peaks": {"bf16_tflops": pk["bf16_tflops"], "hbm_gbs": pk["hbm_gbs"],
                      "source": pk["source"]},
            "gemms": records, "conv": conv}
    print(json.dumps(line), flush=True)
    if args.summary_md:
        write_sweep_md(args, line)


def write_sweep_md(args, line: dict) -> None:
    pk = line["peaks"]
    out = [f"# C5 sweep on one B200: {len(line['gemms'])} GEMMs + conv", "",
           "Command: `python bench.py --config c5sweep --steps {} --warmup {} "
           "--summary-md <file>`".format(args.steps, args.warmup), "",
           f"Peaks ({pk['source']}): dense BF16 {pk['bf16_tflops']:.1f} TFLOP/s (8-bit dense = 2x, "
           "kind::mxf4 = 4x, kind::mxf8f6f4 = 2x), HBM "
           f"{pk['hbm_gbs']:.0f} GB/s.", "",
           "Step = the plan's launches (FP32 activations encoded, then the GEMM) over a batch "
           "of B instances whose operands exceed 2 x L2; median of the per-step event "
           "times.  GEMM = the tensor-core kernel alone over repeated launches.  "
           "Parity: first 32 and last 32 rows against the float64 product, bound "
           "(K/16 + 4) 2^-23 sum|a w|.", "",
           "| format | M | K | N | B | step TFLOP/s | spread | GEMM TFLOP/s | of MMA kind's "
           "dense | of 8-bit dense | GEMM HBM GB/s | max rel err | in bound | vs CPU |",
           "|---|---|---|---|---|---|---|---|---|---|---|---|---|---|"]
    for r in line["gemms"]:
        g = r["gemm"]
        out.append(f"| {r['format']} | {r['M']} | {r['K']} | {r['N']} | {r['batch']} | "
                   f"{r['step_tflops']:.1f} | {r['trials']['spread']:.3f} | {g['tflops']:.1f} | "
                   f"{g['frac_of_kind_dense_peak']:.3f} | {g['frac_of_8bit_dense_peak']:.3f} | "
                   f"{r['hbm_gbs_gemm']:.0f} | {r['parity']['max_rel_err']:.2e} | "
                   f"{r['parity']['within_bound']} | "
                   + (f"{r['vs_cpu']:.0f}x |" if "vs_cpu" in r else "- |"))
    if line["conv"]:
        out += ["", "| conv | ms/step | TFLOP/s | GEMM TFLOP/s | of MMA kind's dense | "
                "of 8-bit dense | CPU (reference, 1 thread) TFLOP/s |", "|---|---|---|---|---|---|---|"]
        for c in line["conv"]:
            ro = c["roofline"]
            cb = c.get("cpu_baseline", {}).get("value")
            out.append(f"| {c['config']['workload']} | {c['ms_per_step']:.3f} | {c['value']:.1f} | "
                       f"{ro['achieved']:.1f} | {ro['frac_of_kind_dense_peak']:.3f} | "
                       f"{ro['frac_of_8bit_dense_peak']:.3f} | "
                       + (f"{cb:.5f} |" if cb else "- |"))
    with open(args.summary_md, "w") as f:
        f.write("\n".join(out) + "\n")


def main() -> None:
    p = argparse.ArgumentParser()
    p.add_argument("--gpus", type=int, default=1)
    p.add_argument("--steps", type=int, default=200)
    p.add_argument("--warmup", type=int, default=10)
    p.add_argument("--impl", choices=["ours", "reference"], default="ours")
    p.add_argument("--config", choices=sorted(WORKLOADS) + [PREFIX.key, GACC.key, EXPERT.key,
                                                            "c5sweep"]
                   + sorted(CONVS),
                   default="c2")
    p.add_argument("--mode", choices=["exact", "fast"], default="fast")
    p.add_argument("--w8-kernel", choices=["planes", "bf16"], default="planes",
                   help="W8 with at most 64 tokens: E2M1 digit planes (kind::mxf4) or int8 "
                        "converted to BF16 in the kernel (kind::f16)")
    p.add_argument("--batch", type=int, default=0, help="GEMMs per step per GPU (0: the "
                   "config's default)")
    p.add_argument("--no-cpu-baseline", action="store_true")
    p.add_argument("--no-e2e", action="store_true", help="skip the host entry-point leg "
                   "(profiling runs)")
    p.add_argument("--gather", choices=["fp32", "mxint8"], default="fp32",
                   help="--shard on a GEMM config: what the fused all-gather moves (mxint8: the "
                        "output's MXINT8 copy only)")
    p.add_argument("--shard", action="store_true", help="split each GEMM along N (c5conv: the "
                   "images along M) over the ranks, with the all-gather fused into the kernel "
                   "(strong scaling)")
    p.add_argument("--sweep-filter", default="", help="c5sweep: only the GEMMs (and convs) "
                   "whose key matches this regex")
    p.add_argument("--summary-md", default="", help="c5sweep: write a markdown table here")
    args = p.parse_args()
    rank = int(os.environ.get("RANK", "0"))
    world = int(os.environ.get("WORLD_SIZE", "1"))
    local_rank = int(os.environ.get("LOCAL_RANK", "0"))
    if args.config == "c5sweep":
        run_sweep(args, rank, world, local_rank)
        return
    if args.config == EXPERT.key:
        run_expert(args, rank, world, local_rank)
        return
    if args.config in CONVS:
        if args.shard and args.impl != "reference":
            run_conv_shard(args, rank, world, local_rank)
        else:
            run_conv(args, rank, world, local_rank)
        return
    if args.config == GACC.key:
        run_gacc(args, rank, world, local_rank)
        return
    if args.config == PREFIX.key:
        run_prefix(args, rank, world, local_rank)
        return
    wl = WORKLOADS[args.config]
    if args.impl == "reference":
        run_reference(args, wl, rank, world)
    elif args.shard:
        run_shard(args, wl, rank, world, local_rank)
    else:
        run_ours(args, wl, rank, world, local_rank)


if __name__ == "__main__":
    main()
