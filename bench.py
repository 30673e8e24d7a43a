"""Benchmark of the quantized GEMM hot path on B200.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]
                    [--mode exact|fast] [--batch B]

Workload (the MXFP4 GEMM the metric is quoted on):
C = A . W^T with A FP32 [64, 2560] ~ N(0,1) encoded to MXINT8 on the device,
W MXFP4 [960, 2560] (E2M1 codes, one E8M0 scale per 32-block, exponent in
[-10, -4], canonicalised as hotarubi's compiler does), FP32 C [64, 960].

One step = the hot path over one batch of B independent instances of that
GEMM, each with its own activations, weights and output (B = 128: 282 MB of
operands, more than twice the 126 MB L2, so every step streams from HBM and
no L2 flush is needed).  Per rank the batch is fixed: weak scaling, no
collective on the data path (the GEMMs are independent).

Reported (one JSON line, rank 0):
  value       TFLOP/s (2*M*N*K per GEMM) over all ranks, operands resident
              in HBM, max over ranks of the device time of K steps.
  e2e         the same metric through the host entry point hrb_gemm_dense_host
              (pinned host buffers in, result back to the host, every step).
  roofline    of the dominant kernel (the GEMM): its algorithmic bytes per
              launch over its CUDA-event duration, against the measured HBM
              copy bandwidth.
  cpu_baseline  the reference's own ExecuteGemm (oracle/_ref) on the host's
              cores on a bounded sample, rank 0 only.

--impl reference times only the reference's CPU implementation of the path
(rank 0), in the same metric.
"""
from __future__ import annotations

import argparse
import json
import os
import statistics
import subprocess
import sys
import threading
import time

import numpy as np

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, ROOT)

M, N, K = 64, 960, 2560
KB = K // 32
FLOPS_PER_GEMM = 2 * M * N * K
# Compulsory bytes of one GEMM: FP32 A in, MXFP4 W (4 bits), E8M0 scales, C out.
ALG_BYTES_STEP = M * K * 4 + N * K // 2 + N * KB + M * N * 4
# ... and of the GEMM kernel alone, which reads the MXINT8 activations.
ALG_BYTES_GEMM = M * K + M * KB + N * K // 2 + N * KB + M * N * 4
ALG_BYTES_QUANT = M * K * 4 + M * K + M * KB


def peaks() -> dict:
    p = os.path.join(ROOT, "MEASURED_PEAKS.json")
    if os.path.exists(p):
        with open(p) as f:
            d = json.load(f)
        return {"hbm_gbs": d["hbm_gbs"], "source": "measured"}
    return {"hbm_gbs": 6650.0, "source": "fallback"}


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
# The reference's CPU implementation (test infrastructure, timed only)

def cpu_reference(min_seconds: float = 2.0, max_reps: int = 50) -> dict:
    """hotarubi's ExecuteGemm, compiled from the reference sources
    (oracle/_ref), tiled into legal GEMM instructions over all host threads,
    on C2 GEMMs until ~min_seconds of wall time."""
    from hotarubi_b200 import workloads
    from oracle import cpu
    ref = cpu.ref()
    threads = os.cpu_count() or 1
    x = workloads.activations(0, M, K)
    w, ws = workloads.mxfp4_weights(1, N, K)
    q, s = cpu.encode_mxint8(x.view(np.uint32))
    a_words = cpu.pack_abuf(q, s).reshape(-1)
    codes = np.zeros((N, K), np.uint8)
    codes[:, 0::2] = w & 0xF
    codes[:, 1::2] = w >> 4
    planes = cpu.pack_wbuf(codes, ws).reshape(-1)
    c = np.zeros((M, N), np.uint32)
    if ref is None:
        # No reference build on this machine: the C restatement stands in.
        kind = "port"
        t0 = time.perf_counter()
        reps = 0
        while reps < 1 or time.perf_counter() - t0 < min_seconds / 4:
            cpu.gemm_dense(0, q, s, w, ws, N)
            reps += 1
        dt = time.perf_counter() - t0
        return {"value": reps * FLOPS_PER_GEMM / dt / 1e12, "unit": "TFLOP/s", "cores": 1,
                "kind": kind, "sample": f"{reps} x C2 GEMM (64x2560x960) on 1 thread",
                "seconds": dt}
    ref.hrbref_dense_gemm_iss(1, M, N, KB, a_words, planes, c, threads, 0, M)  # warm
    t0 = time.perf_counter()
    reps = 0
    while reps < max_reps and (reps < 1 or time.perf_counter() - t0 < min_seconds):
        ref.hrbref_dense_gemm_iss(1, M, N, KB, a_words, planes, c, threads, 0, M)
        reps += 1
    dt = time.perf_counter() - t0
    return {"value": reps * FLOPS_PER_GEMM / dt / 1e12, "unit": "TFLOP/s", "cores": threads,
            "kind": "reference",
            "sample": f"{reps} x C2 GEMM (64x2560x960) through ExecuteGemm tiles on "
                      f"{threads} threads", "seconds": dt}


def run_reference(args, rank: int, world: int) -> None:
    if rank != 0:
        return
    steps = []
    for i in range(args.warmup + args.steps):
        r = cpu_reference(min_seconds=0.5, max_reps=20)
        if i >= args.warmup:
            steps.append(r)
    value = statistics.median(r["value"] for r in steps)
    secs = statistics.median(r["seconds"] for r in steps)
    base = steps[-1]
    line = {
        "impl": "reference", "metric": "MXFP4 GEMM TFLOP/s (C2 64x2560x960)",
        "value": value, "unit": "TFLOP/s", "n_gpus": args.gpus, "steps": args.steps,
        "warmup": args.warmup, "ms_per_step": secs * 1e3, "higher_is_better": True,
        "scaling": "weak", "vs_baseline": None, "dtype": "int8 block dot + fp32 accumulate",
        "data": "synthetic",
        "config": {"workload": "c2_mxfp4_64x2560x960", "M": M, "N": N, "K": K,
                   "format": "mxfp4", "sample": base["sample"]},
        "cpu_baseline": {"value": value, "unit": "TFLOP/s", "cores": base["cores"],
                         "kind": base["kind"], "sample": base["sample"]},
        "e2e": {"value": value, "unit": "TFLOP/s", "h2d_bytes_per_step": 0,
                "d2h_bytes_per_step": 0},
    }
    print(json.dumps(line), flush=True)


# ---------------------------------------------------------------------------
# Our implementation

def build_batch(torch, lib, capi, batch: int, mode: int, distinct: int = 4):
    """B instances on the device: `distinct` seeded operand sets copied into
    B separate buffers (distinct memory, so every instance streams)."""
    from hotarubi_b200 import workloads
    sets = []
    for i in range(distinct):
        x = workloads.activations(100 + i, M, K)
        w, ws = workloads.mxfp4_weights(200 + i, N, K)
        sets.append((x, w, ws))
    inst = []
    for b in range(batch):
        x, w, ws = sets[b % distinct]
        inst.append(dict(
            a=torch.from_numpy(x).cuda(), w=torch.from_numpy(w).cuda(),
            ws=torch.from_numpy(ws).cuda(),
            c=torch.zeros((M, N), dtype=torch.float32, device="cuda")))
    full = [capi.Library.desc(capi.WFMT_MXFP4, M, N, K, a=d["a"], w=d["w"], wscale=d["ws"],
                              c=d["c"], mode=mode) for d in inst]
    torch.cuda.synchronize()
    return inst, lib.plan(full), sets


def traffic_from_profiles(kernel: str):
    """DRAM bytes per launch of `kernel` on this workload, as summarised from
    an ncu capture in profiles/dram_traffic.txt (kernel=bytes per GEMM)."""
    path = os.path.join(ROOT, "profiles", "dram_traffic.txt")
    if not os.path.exists(path):
        return None
    for line in open(path):
        parts = line.split()
        if len(parts) >= 2 and parts[0] == kernel:
            return float(parts[1])
    return None


def time_e2e(lib, capi, sets, batch: int, steps: int, warmup: int, mode: int) -> dict:
    """hrb_gemm_dense_host over the batch: operands from pinned host memory
    to the device, the GEMM, C back to the host, every step."""
    import torch
    pinned = []
    for b in range(batch):
        x, w, ws = sets[b % len(sets)]
        pinned.append(dict(a=torch.from_numpy(x).pin_memory(), w=torch.from_numpy(w).pin_memory(),
                           ws=torch.from_numpy(ws).pin_memory(),
                           c=torch.zeros((M, N), dtype=torch.float32).pin_memory()))
    descs = [capi.Library.desc(capi.WFMT_MXFP4, M, N, K, a=p["a"].data_ptr(),
                               w=p["w"].data_ptr(), wscale=p["ws"].data_ptr(),
                               c=p["c"].data_ptr(), mode=mode) for p in pinned]
    for _ in range(warmup):
        for d in descs:
            lib.dense_host(d)
    t0 = time.perf_counter()
    for _ in range(steps):
        for d in descs:
            lib.dense_host(d)
    dt = (time.perf_counter() - t0) / steps
    h2d = batch * (M * K * 4 + N * K // 2 + N * KB)
    d2h = batch * M * N * 4
    return {"value": batch * FLOPS_PER_GEMM / dt / 1e12, "unit": "TFLOP/s",
            "h2d_bytes_per_step": h2d, "d2h_bytes_per_step": d2h, "ms_per_step": dt * 1e3,
            "entry_point": "hrb_gemm_dense_host"}


def run_ours(args, rank: int, world: int, local_rank: int) -> None:
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
    inst, plan_full, sets = build_batch(torch, lib, capi, args.batch, mode)

    # Per-kernel device times (the dominant kernel's roofline): events around
    # each launch of the plan, a few runs (not the timed region).
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
        start = torch.cuda.Event(enable_timing=True)
        end = torch.cuda.Event(enable_timing=True)
        start.record(stream)
        launches = 0
        for _ in range(args.steps):
            launches += plan_full.run(stream.cuda_stream)
        end.record(stream)
        end.synchronize()
        torch.cuda.synchronize()
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
        e2e = time_e2e(lib, capi, sets, args.batch, max(1, min(args.steps, 3)), 1, mode)
    if dist is not None and e2e is not None:
        t = torch.tensor([e2e["ms_per_step"]], device="cuda")
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        e2e["ms_per_step"] = float(t.item())
        e2e["value"] = world * args.batch * FLOPS_PER_GEMM / (e2e["ms_per_step"] / 1e3) / 1e12
        e2e["h2d_bytes_per_step"] *= world
        e2e["d2h_bytes_per_step"] *= world

    if rank == 0:
        pk = peaks()
        gemm_gbs = args.batch * ALG_BYTES_GEMM / (gemm_ms / 1e3) / 1e9
        quant_gbs = args.batch * ALG_BYTES_QUANT / (quant_ms / 1e3) / 1e9
        kname = "k_gemm_mxf4" if mode == capi.MODE_FAST else "k_dense_exact"
        per_gemm_traffic = traffic_from_profiles(kname)  # ncu DRAM bytes per GEMM
        step_gbs = args.batch * ALG_BYTES_STEP / (ms / 1e3) / 1e9
        total_gemms = world * args.batch
        line = {
            "metric": "MXFP4 GEMM TFLOP/s (C2 64x2560x960)",
            "value": total_gemms * FLOPS_PER_GEMM / (ms / 1e3) / 1e12,
            "unit": "TFLOP/s", "n_gpus": world, "steps": args.steps, "warmup": args.warmup,
            "ms_per_step": ms, "higher_is_better": True, "scaling": "weak",
            "vs_baseline": None, "dtype": "int8 block dot + fp32 accumulate",
            "data": "synthetic",
            "config": {"workload": "c2_mxfp4_64x2560x960", "batch_per_gpu": args.batch,
                       "M": M, "N": N, "K": K, "format": "mxfp4", "mode": args.mode,
                       "activations": "fp32, encoded to mxint8 on device each step",
                       "l2": f"working set {args.batch * ALG_BYTES_STEP / 1e6:.0f} MB per GPU "
                             "> 2 x 126 MB L2, no flush",
                       "parallelism": f"replicas x{world} (independent GEMMs)"},
            "step_hbm_gbs": step_gbs,
            "roofline": {"bound": "hbm", "kernel": kname,
                         "achieved": gemm_gbs, "peak": pk["hbm_gbs"], "unit": "GB/s",
                         "frac": gemm_gbs / pk["hbm_gbs"], "peak_source": pk["source"],
                         "traffic": (None if per_gemm_traffic is None
                                     else per_gemm_traffic * args.batch),
                         "alg_bytes_per_launch": args.batch * ALG_BYTES_GEMM,
                         "launch_ms": gemm_ms},
            "encoder": {"kernel": "k_quantize_planes" if mode == capi.MODE_FAST else "k_quantize",
                        "launch_ms": quant_ms, "achieved_gbs": quant_gbs,
                        "frac": quant_gbs / pk["hbm_gbs"],
                        "alg_bytes_per_launch": args.batch * ALG_BYTES_QUANT,
                        "traffic": (None if traffic_from_profiles("k_quantize_planes") is None
                                    or mode != capi.MODE_FAST
                                    else traffic_from_profiles("k_quantize_planes") * args.batch)},
            "e2e": e2e, "gpu_launches": launches,
            "clocks": clocks.summary(),
        }
        if not args.no_cpu_baseline:
            line["cpu_baseline"] = {k: v for k, v in cpu_reference().items() if k != "seconds"}
        print(json.dumps(line), flush=True)
    plan_full.close()
    lib.close()
    if dist is not None:
        dist.barrier()
        dist.destroy_process_group()


def main() -> None:
    p = argparse.ArgumentParser()
    p.add_argument("--gpus", type=int, default=1)
    p.add_argument("--steps", type=int, default=200)
    p.add_argument("--warmup", type=int, default=10)
    p.add_argument("--impl", choices=["ours", "reference"], default="ours")
    p.add_argument("--mode", choices=["exact", "fast"], default="fast")
    p.add_argument("--batch", type=int, default=128)
    p.add_argument("--no-cpu-baseline", action="store_true")
    p.add_argument("--no-e2e", action="store_true", help="skip the host entry-point leg "
                   "(profiling runs)")
    args = p.parse_args()
    rank = int(os.environ.get("RANK", "0"))
    world = int(os.environ.get("WORLD_SIZE", "1"))
    local_rank = int(os.environ.get("LOCAL_RANK", "0"))
    if args.impl == "reference":
        run_reference(args, rank, world)
    else:
        run_ours(args, rank, world, local_rank)


if __name__ == "__main__":
    main()
