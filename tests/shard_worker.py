"""Worker for the multi-process tests of hotarubi_b200.shard, launched with
torch.distributed.run (one process per rank, rendezvous on 127.0.0.1).

    --mode cpu   gloo ranks: each computes its column slice of a GEMM with
                 the CPU oracle; the slices are gathered with
                 shard.gather_columns and compared with the whole GEMM.
    --mode gpu   NCCL ranks, one GPU each: a batch of column-sharded GEMMs
                 whose epilogues store every output into all ranks' C
                 (shard.PeerOutput + Plan.set_peers); every rank's C must equal
                 the unsharded GEMM bit for bit, and so must the library
                 all-gather of the slices.
Exits non-zero on a mismatch.
"""
import argparse
import datetime
import os
import sys

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
sys.path.insert(0, ROOT)

import numpy as np  # noqa: E402
import torch  # noqa: E402
import torch.distributed as dist  # noqa: E402

from hotarubi_b200 import shard, workloads  # noqa: E402


def run_cpu() -> None:
    from oracle import cpu
    rank, ranks = dist.get_rank(), dist.get_world_size()
    m, n, k = 32, 600, 256
    x = workloads.activations(1, m, k)
    w, ws = workloads.mxfp4_weights(2, n, k)
    q, s = cpu.encode_mxint8(x.view(np.uint32))
    spans = [shard.columns(n, r, ranks) for r in range(ranks)]
    assert spans[0][0] == 0 and spans[-1][1] == n
    assert all(spans[i][1] == spans[i + 1][0] for i in range(ranks - 1))
    assert all(a % 128 == 0 for a, _ in spans)
    assert shard.exchange(rank * 10) == [r * 10 for r in range(ranks)]
    n0, n1 = shard.columns(n)
    local = cpu.gemm_dense(0, q, s, w[n0:n1], ws[n0:n1], n1 - n0)
    full = shard.gather_columns(torch.from_numpy(local.view(np.int32)), n).numpy()
    want = cpu.gemm_dense(0, q, s, w, ws, n)
    assert np.array_equal(full.view(np.uint32), want), "gathered columns differ"


def run_gpu() -> None:
    from hotarubi_b200 import capi
    rank, ranks = dist.get_rank(), dist.get_world_size()
    lib = capi.Library(torch.cuda.current_device())
    batch, m, n, k = 3, 96, 1000, 768
    out = shard.PeerOutput(lib, (batch, m, n))
    out.tensor.zero_()
    n0, n1 = shard.columns(n)
    keep, local_descs, full_descs = [], [], []
    ref = torch.zeros((batch, m, n), dtype=torch.float32, device="cuda")
    for b in range(batch):
        wfmt = 0 if b % 2 == 0 else 1
        x = torch.from_numpy(workloads.activations(10 + b, m, k)).cuda()
        if wfmt == 0:
            w, ws = workloads.mxfp4_weights(20 + b, n, k)
        else:
            rng = np.random.default_rng(30 + b)
            w = rng.integers(-128, 128, (n, k)).astype(np.int8).view(np.uint8)
            ws = rng.integers(110, 125, (n, k // 32)).astype(np.uint8)
        wd, wsd = torch.from_numpy(w).cuda(), torch.from_numpy(ws).cuda()
        keep += [x, wd, wsd]
        full_descs.append(capi.Library.desc(wfmt, m, n, k, a=x, w=wd, wscale=wsd, c=ref[b],
                                            mode=capi.MODE_FAST))
        if n1 > n0:
            c_local = out.tensor[b].data_ptr() + 4 * n0
            local_descs.append(capi.Library.desc(wfmt, m, n1 - n0, k, a=x, w=wd[n0:n1],
                                                 wscale=wsd[n0:n1], c=c_local, ldc=n,
                                                 mode=capi.MODE_FAST))
    torch.cuda.synchronize()
    full = lib.plan(full_descs)
    full.run()
    lib.sync()
    plans = []
    # One plan per weight format (a plan's MXFP4 and W8 GEMMs are separate
    # launches either way).
    for f in (0, 1):
        ds = [d for d in local_descs if d.wfmt == f]
        if ds:
            p = lib.plan(ds)
            p.set_peers(out.ptr, out.peer_bases)
            plans.append(p)
    dist.barrier()
    for p in plans:
        p.run()
    lib.sync()
    shard.complete()
    got = out.tensor.cpu().numpy()
    want = ref.cpu().numpy()
    assert np.array_equal(got.view(np.uint32), want.view(np.uint32)), f"rank {rank}: fused gather"
    # The library baseline: gather this rank's slices with NCCL.
    for b in range(batch):
        g = shard.gather_columns(out.tensor[b][:, n0:n1].contiguous(), n)
        assert torch.equal(g.view(torch.int32), ref[b].view(torch.int32)), f"rank {rank}: nccl"
    dist.barrier()
    for p in plans:
        p.close()
    full.close()
    torch.cuda.synchronize()
    dist.barrier()
    out.close()
    lib.close()


def main() -> None:
    ap = argparse.ArgumentParser()
    ap.add_argument("--mode", choices=["cpu", "gpu"], required=True)
    args = ap.parse_args()
    timeout = datetime.timedelta(seconds=60)
    if args.mode == "gpu":
        torch.cuda.set_device(int(os.environ["LOCAL_RANK"]))
        dist.init_process_group("nccl", timeout=timeout,
                                device_id=torch.device("cuda", int(os.environ["LOCAL_RANK"])))
        run_gpu()
    else:
        dist.init_process_group("gloo", timeout=timeout)
        run_cpu()
    dist.destroy_process_group()


if __name__ == "__main__":
    main()
