"""Worker for the multi-process tests of hotarubi_b200.shard, launched with
torch.distributed.run (one process per rank, rendezvous on 127.0.0.1).

    --mode cpu   gloo ranks, host logic only:
                 columns: each rank computes its column slice of a GEMM with
                 the CPU oracle; shard.gather_columns must rebuild the whole
                 GEMM;
                 rows: each rank convolves its images (shard.rows) with the
                 oracle; the row ranges (shard.row_offsets) gathered must
                 rebuild the whole convolution.
    --mode gpu   NCCL ranks, one GPU each, data plane through the library's
                 communicator (shard.Group):
                 columns: a batch of column-sharded GEMMs whose epilogues
                 store every output into all ranks' C (PeerOutput +
                 Plan.set_peers); every rank's C must equal the unsharded
                 GEMM bit for bit, and so must the library all-gather;
                 rows: the C5-shaped convolution (smaller batch) split by
                 images, FP32 output and its MXINT8 copy stored into all
                 ranks by the epilogue (ConvPlan.set_peers); both equal the
                 unsharded convolution bit for bit, and so does the
                 communicator's in-place all-gather of the row ranges.
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

# The row-sharded convolution of the tests: 3x3, 256 -> 256 channels (the C5
# conv's layer) on 2 x 3 images of 8 x 12.
CONV = dict(images=6, H=8, W=12, cin=256, cout=256, kh=3, stride=1)


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
    # Rows: images split over the ranks, outputs contiguous along M.
    c = CONV
    hw, per = c["H"] * c["W"], (c["H"] // c["stride"]) * (c["W"] // c["stride"])
    spans = [shard.rows(c["images"], r, ranks) for r in range(ranks)]
    assert spans[0][0] == 0 and spans[-1][1] == c["images"]
    assert all(spans[i][1] == spans[i + 1][0] for i in range(ranks - 1))
    offs = shard.row_offsets(c["images"], per * c["cout"] * 4, ranks)
    assert offs == [a * per * c["cout"] * 4 for a, _ in spans] + [c["images"] * per * c["cout"] * 4]
    xa = workloads.activations(3, c["images"] * hw, c["cin"])
    aq, asc = cpu.encode_mxint8(xa.view(np.uint32))
    wc, wcs = workloads.mxfp4_weights(4, c["cout"], c["kh"] ** 2 * c["cin"])
    i0, i1 = shard.rows(c["images"])
    geo = (c["H"], c["W"], c["cin"], c["cout"], c["kh"], c["stride"])
    mine = cpu.conv_dense(0, aq[i0 * hw:i1 * hw], asc[i0 * hw:i1 * hw], i1 - i0, *geo, wc, wcs)
    width = max(b - a for a, b in spans) * per
    padded = np.zeros((width, c["cout"]), np.uint32)
    padded[:mine.shape[0]] = mine
    parts = [torch.empty((width, c["cout"]), dtype=torch.int32) for _ in range(ranks)]
    dist.all_gather(parts, torch.from_numpy(padded.view(np.int32)))
    got = np.concatenate([parts[r].numpy()[:(b - a) * per] for r, (a, b) in enumerate(spans)])
    want = cpu.conv_dense(0, aq, asc, c["images"], *geo, wc, wcs)
    assert np.array_equal(got.view(np.uint32), want), "gathered rows differ"


def run_gpu_columns(lib, group) -> None:
    from hotarubi_b200 import capi
    rank = group.rank
    batch, m, n, k = 3, 96, 1000, 768
    out = shard.PeerOutput(lib, group, (batch, m, n))
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
    group.barrier()
    for p in plans:
        p.run()
    group.fence()
    lib.sync()
    got = out.tensor.cpu().numpy()
    want = ref.cpu().numpy()
    assert np.array_equal(got.view(np.uint32), want.view(np.uint32)), f"rank {rank}: fused gather"
    # The library baseline: gather this rank's slices with torch's NCCL.
    for b in range(batch):
        g = shard.gather_columns(out.tensor[b][:, n0:n1].contiguous(), n)
        assert torch.equal(g.view(torch.int32), ref[b].view(torch.int32)), f"rank {rank}: nccl"
    group.barrier()
    for p in plans:
        p.close()
    full.close()
    torch.cuda.synchronize()
    group.barrier()
    out.close()


def run_gpu_columns_mxint8(lib, group) -> None:
    """Column shards that gather only the MXINT8 copy (hrb_gemm_desc.ldcq):
    each rank's GEMM over its columns writes the copy, and no FP32 output,
    into the full matrix's layout in every rank's buffer; bit-equal to the
    unsharded GEMM's copy."""
    from hotarubi_b200 import capi
    rank = group.rank
    batch, m, n, k = 2, 80, 1000, 512
    kpn = (n + 31) // 32 * 32
    out = shard.PeerOutput(lib, group, (1,), mx_shape=(batch * m, kpn))
    out.q.zero_()
    out.s.zero_()
    n0, n1 = shard.columns(n)
    keep, local_descs, full_descs = [], [], []
    ref_c = torch.zeros((batch, m, n), dtype=torch.float32, device="cuda")
    ref_q = torch.zeros((batch * m, kpn), dtype=torch.int8, device="cuda")
    ref_s = torch.zeros((batch * m, kpn // 32), dtype=torch.uint8, device="cuda")
    for b in range(batch):
        x = torch.from_numpy(workloads.activations(40 + b, m, k)).cuda()
        w, ws = workloads.mxfp4_weights(50 + b, n, k)
        wd, wsd = torch.from_numpy(w).cuda(), torch.from_numpy(ws).cuda()
        keep += [x, wd, wsd]
        rows = slice(b * m, (b + 1) * m)
        full_descs.append(capi.Library.desc(0, m, n, k, a=x, w=wd, wscale=wsd, c=ref_c[b],
                                            mode=capi.MODE_FAST, cq=ref_q[rows],
                                            cscale=ref_s[rows]))
        if n1 > n0:
            local_descs.append(capi.Library.desc(
                0, m, n1 - n0, k, a=x, w=wd[n0:n1], wscale=wsd[n0:n1], c=None,
                mode=capi.MODE_FAST, cq=out.q[rows].data_ptr() + n0,
                cscale=out.s[rows].data_ptr() + n0 // 32, ldcq=kpn))
    torch.cuda.synchronize()
    full = lib.plan(full_descs)
    full.run()
    lib.sync()
    plan = None
    if local_descs:
        plan = lib.plan(local_descs)
        plan.set_peers(out.ptr, out.peer_bases)
    group.barrier()
    if plan is not None:
        plan.run()
    group.fence()
    lib.sync()
    assert torch.equal(out.q, ref_q), f"rank {rank}: gathered MXINT8 codes"
    assert torch.equal(out.s, ref_s), f"rank {rank}: gathered MXINT8 scales"
    group.barrier()
    if plan is not None:
        plan.close()
    full.close()
    torch.cuda.synchronize()
    group.barrier()
    out.close()


def run_gpu_rows(lib, group, wfmt: int = 0) -> None:
    from hotarubi_b200 import capi
    rank, ranks = group.rank, group.ranks
    c = CONV
    hw = c["H"] * c["W"]
    per = (c["H"] // c["stride"]) * (c["W"] // c["stride"])
    m = c["images"] * per
    kpn = (c["cout"] + 31) // 32 * 32
    geo = (c["H"], c["W"], c["cin"], c["cout"], c["kh"], c["stride"])
    xa = torch.from_numpy(workloads.activations(5, c["images"] * hw, c["cin"])).cuda()
    kk = c["kh"] ** 2 * c["cin"]
    if wfmt == 0:
        w, ws = workloads.mxfp4_weights(6, c["cout"], kk)
    else:  # W8: MXINT8 codes with their block scale bytes
        rng = np.random.default_rng(6)
        w = rng.integers(-127, 128, (c["cout"], kk)).astype(np.int8).view(np.uint8)
        ws = rng.integers(116, 124, (c["cout"], kk // 32)).astype(np.uint8)
    bias = (np.random.default_rng(7).standard_normal(c["cout"]) * 0.01).astype(np.float32)
    wd, wsd, bd = (torch.from_numpy(v).cuda() for v in (w, ws, bias))
    # The unsharded convolution on this GPU.
    ref = torch.zeros((m, c["cout"]), dtype=torch.float32, device="cuda")
    ref_q = torch.zeros((m, kpn), dtype=torch.int8, device="cuda")
    ref_s = torch.zeros((m, kpn // 32), dtype=torch.uint8, device="cuda")
    full = lib.conv_plan(capi.conv_desc(wfmt, c["images"], *geo, order=capi.CONV_YMAJOR, a=xa,
                                        w=wd, wscale=wsd, bias=bd, c=ref, relu=True,
                                        mode=capi.MODE_FAST, cq=ref_q, cscale=ref_s))
    full.run()
    lib.sync()
    # This rank's images, outputs into the shared buffer at their rows.
    out = shard.PeerOutput(lib, group, (m, c["cout"]), mx_shape=(m, kpn))
    out.tensor.zero_()
    out.q.zero_()
    out.s.zero_()
    i0, i1 = shard.rows(c["images"])
    r0, r1 = i0 * per, i1 * per
    plan = None
    if i1 > i0:
        plan = lib.conv_plan(capi.conv_desc(wfmt, i1 - i0, *geo, order=capi.CONV_YMAJOR,
                                            a=xa[i0 * hw:i1 * hw], w=wd, wscale=wsd, bias=bd,
                                            c=out.tensor[r0:r1], relu=True, mode=capi.MODE_FAST,
                                            cq=out.q[r0:r1], cscale=out.s[r0:r1]))
        plan.set_peers(out.ptr, out.peer_bases)
    torch.cuda.synchronize()
    group.barrier()
    if plan is not None:
        plan.run()
    group.fence()
    lib.sync()
    assert torch.equal(out.tensor.view(torch.int32), ref.view(torch.int32)), \
        f"rank {rank}: fused row gather (FP32, format {wfmt})"
    assert torch.equal(out.q, ref_q) and torch.equal(out.s, ref_s), \
        f"rank {rank}: fused row gather (MXINT8 copy)"
    # The communicator's in-place all-gather of the row ranges.
    group.barrier()
    loose = torch.zeros((m, c["cout"]), dtype=torch.float32, device="cuda")
    loose[r0:r1] = ref[r0:r1]
    torch.cuda.synchronize()
    group.allgather(loose, shard.row_offsets(c["images"], per * c["cout"] * 4, ranks))
    lib.sync()
    assert torch.equal(loose.view(torch.int32), ref.view(torch.int32)), \
        f"rank {rank}: communicator all-gather"
    group.barrier()
    if plan is not None:
        plan.close()
    full.close()
    torch.cuda.synchronize()
    group.barrier()
    out.close()


def main() -> None:
    ap = argparse.ArgumentParser()
    ap.add_argument("--mode", choices=["cpu", "gpu"], required=True)
    args = ap.parse_args()
    timeout = datetime.timedelta(seconds=60)
    if args.mode == "gpu":
        from hotarubi_b200 import capi
        local = int(os.environ["LOCAL_RANK"])
        torch.cuda.set_device(local)
        # torch.distributed carries the communicator's bootstrap id and the
        # column baseline (gather_columns); the rest is the library's.
        dist.init_process_group("nccl", timeout=timeout, device_id=torch.device("cuda", local))
        lib = capi.Library(local)
        group = shard.Group(lib)
        run_gpu_columns(lib, group)
        run_gpu_columns_mxint8(lib, group)
        run_gpu_rows(lib, group, 0)
        run_gpu_rows(lib, group, 1)
        group.barrier()
        group.close()
        lib.close()
    else:
        dist.init_process_group("gloo", timeout=timeout)
        run_cpu()
    dist.destroy_process_group()


if __name__ == "__main__":
    main()
