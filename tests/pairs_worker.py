"""Child process of tests/test_gpu_pairs.py: runs a fixed set of MXFP4
fast-mode GEMMs (single calls and one plan) and saves every output under
the directory given on the command line.  The parent runs it with
HRB_CTA_PAIRS=1 (the CTA-pair kernel) and =0 (one CTA a tile)."""
import os
import sys

import numpy as np
import torch

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
sys.path.insert(0, ROOT)

from hotarubi_b200 import capi, workloads  # noqa: E402

# M, N, K, bias, accumulate, MXINT8 copy: even and odd column-tile counts,
# 64- and 128-token tiles, a launch with several pairs a cluster (early
# accumulator release), epilogue options.
CASES = [(64, 960, 2560, False, False, False), (64, 320, 512, True, False, False),
         (300, 200, 256, True, True, True), (1100, 1152, 1024, False, False, True),
         (4096, 1792, 256, True, False, False)]


def operands(i, m, n, k):
    x = workloads.activations(10 + i, m, k)
    w, ws = workloads.mxfp4_weights(20 + i, n, k)
    b = workloads.bias(30 + i, n)
    c0 = workloads.activations(40 + i, m, n)
    return x, w, ws, b, c0


def main(out):
    lib = capi.Library(0)
    dev = lambda a: torch.from_numpy(np.ascontiguousarray(a)).cuda()  # noqa: E731
    descs, keep = [], []
    for i, (m, n, k, bias, acc, cq) in enumerate(CASES):
        x, w, ws, b, c0 = operands(i, m, n, k)
        t = {"x": dev(x), "w": dev(w), "ws": dev(ws), "b": dev(b) if bias else None,
             "c": dev(c0) if acc else torch.zeros((m, n), dtype=torch.float32, device="cuda")}
        kq = (n + 31) // 32
        t["q"] = torch.zeros((m, kq * 32), dtype=torch.int8, device="cuda") if cq else None
        t["s"] = torch.zeros((m, kq), dtype=torch.uint8, device="cuda") if cq else None
        d = capi.Library.desc(0, m, n, k, a=t["x"], w=t["w"], wscale=t["ws"], bias=t["b"],
                              c=t["c"], accumulate=acc, mode=capi.MODE_FAST, cq=t["q"],
                              cscale=t["s"])
        torch.cuda.synchronize()  # torch's fills before the library's stream
        lib.dense(d)
        lib.sync()
        np.save(os.path.join(out, f"dense{i}_c.npy"), t["c"].cpu().numpy())
        if cq:
            np.save(os.path.join(out, f"dense{i}_q.npy"), t["q"].cpu().numpy())
            np.save(os.path.join(out, f"dense{i}_s.npy"), t["s"].cpu().numpy())
        if not acc:
            t["c"].zero_()
            descs.append(d)
            keep.append(t)
    plan = lib.plan(descs)
    torch.cuda.synchronize()
    plan.run(0)
    lib.sync()
    for j, t in enumerate(keep):
        np.save(os.path.join(out, f"plan{j}_c.npy"), t["c"].cpu().numpy())
    plan.close()
    lib.close()


if __name__ == "__main__":
    main(sys.argv[1])
