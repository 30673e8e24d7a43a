"""The pair kernel (MXFP4, at most 64 tokens, launches of at least as many
column-tile pairs as SMs): one CTA runs two adjacent 128-column weight tiles
against one activation block.  Its products and their order are those of the
plain kernel for each tile, so every output must be bit-identical to the
plain kernel's (the same GEMM in launches too small to pair), and within the
fast-mode bound of the float64 product (tests/test_gpu_fast.py).

Covered: a plan of C2-shaped GEMMs; odd numbers of column tiles (the second
tile of the last pair absent) with ragged token and column tiles, bias,
accumulate, the MXINT8 output copy and per-column scales; one large GEMM
launched without a plan; and hrb_plan_run_host, which launches the pairs of
chunks of the plan.
"""
import numpy as np
import pytest

from oracle import cpu

pytestmark = pytest.mark.gpu

torch = pytest.importorskip("torch")

SMS = 148


def pairs_of(m, n):
    return ((m + 63) // 64) * (((n + 127) // 128 + 1) // 2)


def weights(rng, n, k):
    from hotarubi_b200 import workloads
    return workloads.mxfp4_weights(int(rng.integers(0, 1 << 30)), n, k)


def dev(x):
    return torch.from_numpy(np.ascontiguousarray(x)).cuda()


def make(rng, m, n, k, *, bias=False, acc=False, cq=False, colscale=False):
    from hotarubi_b200 import capi
    x = dev(rng.standard_normal((m, k)).astype(np.float32))
    w, ws = weights(rng, n, k)
    t = {"x": x, "w": dev(w), "ws": dev(ws), "n": n, "m": m, "k": k}
    t["bias"] = dev((rng.standard_normal(n) * 0.01).astype(np.float32)) if bias else None
    t["c0"] = dev(rng.standard_normal((m, n)).astype(np.float32)) if acc else None
    t["cs"] = dev((rng.uniform(0.5, 2.0, n) * 2.0 ** -3).astype(np.float32)) if colscale else None
    t["cq"] = cq

    def desc(c, q=None, s=None):
        return capi.Library.desc(0, m, n, k, a=x, w=t["w"], wscale=t["ws"], bias=t["bias"], c=c,
                                 accumulate=acc, mode=capi.MODE_FAST, cq=q, cscale=s,
                                 cquant=capi.QUANT_HOST, wcol_scale=t["cs"])
    t["desc"] = desc
    return t


def outputs(t):
    kbq = (t["n"] + 31) // 32
    c = t["c0"].clone() if t["c0"] is not None else torch.zeros((t["m"], t["n"]), device="cuda")
    q = torch.zeros((t["m"], kbq * 32), dtype=torch.int8, device="cuda") if t["cq"] else None
    s = torch.zeros((t["m"], kbq), dtype=torch.uint8, device="cuda") if t["cq"] else None
    return c, q, s


def plain(hrb, t):
    """The GEMM alone: far fewer pairs than SMs, so the plain kernel."""
    assert pairs_of(t["m"], t["n"]) < SMS
    c, q, s = outputs(t)
    hrb.dense(t["desc"](c, q, s))
    hrb.sync()
    return c, q, s


def same(a, b):
    return torch.equal(a.view(torch.int32) if a.dtype == torch.float32 else a,
                       b.view(torch.int32) if b.dtype == torch.float32 else b)


@pytest.mark.parametrize("shape,extras", [
    ((64, 960, 2560), ""),             # C2: 8 column tiles, 4 pairs a GEMM
    ((50, 840, 736), "acc"),           # 7 column tiles (the last pair half), ragged tiles
    ((50, 840, 736), "colscale"),      # per-column scales (not with accumulate)
], ids=["c2", "odd-ragged-bias-acc-cq", "odd-ragged-bias-colscale-cq"])
def test_plan_of_pairs_equals_the_plain_kernel(hrb, shape, extras):
    m, n, k = shape
    rng = np.random.default_rng(m + n + len(extras))
    count = -(-SMS // pairs_of(m, n)) + 3   # pairs enough for every SM
    ts = [make(rng, m, n, k, bias=bool(extras), acc=extras == "acc", cq=bool(extras),
               colscale=extras == "colscale") for _ in range(count)]
    outs = [outputs(t) for t in ts]
    p = hrb.plan([t["desc"](*o) for t, o in zip(ts, outs)])
    p.run()
    hrb.sync()
    p.close()
    for i, (t, o) in enumerate(zip(ts, outs)):
        want = plain(hrb, t)
        for got, ref in zip(o, want):
            if got is not None:
                assert same(got, ref), f"GEMM {i}: pair kernel differs from the plain kernel"
    # Within the bound of the float64 product (GEMM 0; with column scales the
    # bound scales by |s|, their one more rounding inside its slack).
    t = ts[0]
    x = t["x"].cpu().numpy()
    q, s = cpu.encode_mxint8(x.view(np.uint32))
    a = q.astype(np.float64) * np.repeat(np.ldexp(1.0, s.astype(np.int64) - 133), 32, axis=1)
    w = t["w"].cpu().numpy()
    codes = np.zeros((n, k), np.uint8)
    codes[:, 0::2], codes[:, 1::2] = w & 0xF, w >> 4
    e2m1 = np.array([0, .5, 1, 1.5, 2, 3, 4, 6])
    wd = e2m1[codes & 7] * np.where(codes & 8, -1.0, 1.0) * np.repeat(
        np.ldexp(1.0, t["ws"].cpu().numpy().astype(np.int64) - 127), 32, axis=1)
    ref, absref = a @ wd.T, np.abs(a) @ np.abs(wd).T
    if t["cs"] is not None:
        cs = t["cs"].cpu().numpy().astype(np.float64)
        ref, absref = ref * cs, absref * np.abs(cs)
    if t["c0"] is not None:
        c0 = t["c0"].cpu().numpy()
        ref, absref = ref + c0, absref + np.abs(c0)
    if t["bias"] is not None:
        b = t["bias"].cpu().numpy()
        ref, absref = ref + b, absref + np.abs(b)
    got = outs[0][0].cpu().numpy().astype(np.float64)
    tol = (k / 16 + 4) * 2.0 ** -23
    assert (np.abs(got - ref) <= tol * absref + 1e-30).all()


def test_one_large_gemm_without_a_plan(hrb):
    """64 x 38000 x 256: 297 column tiles, 149 pairs (the last one half) in
    one hrb_gemm_dense launch; each 4096-column slice alone (plain kernel)
    gives the same bits."""
    from hotarubi_b200 import capi
    m, n, k = 64, 38000, 256
    assert pairs_of(m, n) >= SMS
    rng = np.random.default_rng(5)
    t = make(rng, m, n, k, bias=True)
    c, _, _ = outputs(t)
    hrb.dense(t["desc"](c))
    hrb.sync()
    for n0 in range(0, n, 4096):
        n1 = min(n, n0 + 4096)
        want = torch.zeros((m, n1 - n0), device="cuda")
        hrb.dense(capi.Library.desc(0, m, n1 - n0, k, a=t["x"], w=t["w"][n0:n1],
                                    wscale=t["ws"][n0:n1], bias=t["bias"][n0:n1], c=want,
                                    mode=capi.MODE_FAST))
        hrb.sync()
        assert same(c[:, n0:n1].contiguous(), want), f"columns {n0}..{n1}"


def test_run_host_in_chunks_of_pairs(hrb):
    """hrb_plan_run_host on a plan of pairs (its chunks launch pair ranges of
    the tile array) gives the device run's bits."""
    from hotarubi_b200 import capi
    m, n, k = 64, 960, 512
    count = 48                      # 192 pairs
    rng = np.random.default_rng(9)
    a_dev = torch.zeros((count, m, k), device="cuda")
    c_dev = torch.zeros((count, m, n), device="cuda")
    keep, descs = [], []
    for i in range(count):
        w, ws = weights(rng, n, k)
        t = [dev(w), dev(ws)]
        keep += t
        descs.append(capi.Library.desc(0, m, n, k, a=a_dev[i], w=t[0], wscale=t[1], c=c_dev[i],
                                       mode=capi.MODE_FAST))
    plan = hrb.plan(descs)
    x = rng.standard_normal((count, m, k)).astype(np.float32)
    a_dev.copy_(torch.from_numpy(x))
    plan.run()
    hrb.sync()
    want = c_dev.cpu().numpy().copy()
    c_dev.zero_()
    a_pin = torch.from_numpy(x).pin_memory()
    c_pin = torch.zeros((count, m, n)).pin_memory()
    torch.cuda.synchronize()
    plan.run_host([a_pin[i] for i in range(count)], [c_pin[i] for i in range(count)])
    hrb.sync()
    assert np.array_equal(c_pin.numpy().view(np.uint32), want.view(np.uint32))
    plan.close()
