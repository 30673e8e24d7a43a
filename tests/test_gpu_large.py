"""Large-M tensor-core GEMMs against the exact answer, at the sizes the
benchmark's tensor-bound configurations run.

With more than 64 tokens the fast path runs 128-token tiles, whose single
TMEM accumulator is released to the MMA warp before the epilogue's stores
once every CTA has at least three tiles (tiles >= 3 x 148 on a B200): the
``kEarly`` instantiation of k_gemm_mxf4.  These tests reach it for all three
weight formats (C5's sweep shapes M in {256, 4096, 65536} x (K, N) in
{(960, 2560), (2560, 960), (4096, 4096)}, C4's 1600 x 720 -> 2048 MXFP8 as a
batched plan) and for ragged shapes with bias, accumulate and the MXINT8
output copy, and check:

* every sampled output against the real-valued dot product of the
  dequantized operands (float64) within the stated tolerance
  (K/16 + 4) * 2^-23 * sum_k |a_k w_k| (the bound of tests/test_gpu_fast.py;
  the reference's chain, ExecuteGemm tools/iss/gemm_array.cpp:112-149, is
  within the same bound of that product);
* the early-release launch bit-equal to the plain kernel on the same rows
  (row slices of 256 rows are launches of a few tiles, which take the plain
  instantiation).

Activations are drawn on the device (seeded torch generator) and only the
sampled rows come back: the first and the last 128-token tile in full and 64
rows between.
"""
import functools

import numpy as np
import pytest

from oracle import cpu

pytestmark = pytest.mark.gpu

torch = pytest.importorskip("torch")

TILE = 128


def dev(x):
    return torch.from_numpy(np.ascontiguousarray(x)).cuda()


E2M1 = np.array([0, .5, 1, 1.5, 2, 3, 4, 6], np.float64)


@functools.lru_cache(maxsize=None)
def _e4m3_units():
    return np.array([cpu.oracle().hrbo_e4m3_units(int(c)) for c in range(256)], np.float64)


@functools.lru_cache(maxsize=8)
def weights(wfmt, n, k, seed):
    """Dense weights [N][kp] in `wfmt` with their scales, the survey's
    distributions (MXFP4 through CanonicalMxfp4), and their float64 values."""
    rng = np.random.default_rng(seed)
    kb = (k + 31) // 32
    kp = kb * 32
    if wfmt == 0:
        code = rng.integers(0, 16, (n, kp)).astype(np.uint8)
        code[:, k:] = 0
        e = rng.integers(-10, -3, (n, kb))
        code, e = cpu.canonical_mxfp4(code, e)
        w, ws = cpu.pack_nibbles(code), (e + 127).astype(np.uint8)
        v = E2M1[code & 7] * np.where(code & 8, -1.0, 1.0)
    elif wfmt == 1:
        w = rng.integers(-127, 128, (n, kp)).astype(np.int8)
        w[:, k:] = 0
        ws = rng.integers(115, 125, (n, kb)).astype(np.uint8)
        v = w.astype(np.float64) * 2.0**-6
        w = w.view(np.uint8)
    else:
        w = rng.integers(0, 254, (n, kp)).astype(np.uint8)
        w[w >= 0x7F] += 1
        w[:, k:] = 0
        ws = rng.integers(117, 124, (n, kb)).astype(np.uint8)
        v = _e4m3_units()[w] * 2.0**-9
    sc = np.repeat(np.ldexp(1.0, ws.astype(np.int64) - 127), 32, axis=1)
    return w, ws, v * sc


def device_activations(m, k, seed):
    g = torch.Generator(device="cuda")
    g.manual_seed(seed)
    return torch.randn((m, k), generator=g, device="cuda", dtype=torch.float32)


def sample_rows(m, seed):
    """The first and the last token tile in full, and 64 rows between."""
    last0 = ((m - 1) // TILE) * TILE
    rows = set(range(min(TILE, m))) | set(range(last0, m))
    rng = np.random.default_rng(seed)
    rows |= set(int(r) for r in rng.integers(0, m, 64))
    return np.array(sorted(rows), np.int64)


def dequant_rows(x_rows, k):
    """MXINT8 encoding of FP32 rows (EncodeMxint8) and its float64 values."""
    kp = ((k + 31) // 32) * 32
    xp = np.zeros((x_rows.shape[0], kp), np.float32)
    xp[:, :k] = x_rows
    q, s = cpu.encode_mxint8(xp.view(np.uint32))
    sc = np.ldexp(1.0, s.astype(np.int64) - 133)
    return q.astype(np.float64) * np.repeat(sc, 32, axis=1)


def check_rows(got, rows, x_dev, w_deq, k, *, bias=None, c0=None):
    """Sampled outputs against the float64 product within the bound."""
    x_rows = x_dev[torch.from_numpy(rows).cuda()].cpu().numpy()
    a = dequant_rows(x_rows, k)
    ref = a @ w_deq.T
    absref = np.abs(a) @ np.abs(w_deq).T
    if c0 is not None:
        ref += c0
        absref += np.abs(c0)
    if bias is not None:
        ref += bias
        absref += np.abs(bias)
    tol = (k / 16 + 4) * 2.0**-23
    err = np.abs(got.astype(np.float64) - ref)
    bad = err > tol * absref + 1e-30
    assert not bad.any(), (f"{int(bad.sum())} of {bad.size} sampled outputs off; worst rel "
                           f"{(err / (absref + 1e-30)).max():.3e}, tol {tol:.3e}")
    return float((err / (absref + 1e-30)).max())


def tiles_of(m, n):
    return ((m + TILE - 1) // TILE) * ((n + TILE - 1) // TILE)


def early_release(m, n, gemms=1):
    # The launcher's rule (gemm_mxf4.cu launch_mx): 128-token tiles, at
    # least three per CTA of a 148-SM grid.
    return m > 64 and gemms * tiles_of(m, n) >= 3 * 148


SWEEP = [(m, k, n) for m in (256, 4096, 65536) for (k, n) in ((960, 2560), (2560, 960),
                                                              (4096, 4096))]


@pytest.mark.parametrize("wfmt", [0, 1, 2], ids=["mxfp4", "w8", "mxfp8"])
@pytest.mark.parametrize("shape", SWEEP, ids=[f"{m}x{k}x{n}" for m, k, n in SWEEP])
def test_c5_sweep_sampled_rows(hrb, wfmt, shape):
    from hotarubi_b200 import capi
    m, k, n = shape
    w, ws, w_deq = weights(wfmt, n, k, 100 + wfmt)
    x = device_activations(m, k, seed=m + k + n + wfmt)
    c = torch.empty((m, n), dtype=torch.float32, device="cuda")
    dw, dws = dev(w), dev(ws)
    hrb.dense(capi.Library.desc(wfmt, m, n, k, a=x, w=dw, wscale=dws, c=c,
                                mode=capi.MODE_FAST))
    hrb.sync()
    rows = sample_rows(m, seed=m + n)
    got = c[torch.from_numpy(rows).cuda()].cpu().numpy()
    check_rows(got, rows, x, w_deq, k)
    assert np.isfinite(c.sum().item())
    del x, c
    torch.cuda.empty_cache()


def _run_slices(hrb, wfmt, m, n, k, x, dw, dws, *, bias=None, c0=None, cq=False, step=256):
    """The same GEMM launched on row slices of `step` rows (few tiles each:
    the plain kernel), outputs into one C and one MXINT8 copy."""
    from hotarubi_b200 import capi
    kbq = (n + 31) // 32
    c = c0.clone() if c0 is not None else torch.zeros((m, n), dtype=torch.float32, device="cuda")
    q = torch.zeros((m, kbq * 32), dtype=torch.int8, device="cuda") if cq else None
    s = torch.zeros((m, kbq), dtype=torch.uint8, device="cuda") if cq else None
    for r0 in range(0, m, step):
        r1 = min(m, r0 + step)
        assert not early_release(r1 - r0, n)
        d = capi.Library.desc(wfmt, r1 - r0, n, k, a=x[r0:r1], w=dw, wscale=dws, bias=bias,
                              c=c[r0:r1], accumulate=c0 is not None, mode=capi.MODE_FAST,
                              cq=None if q is None else q[r0:r1],
                              cscale=None if s is None else s[r0:r1], cquant=capi.QUANT_HOST)
        hrb.dense(d)
    hrb.sync()
    return c, q, s


@pytest.mark.parametrize("wfmt", [0, 1, 2], ids=["mxfp4", "w8", "mxfp8"])
@pytest.mark.parametrize("shape,extras", [
    ((2048, 4096, 256), False),       # 16 x 32 = 512 tiles, whole tiles
    ((2017, 3880, 736), True),        # ragged last token and column tiles
], ids=["whole", "ragged-bias-acc-cq"])
def test_early_release_equals_plain_kernel(hrb, wfmt, shape, extras):
    """The early-release launch (one CTA per SM, >= 3 tiles each) gives the
    same bits as the plain kernel on the same inputs, and both lie within the
    bound; with `extras` also bias, accumulate and the MXINT8 output copy."""
    from hotarubi_b200 import capi
    m, n, k = shape
    assert early_release(m, n)
    w, ws, w_deq = weights(wfmt, n, k, 200 + wfmt)
    x = device_activations(m, k, seed=7 + wfmt + m)
    dw, dws = dev(w), dev(ws)
    rng = np.random.default_rng(m + wfmt)
    bias_np = (rng.standard_normal(n) * 0.01).astype(np.float32) if extras else None
    bias = dev(bias_np) if extras else None
    c0 = torch.randn((m, n), device="cuda", dtype=torch.float32) if extras else None
    kbq = (n + 31) // 32
    c = c0.clone() if extras else torch.zeros((m, n), dtype=torch.float32, device="cuda")
    q = torch.zeros((m, kbq * 32), dtype=torch.int8, device="cuda") if extras else None
    s = torch.zeros((m, kbq), dtype=torch.uint8, device="cuda") if extras else None
    hrb.dense(capi.Library.desc(wfmt, m, n, k, a=x, w=dw, wscale=dws, bias=bias, c=c,
                                accumulate=extras, mode=capi.MODE_FAST, cq=q, cscale=s,
                                cquant=capi.QUANT_HOST))
    hrb.sync()
    c_pl, q_pl, s_pl = _run_slices(hrb, wfmt, m, n, k, x, dw, dws, bias=bias, c0=c0, cq=extras)
    diff = (c.view(torch.int32) != c_pl.view(torch.int32)).sum().item()
    assert diff == 0, f"{diff} outputs differ between the early-release and the plain kernel"
    if extras:
        assert torch.equal(q, q_pl) and torch.equal(s, s_pl)
        # The MXINT8 copy is the encoding of the FP32 output (host rule).
        rows = sample_rows(m, seed=3)
        crow = c[torch.from_numpy(rows).cuda()].cpu().numpy()
        cp = np.zeros((len(rows), kbq * 32), np.float32)
        cp[:, :n] = crow
        wq, wsc = cpu.encode_mxint8(cp.view(np.uint32))
        assert (q[torch.from_numpy(rows).cuda()].cpu().numpy() == wq).all()
        assert (s[torch.from_numpy(rows).cuda()].cpu().numpy() == wsc).all()
    rows = sample_rows(m, seed=m)
    got = c[torch.from_numpy(rows).cuda()].cpu().numpy()
    c0_rows = c0[torch.from_numpy(rows).cuda()].cpu().numpy() if extras else None
    check_rows(got, rows, x, w_deq, k, bias=bias_np, c0=c0_rows)


@pytest.mark.parametrize("wfmt", [0, 1, 2], ids=["mxfp4", "w8", "mxfp8"])
def test_batched_plan_c4_shape(hrb, wfmt):
    """A plan of three C4-shaped GEMMs (1600 tokens, 720 -> 2048; the action
    expert's MLP for 32 requests of 50 tokens): 624 tiles in one launch, so
    the early-release kernel runs; each GEMM with its own operands and bias."""
    from hotarubi_b200 import capi
    m, n, k = 1600, 2048, 720
    assert early_release(m, n, gemms=3) and not early_release(m, n)
    descs, keep, checks = [], [], []
    for g in range(3):
        w, ws, w_deq = weights(wfmt, n, k, 300 + 10 * g + wfmt)
        x = device_activations(m, k, seed=40 + g + wfmt)
        b = (np.random.default_rng(g).standard_normal(n) * 0.01).astype(np.float32)
        t = [dev(w), dev(ws), dev(b)]
        c = torch.zeros((m, n), dtype=torch.float32, device="cuda")
        keep += t + [x, c]
        descs.append(capi.Library.desc(wfmt, m, n, k, a=x, w=t[0], wscale=t[1], bias=t[2], c=c,
                                       mode=capi.MODE_FAST))
        checks.append((x, c, w_deq, b))
    p = hrb.plan(descs)
    p.run()
    hrb.sync()
    p.close()
    for g, (x, c, w_deq, b) in enumerate(checks):
        rows = sample_rows(m, seed=g)
        got = c[torch.from_numpy(rows).cuda()].cpu().numpy()
        check_rows(got, rows, x, w_deq, k, bias=b)
