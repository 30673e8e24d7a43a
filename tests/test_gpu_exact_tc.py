"""The exact GEMM with its block dots on the tensor cores (k_exact_tc).

MXFP4 and W8 exact GEMMs run k_exact_tc: one tcgen05 kind::i8 MMA per
32-element block, the block values and the FP32 chain on the CUDA cores.
These cases aim at what is new in it: many 4-block steps and table chunks
(kb past 128), W8 pieces that split a step, tokens whose activation scale
leaves the two-multiply range (the integer rule per block), ragged M and N
across several tiles, plans of mixed jobs.  Every result is compared bit for
bit with the oracle; the last test reruns this file with HRB_EXACT_TC=0, so
that k_dense_exact passes the same cases.
"""
import os
import subprocess
import sys

import numpy as np
import pytest

from oracle import cpu

pytestmark = pytest.mark.gpu

torch = pytest.importorskip("torch")

TC = os.environ.get("HRB_EXACT_TC", "1") != "0"


def dev(x: np.ndarray):
    return torch.from_numpy(np.ascontiguousarray(x)).cuda()


def _weights(rng, wfmt, n, kb, lo=-10, hi=-3):
    k = kb * 32
    if wfmt == cpu.WFMT_MXFP4:
        code = rng.integers(0, 16, (n, k)).astype(np.uint8)
        e = rng.integers(lo, hi, (n, kb))
        code, e = cpu.canonical_mxfp4(code, e)
        return cpu.pack_nibbles(code), (e + 127).astype(np.uint8)
    return (rng.integers(-128, 128, (n, k)).astype(np.int8).view(np.uint8),
            rng.integers(115, 125, (n, kb)).astype(np.uint8))


def _mxint8(rng, m, kb, lo=120, hi=135):
    q = rng.integers(-127, 128, (m, kb * 32)).astype(np.int8)
    s = rng.integers(lo, hi, (m, kb)).astype(np.uint8)
    return q, s


def _run(hrb, wfmt, q, s, w, ws, n, *, bias=None, c_init=None, pieces=None, colscale=None):
    """One hrb_gemm_dense call on MXINT8 activations; returns C's bits and the
    number of kernels it launched."""
    from hotarubi_b200 import capi
    m = q.shape[0]
    c = dev(c_init.view(np.float32)) if c_init is not None else torch.zeros(
        (m, n), dtype=torch.float32, device="cuda")
    t = dict(aq=dev(q), ascale=dev(s), w=dev(w), wscale=dev(ws),
             bias=None if bias is None else dev(bias.view(np.float32)),
             wcol_scale=None if colscale is None else dev(colscale))
    torch.cuda.synchronize()
    d = capi.Library.desc(wfmt, m, n, q.shape[1], c=c, accumulate=c_init is not None,
                          pieces=pieces, **t)
    before = hrb.launches()
    hrb.dense(d)
    hrb.sync()
    launched = hrb.launches() - before
    return c.cpu().numpy().view(np.uint32), launched


def _check(hrb, wfmt, q, s, w, ws, n, **kw):
    want = cpu.gemm_dense(wfmt, q, s, w, ws, n,
                          bias_bits=kw.get("bias"), c_init=kw.get("c_init"),
                          pieces=kw.get("pieces"),
                          colscale_bits=None if kw.get("colscale") is None
                          else kw["colscale"].view(np.uint32))
    got, launched = _run(hrb, wfmt, q, s, w, ws, n, **kw)
    # k_exact_tc runs as the weight translation and the GEMM.
    assert launched == (2 if TC else 1)
    bad = np.argwhere(got != want)
    assert bad.size == 0, (len(bad), bad[:4].tolist(), got[tuple(bad[0])], want[tuple(bad[0])])


@pytest.mark.parametrize("wfmt", [0, 1])
@pytest.mark.parametrize("shape", [(1, 8, 1), (64, 128, 4), (65, 129, 5), (200, 300, 3),
                                   (7, 520, 33), (130, 70, 150), (3, 40, 300)])
def test_shapes(hrb, wfmt, shape):
    """One and several tiles each way, partial last steps, and kb past the
    128-block table chunk."""
    m, n, kb = shape
    rng = np.random.default_rng(11 * m + 7 * n + kb + wfmt)
    q, s = _mxint8(rng, m, kb)
    w, ws = _weights(rng, wfmt, n, kb)
    _check(hrb, wfmt, q, s, w, ws, n)


def test_w8_pieces_split_steps(hrb):
    """W8 runs every HI block of a piece, then its LO blocks: pieces that
    start and end inside 4-block steps, of one block, and past a table chunk."""
    rng = np.random.default_rng(3)
    for m, n, kb, pieces in ((70, 150, 11, [1, 6, 3, 1]), (64, 128, 9, [2, 4, 3]),
                             (33, 64, 140, [5, 1, 126, 8]), (5, 30, 7, [7])):
        q, s = _mxint8(rng, m, kb)
        w, ws = _weights(rng, 1, n, kb)
        bias = (rng.standard_normal(n).astype(np.float32) * 0.01).view(np.uint32)
        c0 = rng.standard_normal((m, n)).astype(np.float32).view(np.uint32)
        _check(hrb, 1, q, s, w, ws, n, pieces=pieces)
        _check(hrb, 1, q, s, w, ws, n, pieces=pieces, bias=bias, c_init=c0)


@pytest.mark.parametrize("wfmt", [0, 1])
def test_activation_scales_outside_the_fast_range(hrb, wfmt):
    """Activation scale bytes 0, 1, 237, 238 and 254 on some tokens and
    blocks: those blocks take the integer rule (flush to zero, infinities),
    the others the two multiplies, within one tile."""
    rng = np.random.default_rng(40 + wfmt)
    m, n, kb = 96, 160, 10
    q, s = _mxint8(rng, m, kb)
    s[3, :] = 0
    s[5, 2] = 1
    s[9, 4] = 237
    s[17, 4] = 238
    s[33, 7] = 254
    s[64:70, 1] = 200
    s[70:72, 8] = 60
    w, ws = _weights(rng, wfmt, n, kb)
    _check(hrb, wfmt, q, s, w, ws, n)
    bias = (rng.standard_normal(n).astype(np.float32)).view(np.uint32)
    _check(hrb, wfmt, q, s, w, ws, n, bias=bias)


@pytest.mark.parametrize("wfmt", [0, 1])
def test_weight_scales_at_the_edges(hrb, wfmt):
    """Weight scale bytes whose biased exponent leaves [1, 254] (W8 HI
    subtracts 8, LO 12, MXFP4 7): the integer rule; 254 overflows chains to
    infinity, which the integer adder then recomputes."""
    rng = np.random.default_rng(50 + wfmt)
    m, n, kb = 80, 140, 9
    q, s = _mxint8(rng, m, kb)
    w, ws = _weights(rng, wfmt, n, kb)
    ws[::7, 0] = 1
    ws[1::7, 3] = 8
    ws[2::7, 5] = 12
    ws[3::11, 6] = 254
    ws[4::13, 8] = 0
    _check(hrb, wfmt, q, s, w, ws, n)
    c0 = rng.standard_normal((m, n)).astype(np.float32).view(np.uint32)
    c0[::3, ::4] = 0x7F800000
    c0[1::3, ::5] = 0xFFC00000
    c0[2::3, ::6] = 0x00000003
    _check(hrb, wfmt, q, s, w, ws, n, c_init=c0)


@pytest.mark.parametrize("wfmt", [0, 1])
def test_column_scales_and_zeros(hrb, wfmt):
    """Per-column scales and biases after the chain; all-zero activation
    rows and weight rows give +0."""
    rng = np.random.default_rng(60 + wfmt)
    m, n, kb = 72, 136, 6
    q, s = _mxint8(rng, m, kb)
    q[4] = 0
    w, ws = _weights(rng, wfmt, n, kb)
    w[9] = 0
    cs = (rng.uniform(0.5, 2.0, n) * np.ldexp(1.0, rng.integers(-20, 20, n))).astype(np.float32)
    cs[::6] *= -1
    cs[5] = 0.0
    bias = (rng.standard_normal(n).astype(np.float32) * 0.01).view(np.uint32)
    bias[9] = 0x80000000
    _check(hrb, wfmt, q, s, w, ws, n, colscale=cs)
    _check(hrb, wfmt, q, s, w, ws, n, colscale=cs, bias=bias)


def test_plan_of_mixed_exact_jobs(hrb):
    """A plan of MXFP4, W8 (with pieces) and MXFP8 exact GEMMs, FP32 and
    MXINT8 inputs: one k_exact_tc launch per tensor-core format over its jobs'
    tiles, weights translated once at creation."""
    from hotarubi_b200 import capi
    rng = np.random.default_rng(91)
    descs, keep, wants, outs = [], [], [], []
    for i in range(9):
        wfmt = (0, 1, 1, 0, 2)[i % 5]
        m, n, kb = int(rng.integers(1, 200)), int(rng.integers(8, 400)), int(rng.integers(1, 40))
        w, ws = _weights(rng, wfmt, n, kb) if wfmt != 2 else (
            rng.integers(0, 0x7E, (n, kb * 32)).astype(np.uint8),
            rng.integers(117, 124, (n, kb)).astype(np.uint8))
        pieces = None
        if wfmt == 1 and kb > 2:
            cut = sorted(rng.choice(np.arange(1, kb), size=2, replace=False))
            pieces = [int(cut[0]), int(cut[1] - cut[0]), int(kb - cut[1])]
        dw, dws = dev(w), dev(ws)
        c = torch.full((m, n), -1.0, device="cuda")
        if i % 2 == 0:
            x = rng.standard_normal((m, kb * 32)).astype(np.float32)
            q, s = cpu.encode_mxint8(x.view(np.uint32))
            a = dev(x)
            keep += [a]
            descs.append(capi.Library.desc(wfmt, m, n, kb * 32, a=a, w=dw, wscale=dws, c=c,
                                           pieces=pieces))
        else:
            q, s = _mxint8(rng, m, kb)
            aq, sq = dev(q), dev(s)
            keep += [aq, sq]
            descs.append(capi.Library.desc(wfmt, m, n, kb * 32, aq=aq, ascale=sq, w=dw,
                                           wscale=dws, c=c, pieces=pieces))
        wants.append(cpu.gemm_dense(wfmt, q, s, w, ws, n, pieces=pieces))
        keep += [dw, dws]
        outs.append(c)
    torch.cuda.synchronize()
    plan = hrb.plan(descs)
    for _ in range(2):
        plan.run()
        hrb.sync()
        for i, (c, want) in enumerate(zip(outs, wants)):
            assert (c.cpu().numpy().view(np.uint32) == want).all(), i
    plan.close()


@pytest.mark.parametrize("wfmt", [0, 1])
def test_larger_gemm(hrb, wfmt):
    """512 tokens x 1024 weight rows x 64 blocks: eight token tiles per
    weight tile, every CTA through several tiles."""
    rng = np.random.default_rng(70 + wfmt)
    q, s = _mxint8(rng, 512, 64)
    w, ws = _weights(rng, wfmt, 1024, 64)
    _check(hrb, wfmt, q, s, w, ws, 1024)


@pytest.mark.parametrize("wfmt", [0, 1])
def test_decode_token_tile(hrb, wfmt):
    """GEMMs of at most 16 tokens run 16-token tiles (four epilogue warps, two
    CTAs an SM); 17 tokens the 64-token tile: both sides of the switch, W8
    pieces, bias and accumulate."""
    rng = np.random.default_rng(80 + wfmt)
    for m, n, kb in ((1, 1000, 80), (16, 300, 40), (17, 300, 40), (9, 129, 130)):
        q, s = _mxint8(rng, m, kb)
        w, ws = _weights(rng, wfmt, n, kb)
        _check(hrb, wfmt, q, s, w, ws, n)
        bias = (rng.standard_normal(n).astype(np.float32)).view(np.uint32)
        c0 = rng.standard_normal((m, n)).astype(np.float32).view(np.uint32)
        pieces = [kb // 3, kb - kb // 3] if wfmt == 1 else None
        _check(hrb, wfmt, q, s, w, ws, n, bias=bias, c_init=c0, pieces=pieces)


@pytest.mark.skipif(not TC, reason="the rerun itself")
def test_dense_exact_kernel_passes_the_same_cases():
    """k_dense_exact (HRB_EXACT_TC=0) on every case above: both kernels give
    the oracle's bits."""
    env = dict(os.environ, HRB_EXACT_TC="0")
    here = os.path.dirname(os.path.abspath(__file__))
    r = subprocess.run([sys.executable, "-m", "pytest", "-x", "-q", "-m", "gpu",
                        "-p", "no:cacheprovider", os.path.join(here, "test_gpu_exact_tc.py")],
                       cwd=os.path.dirname(here), env=env, capture_output=True, text=True,
                       timeout=900)
    assert r.returncode == 0, r.stdout[-3000:] + r.stderr[-2000:]
