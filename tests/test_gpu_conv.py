"""Convolutions on the GPU (hrb_conv_dense, hrb_conv_plan_*), against the
conv chain of the oracle (pinned to a conv composed on the reference's DMA
engine and ExecuteGemm by tests/test_oracle_conv.py) and against that
composition's own outputs in tests/golden/conv.npz.

* HRB_MODE_EXACT: bit-exact, FP32 or MXINT8 maps, both position orders,
  several images, every weight format, channel planes (cin > 256), residual
  (accumulate), bias, RELU and the MXINT8 output copy.
* HRB_MODE_FAST (tensor cores; the map is encoded once and each output
  row's taps are gathered as operand blocks): within
  (K/16 + 4) * 2^-23 * sum_k |a_k w_k| of the real-valued conv of the
  dequantized operands, K = kh * kh * cin — the tolerance of every
  tensor-core test; RELU keeps the bound (it is 1-Lipschitz).
"""
import numpy as np
import pytest

from oracle import cpu

pytestmark = pytest.mark.gpu

torch = pytest.importorskip("torch")

E2M1 = np.array([0, .5, 1, 1.5, 2, 3, 4, 6], np.float64)


def dev(x):
    return torch.from_numpy(np.ascontiguousarray(x)).cuda()


def conv_weights(rng, wfmt, cout, k):
    kb = k // 32
    if wfmt == cpu.WFMT_MXFP4:
        code = rng.integers(0, 16, (cout, k)).astype(np.uint8)
        e = rng.integers(-10, -3, (cout, kb))
        code, e = cpu.canonical_mxfp4(code, e)
        return cpu.pack_nibbles(code), (e + 127).astype(np.uint8)
    if wfmt == cpu.WFMT_W8:
        return (rng.integers(-128, 128, (cout, k)).astype(np.int8).view(np.uint8),
                rng.integers(115, 125, (cout, kb)).astype(np.uint8))
    code = rng.integers(0, 254, (cout, k)).astype(np.uint8)
    code[code >= 0x7F] += 1
    return code, rng.integers(117, 124, (cout, kb)).astype(np.uint8)


def dequant_w(wfmt, w, ws):
    n = w.shape[0]
    sc = np.repeat(np.ldexp(1.0, ws.astype(np.int64) - 127), 32, axis=1)
    if wfmt == cpu.WFMT_MXFP4:
        codes = np.zeros((n, w.shape[1] * 2), np.uint8)
        codes[:, 0::2] = w & 0xF
        codes[:, 1::2] = w >> 4
        return E2M1[codes & 7] * np.where(codes & 8, -1.0, 1.0) * sc
    if wfmt == cpu.WFMT_W8:
        return w.view(np.int8).astype(np.float64) * sc * 2.0**-6
    units = np.array([cpu.oracle().hrbo_e4m3_units(c) for c in range(256)], np.int64)
    return units[w].astype(np.float64) * 2.0**-9 * sc


def run_conv(hrb, wfmt, x, images, H, W, cin, cout, kh, stride, w, ws, *, mode, order=0,
             bias=None, c0=None, relu=False, mxint8_map=None, cq=False, plan=False):
    from hotarubi_b200 import capi
    ho, wo = H // stride, W // stride
    m = images * ho * wo
    c = dev(c0) if c0 is not None else torch.zeros((m, cout), dtype=torch.float32, device="cuda")
    keep = [dev(w), dev(ws), None if bias is None else dev(bias)]
    kw = {}
    if mxint8_map is not None:
        keep += [dev(mxint8_map[0]), dev(mxint8_map[1])]
        kw = {"aq": keep[-2], "ascale": keep[-1]}
    else:
        keep.append(dev(x))
        kw = {"a": keep[-1]}
    kpn = (cout + 31) // 32 * 32
    q = torch.zeros((m, kpn), dtype=torch.int8, device="cuda") if cq else None
    s = torch.zeros((m, kpn // 32), dtype=torch.uint8, device="cuda") if cq else None
    d = capi.conv_desc(wfmt, images, H, W, cin, cout, kh, stride, order=order, w=keep[0],
                       wscale=keep[1], bias=keep[2], c=c, accumulate=c0 is not None, relu=relu,
                       mode=mode, cq=q, cscale=s, **kw)
    if plan:
        p = hrb.conv_plan(d)
        p.run()
        hrb.sync()
        p.close()
    else:
        hrb.conv(d)
        hrb.sync()
    out = c.cpu().numpy()
    if cq:
        return out, q.cpu().numpy(), s.cpu().numpy()
    return out


@pytest.mark.parametrize("name", ["s1_3x3_16x12x64x32", "s1_3x3_4x4x512x16_res_relu",
                                  "s2_3x3_8x6x64x256_relu", "s1_1x1_4x4x256x512_res",
                                  "s2_1x1_12x8x64x24_relu"])
@pytest.mark.parametrize("mxint8", [False, True])
def test_conv_exact_on_reference_golden(hrb, golden, name, mxint8):
    from hotarubi_b200 import capi
    g = golden("conv.npz")
    parts = name.split("_")
    stride, kh = int(parts[0][1:]), int(parts[1][0])
    H, W, cin, cout = (int(v) for v in parts[2].split("x"))
    x = g[f"{name}/x"]
    res = g.get(f"{name}/residual")
    mmap = cpu.encode_mxint8(x.view(np.uint32)) if mxint8 else None
    got = run_conv(hrb, capi.WFMT_MXFP4, x, 1, H, W, cin, cout, kh, stride, g[f"{name}/w"],
                   g[f"{name}/wscale"], mode=capi.MODE_EXACT, bias=g[f"{name}/bias"].view(np.float32),
                   c0=None if res is None else res.view(np.float32), relu="relu" in parts,
                   mxint8_map=mmap)
    assert (got.view(np.uint32) == g[f"{name}/c"]).all()


CASES = [  # wfmt, images, H, W, cin, cout, kh, stride, order, bias, residual, relu
    (0, 2, 8, 12, 64, 48, 3, 1, 0, True, False, True),
    (0, 3, 6, 10, 128, 136, 3, 2, 1, True, True, False),
    (1, 2, 8, 8, 256, 40, 3, 1, 1, False, True, True),
    (2, 2, 4, 12, 96, 64, 3, 1, 0, True, False, False),
    (0, 1, 8, 4, 512, 24, 3, 1, 0, True, False, True),      # two channel planes
    (1, 1, 4, 8, 512, 16, 1, 2, 1, True, True, False),
    (2, 4, 12, 6, 32, 8, 1, 1, 0, False, False, True),
    (0, 3, 10, 14, 256, 136, 3, 2, 1, True, True, True),    # the GEMM gathers its own blocks
    (0, 2, 16, 20, 256, 64, 1, 1, 0, False, False, False),
]


def case_inputs(case, seed):
    wfmt, images, H, W, cin, cout, kh, stride, order, b, r, relu = case
    rng = np.random.default_rng(seed)
    x = rng.standard_normal((images, H * W, cin)).astype(np.float32)
    x[:, rng.random(H * W) < 0.1] = 0.0
    w, ws = conv_weights(rng, wfmt, cout, kh * kh * cin)
    bias = (rng.standard_normal(cout) * 0.1).astype(np.float32) if b else None
    m = images * (H // stride) * (W // stride)
    c0 = rng.standard_normal((m, cout)).astype(np.float32) if r else None
    return x, w, ws, bias, c0


@pytest.mark.parametrize("case", CASES)
def test_conv_exact_matches_oracle(hrb, case):
    from hotarubi_b200 import capi
    wfmt, images, H, W, cin, cout, kh, stride, order, _, _, relu = case
    x, w, ws, bias, c0 = case_inputs(case, sum(case[:8]))
    aq, asc = cpu.encode_mxint8(x.reshape(-1, cin).view(np.uint32))
    want = cpu.conv_dense(wfmt, aq, asc, images, H, W, cin, cout, kh, stride, w, ws, order=order,
                          bias_bits=None if bias is None else bias.view(np.uint32),
                          c_init=None if c0 is None else c0.view(np.uint32), relu_out=relu)
    for plan in (False, True):
        got, q, s = run_conv(hrb, wfmt, x, images, H, W, cin, cout, kh, stride, w, ws,
                             mode=capi.MODE_EXACT, order=order, bias=bias, c0=c0, relu=relu,
                             cq=True, plan=plan)
        assert (got.view(np.uint32) == want).all()
        wq, wsc = cpu.quantize_vec(want)
        assert (q == wq).all() and (s == wsc).all()


def fast_bound(case, x, w, ws, bias, c0):
    wfmt, images, H, W, cin, cout, kh, stride, order, _, _, relu = case
    aq, asc = cpu.encode_mxint8(x.reshape(-1, cin).view(np.uint32))
    q, sc = cpu.conv_im2col(aq, asc, images, H, W, cin, kh, stride, order)
    wq, wsc = cpu.conv_weights(wfmt, w, ws, cout, cin, kh)
    a_deq = q.astype(np.float64) * np.repeat(np.ldexp(1.0, sc.astype(np.int64) - 133), 32, axis=1)
    w_deq = dequant_w(wfmt, wq, wsc)
    ref = a_deq @ w_deq.T
    absref = np.abs(a_deq) @ np.abs(w_deq).T
    if c0 is not None:
        ref += c0
        absref += np.abs(c0)
    if bias is not None:
        ref += bias
        absref += np.abs(bias)
    if relu:
        ref = np.maximum(ref, 0.0)
    k = kh * kh * cin
    return ref, absref, (k / 16 + 4) * 2.0**-23


@pytest.mark.parametrize("case", CASES)
def test_conv_fast_within_tolerance(hrb, case):
    from hotarubi_b200 import capi
    wfmt, images, H, W, cin, cout, kh, stride, order, _, _, relu = case
    x, w, ws, bias, c0 = case_inputs(case, 7 + sum(case[:8]))
    ref, absref, tol = fast_bound(case, x, w, ws, bias, c0)
    for plan in (False, True):
        got, q, s = run_conv(hrb, wfmt, x, images, H, W, cin, cout, kh, stride, w, ws,
                             mode=capi.MODE_FAST, order=order, bias=bias, c0=c0, relu=relu,
                             cq=True, plan=plan)
        err = np.abs(got.astype(np.float64) - ref)
        assert (err <= tol * absref + 1e-30).all(), f"worst {(err / (absref + 1e-30)).max():.3e}"
        # The epilogue's MXINT8 copy is the VEC encoding of its own FP32 output.
        wq, wsc = cpu.quantize_vec(got.view(np.uint32))
        assert (q == wq).all() and (s == wsc).all()


def test_conv_c5_full_size(hrb):
    """The C5 conv (3x3, 256 -> 256, 16 x 44 maps, 6 cameras x batch 8:
    M = 33,792, K = 2,304): the tensor-core path within tolerance and the
    exact path bit-exact, checked on 512 sampled output rows."""
    from hotarubi_b200 import capi
    rng = np.random.default_rng(55)
    images, H, W, cin, cout = 48, 16, 44, 256, 256
    x = rng.standard_normal((images, H * W, cin)).astype(np.float32)
    w, ws = conv_weights(rng, capi.WFMT_MXFP4, cout, 9 * cin)
    bias = (rng.standard_normal(cout) * 0.1).astype(np.float32)
    aq, asc = cpu.encode_mxint8(x.reshape(-1, cin).view(np.uint32))
    q, sc = cpu.conv_im2col(aq, asc, images, H, W, cin, 3, 1, 1)
    rows = np.sort(rng.choice(q.shape[0], 512, replace=False))
    rows[:2] = [0, 1]   # a corner position
    q, sc = q[rows], sc[rows]
    want = cpu.gemm_dense(capi.WFMT_MXFP4, q, sc, w, ws, cout, bias_bits=bias.view(np.uint32))
    exact = run_conv(hrb, capi.WFMT_MXFP4, x, images, H, W, cin, cout, 3, 1, w, ws,
                     mode=capi.MODE_EXACT, order=1, bias=bias)
    assert (exact[rows].view(np.uint32) == want).all()
    fast = run_conv(hrb, capi.WFMT_MXFP4, x, images, H, W, cin, cout, 3, 1, w, ws,
                    mode=capi.MODE_FAST, order=1, bias=bias)
    a_deq = q.astype(np.float64) * np.repeat(np.ldexp(1.0, sc.astype(np.int64) - 133), 32, axis=1)
    w_deq = dequant_w(capi.WFMT_MXFP4, w, ws)
    ref = a_deq @ w_deq.T + bias
    absref = np.abs(a_deq) @ np.abs(w_deq).T + np.abs(bias)
    tol = (9 * cin / 16 + 4) * 2.0**-23
    assert (np.abs(fast[rows] - ref) <= tol * absref + 1e-30).all()


def test_conv_rejects_what_the_emitter_rejects(hrb):
    from hotarubi_b200 import capi
    x = torch.zeros((16, 320), dtype=torch.float32, device="cuda")
    w = torch.zeros((8, 9 * 320), dtype=torch.uint8, device="cuda")
    ws = torch.zeros((8, 90), dtype=torch.uint8, device="cuda")
    c = torch.zeros((16, 8), dtype=torch.float32, device="cuda")
    with pytest.raises(capi.HrbError) as e:
        hrb.conv(capi.conv_desc(0, 1, 4, 4, 320, 8, 3, 1, a=x, w=w, wscale=ws, c=c))
    assert e.value.status == capi.HRB_EINVAL and "4x4x320 is not supported" in e.value.message
    with pytest.raises(capi.HrbError) as e:
        hrb.conv(capi.conv_desc(0, 1, 4, 4, 32, 8, 5, 1, a=x, w=w, wscale=ws, c=c))
    assert "5x5 kernel" in e.value.message
