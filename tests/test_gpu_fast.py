"""HRB_MODE_FAST (the tcgen05 tensor-core path) against the exact answer.

Tolerance: the fast path computes the same exact products as the reference
(BF16 holds every MXINT8 activation and every W8/MXFP8 weight value exactly;
for MXFP4 weights the activations are split into three exact E2M1 digit
planes) but adds them in the tensor cores' order, in FP32.  Against the real-valued dot
product of the dequantized operands (float64), each output may differ by at
most (K/16 + 4) * 2^-23 * sum_k |a_k * w_k| (one FP32 rounding per 16-wide
MMA step plus the bias/accumulate adds, doubled for safety).  The tests also
report the max relative error and the ulp histogram against the bit-exact
chain of the oracle.
"""
import numpy as np
import pytest

from oracle import cpu

pytestmark = pytest.mark.gpu

torch = pytest.importorskip("torch")


def dev(x):
    return torch.from_numpy(np.ascontiguousarray(x)).cuda()


def dequant_a(x_bits):
    q, s = cpu.encode_mxint8(x_bits)
    sc = np.ldexp(1.0, s.astype(np.int64) - 133)
    return q.astype(np.float64) * np.repeat(sc, 32, axis=1), q, s


E2M1 = np.array([0, .5, 1, 1.5, 2, 3, 4, 6], np.float64)


def dequant_w(wfmt, w, ws, n, kp):
    sc = np.repeat(np.ldexp(1.0, ws.astype(np.int64) - 127), 32, axis=1)
    if wfmt == 0:
        codes = np.zeros((n, kp), np.uint8)
        codes[:, 0::2] = w & 0xF
        codes[:, 1::2] = w >> 4
        v = E2M1[codes & 7] * np.where(codes & 8, -1.0, 1.0)
        return v * sc
    if wfmt == 1:
        return w.view(np.int8).astype(np.float64) * sc * 2.0**-6
    units = np.vectorize(lambda c: cpu.oracle().hrbo_e4m3_units(int(c)))(np.arange(256))
    return units[w].astype(np.float64) * 2.0**-9 * sc


def weights(rng, wfmt, n, kb):
    k = kb * 32
    if wfmt == 0:
        code = rng.integers(0, 16, (n, k)).astype(np.uint8)
        e = rng.integers(-10, -3, (n, kb))
        code, e = cpu.canonical_mxfp4(code, e)
        return cpu.pack_nibbles(code), (e + 127).astype(np.uint8)
    if wfmt == 1:
        return (rng.integers(-128, 128, (n, k)).astype(np.int8).view(np.uint8),
                rng.integers(115, 125, (n, kb)).astype(np.uint8))
    code = rng.integers(0, 254, (n, k)).astype(np.uint8)
    code[code >= 0x7F] += 1
    return code, rng.integers(117, 124, (n, kb)).astype(np.uint8)


def ulp_hist(got, want):
    g = got.view(np.int32).astype(np.int64)
    w = want.view(np.int32).astype(np.int64)
    g = np.where(g < 0, -(g & 0x7FFFFFFF), g)
    w = np.where(w < 0, -(w & 0x7FFFFFFF), w)
    d = np.abs(g - w)
    return {"0": int((d == 0).sum()), "1": int((d == 1).sum()), "2-3": int(((d >= 2) & (d < 4)).sum()),
            "4-15": int(((d >= 4) & (d < 16)).sum()), ">=16": int((d >= 16).sum())}


def check_fast(hrb, wfmt, m, n, k, *, bias=False, accumulate=False, seed=0, plan=False,
               colscale=False, per_channel_w8=False, w8_kernel=0):
    """colscale: a random FP32 scale per output column (wcol_scale), applied
    before the bias (one more rounding, inside the tolerance's slack).
    per_channel_w8: W8 weights whose block scale bytes are all 133, so the
    weights are plain int8 values and wcol_scale carries their scale."""
    from hotarubi_b200 import capi
    rng = np.random.default_rng(seed)
    kb = (k + 31) // 32
    kp = kb * 32
    x = rng.standard_normal((m, k)).astype(np.float32)
    w, ws = weights(rng, wfmt, n, kb)
    if per_channel_w8:
        ws[:] = 133
    b = (rng.standard_normal(n) * 0.01).astype(np.float32) if bias else None
    c0 = rng.standard_normal((m, n)).astype(np.float32) if accumulate else None
    cs = None
    if colscale:
        cs = (rng.uniform(0.5, 2.0, n) * np.where(rng.random(n) < 0.3, -1.0, 1.0)
              * np.ldexp(1.0, rng.integers(-12, 4, n))).astype(np.float32)
    a_deq, q, s = dequant_a(x.view(np.uint32))
    w_deq = dequant_w(wfmt, w, ws, n, kp)
    ref = a_deq @ w_deq.T
    absref = np.abs(a_deq) @ np.abs(w_deq).T
    if cs is not None:
        ref *= cs.astype(np.float64)
        absref *= np.abs(cs.astype(np.float64))
    if c0 is not None:
        ref += c0
        absref += np.abs(c0)
    if b is not None:
        ref += b
        absref += np.abs(b)
    c = dev(c0) if c0 is not None else torch.zeros((m, n), dtype=torch.float32, device="cuda")
    keep = [dev(x), dev(w), dev(ws), None if b is None else dev(b),
            None if cs is None else dev(cs)]
    d = capi.Library.desc(wfmt, m, n, k, a=keep[0], w=keep[1], wscale=keep[2], bias=keep[3],
                          c=c, accumulate=accumulate, mode=capi.MODE_FAST, wcol_scale=keep[4],
                          w8_kernel=w8_kernel)
    if plan:
        p = hrb.plan([d])
        p.run()
        hrb.sync()
        p.close()
    else:
        hrb.dense(d)
        hrb.sync()
    got = c.cpu().numpy()
    tol = (k / 16 + 4) * 2.0**-23
    err = np.abs(got.astype(np.float64) - ref)
    bad = err > tol * absref + 1e-30
    assert not bad.any(), (f"{bad.sum()} outputs off; worst rel "
                           f"{(err / (absref + 1e-30)).max():.3e} tol {tol:.3e}")
    exact = cpu.gemm_dense(wfmt, q, s, w, ws, n,
                           bias_bits=None if b is None else b.view(np.uint32),
                           c_init=None if c0 is None else c0.view(np.uint32),
                           colscale_bits=None if cs is None else cs.view(np.uint32))
    ex = exact.view(np.float32).astype(np.float64)
    rel = np.abs(got - ex) / (np.abs(ex) + 1e-30)
    return {"max_rel_vs_exact": float(rel.max()), "ulp": ulp_hist(got, exact.view(np.float32))}


@pytest.mark.parametrize("wfmt", [0, 1, 2])
@pytest.mark.parametrize("shape", [(64, 960, 2560), (64, 2560, 960), (1, 8, 32),
                                   (100, 130, 224), (300, 200, 320), (70, 72, 720)])
def test_fast_matches_exact_dot_within_tolerance(hrb, wfmt, shape):
    m, n, k = shape
    check_fast(hrb, wfmt, m, n, k, seed=hash(shape) % 1000 + wfmt)


@pytest.mark.parametrize("wfmt", [0, 1, 2])
def test_fast_bias_and_accumulate(hrb, wfmt):
    check_fast(hrb, wfmt, 96, 160, 736, bias=True, accumulate=True, seed=5 + wfmt)


@pytest.mark.parametrize("wfmt", [0, 1, 2])
def test_fast_through_a_plan(hrb, wfmt):
    check_fast(hrb, wfmt, 64, 256, 512, bias=True, plan=True, seed=9 + wfmt)


@pytest.mark.parametrize("wfmt", [0, 1, 2])
@pytest.mark.parametrize("plan", [False, True])
def test_fast_column_scales(hrb, wfmt, plan):
    check_fast(hrb, wfmt, 130, 200, 480, bias=True, colscale=True, plan=plan, seed=31 + wfmt)
    check_fast(hrb, wfmt, 64, 256, 256, colscale=True, plan=plan, seed=41 + wfmt)


@pytest.mark.parametrize("shape", [(64, 960, 2560), (1, 16, 64), (200, 136, 416)])
@pytest.mark.parametrize("w8_kernel", [0, 1])
def test_fast_per_channel_int8_weights(hrb, shape, w8_kernel):
    """int8 weights with a per-output-channel FP32 scale and a fused
    scale/bias epilogue: W8 codes with block scale bytes 133 plus wcol_scale."""
    m, n, k = shape
    check_fast(hrb, 1, m, n, k, bias=True, colscale=True, per_channel_w8=True, seed=m + n,
               w8_kernel=w8_kernel)


@pytest.mark.parametrize("shape", [(64, 960, 2560), (64, 2560, 960), (1, 8, 32), (33, 130, 224),
                                   (64, 72, 720)])
def test_fast_w8_bf16_kernel_within_tolerance(hrb, shape):
    """W8 with at most 64 tokens on the BF16 kernel (w8_kernel = HRB_W8_BF16):
    the same bound as every fast GEMM; with bias, column scales and plans."""
    m, n, k = shape
    check_fast(hrb, 1, m, n, k, seed=hash(shape) % 1000, w8_kernel=1)
    check_fast(hrb, 1, m, n, k, bias=True, colscale=True, seed=7, w8_kernel=1)
    check_fast(hrb, 1, m, n, k, bias=True, plan=True, seed=8, w8_kernel=1)


def test_fast_batched_plan_of_mixed_shapes(hrb):
    from hotarubi_b200 import capi
    rng = np.random.default_rng(41)
    descs, keep, refs, outs = [], [], [], []
    for i in range(9):
        wfmt = i % 3
        m, n, kb = int(rng.integers(1, 300)), int(rng.integers(8, 300)), int(rng.integers(1, 30))
        x = rng.standard_normal((m, kb * 32)).astype(np.float32)
        w, ws = weights(rng, wfmt, n, kb)
        a_deq, _, _ = dequant_a(x.view(np.uint32))
        w_deq = dequant_w(wfmt, w, ws, n, kb * 32)
        refs.append((a_deq @ w_deq.T, np.abs(a_deq) @ np.abs(w_deq).T, kb * 32))
        t = [dev(x), dev(w), dev(ws)]
        keep += t
        c = torch.zeros((m, n), dtype=torch.float32, device="cuda")
        outs.append(c)
        descs.append(capi.Library.desc(wfmt, m, n, kb * 32, a=t[0], w=t[1], wscale=t[2], c=c,
                                       mode=capi.MODE_FAST))
    plan = hrb.plan(descs)
    plan.run()
    hrb.sync()
    for c, (ref, absref, k) in zip(outs, refs):
        got = c.cpu().numpy().astype(np.float64)
        assert (np.abs(got - ref) <= (k / 16 + 4) * 2.0**-23 * absref + 1e-30).all()
    plan.close()


@pytest.mark.parametrize("wfmt,w8_kernel", [(0, 0), (1, 0), (1, 1), (2, 0)])
@pytest.mark.parametrize("quant", [0, 1])
@pytest.mark.parametrize("m", [64, 70, 130])
def test_fast_activation_planes_are_exact(hrb, wfmt, w8_kernel, quant, m):
    """W = I (the code of 1.0: E2M1 0x2, W8 64 or E4M3 0x38, scale byte
    127), so every output is a single activation: C[r][i] = q[r][i] *
    2^(e_r - 6), which the digit-plane products (three E2M1 planes for MXFP4
    and W8, two E4M3 planes for MXFP8) and their FP32 sum give exactly, and
    so do the BF16 values of W8 with at most 64 tokens.  Bit-equality with
    the oracle's MXINT8 encoding pins the encoder (both rounding rules,
    padded K steps, ragged token tiles).  The exceptions: the digit planes
    encode blocks whose scale byte is below 6 (largest magnitude under
    2^-121) as zero; the BF16 path keeps them, and outputs under 2^-126 may
    come out of the tensor cores flushed to zero."""
    from hotarubi_b200 import capi
    rng = np.random.default_rng(70 + m + quant)
    n = k = 544                      # kb = 17: the third 256-element step is mostly padding
    x = rng.standard_normal((m, k)).astype(np.float32)
    x *= np.repeat(np.ldexp(1.0, rng.integers(-90, 90, (m, k // 32))), 32, axis=1).astype(np.float32)
    x[rng.random((m, k)) < 0.02] = 0.0
    x[:, 64:96] = 0.0                # an all-zero block
    sub = rng.random((m, k)) < 0.01  # subnormal inputs: the VEC rule reads them as zero
    x[sub] = np.float32(1e-40)
    if wfmt == 0:
        codes = np.zeros((n, k), np.uint8)
        codes[np.arange(n), np.arange(n)] = 2
        w = cpu.pack_nibbles(codes)
    else:
        w = np.zeros((n, k), np.uint8)
        w[np.arange(n), np.arange(n)] = 64 if wfmt == 1 else 0x38
    ws = np.full((n, k // 32), 127, np.uint8)
    c = torch.zeros((m, n), dtype=torch.float32, device="cuda")
    keep = [dev(x), dev(w), dev(ws)]
    d = capi.Library.desc(wfmt, m, n, k, a=keep[0], w=keep[1], wscale=keep[2], c=c,
                          mode=capi.MODE_FAST, quant=quant, w8_kernel=w8_kernel)
    hrb.dense(d)
    hrb.sync()
    got = c.cpu().numpy()
    xb = x.view(np.uint32)
    q, s = cpu.quantize_vec(xb) if quant == 1 else cpu.encode_mxint8(xb)
    want = (q.astype(np.float64) * np.repeat(np.ldexp(1.0, s.astype(np.int64) - 133), 32, axis=1))
    bf16_path = wfmt == 1 and m <= 64 and w8_kernel == 1
    if not bf16_path:
        want[np.repeat(s < 6, 32, axis=1)] = 0.0
    want = want[:, :n].astype(np.float32)
    if quant == 0:
        assert (s < 6).any()         # the subnormal-only block is covered
    if bf16_path:
        flushed = (got == 0) & (np.abs(want) < 2.0**-126)
        assert np.array_equal(np.where(flushed, 0, got.view(np.uint32)),
                              np.where(flushed, 0, want.view(np.uint32)))
    else:
        assert np.array_equal(got.view(np.uint32), want.view(np.uint32))


@pytest.mark.parametrize("quant", [0, 1])
@pytest.mark.parametrize("m,lda", [(70, 544), (64, 544), (130, 545)])
def test_fast_e2m1_planes_at_scale_boundaries(hrb, quant, m, lda):
    """W = I with MXFP4 weights as above, activation blocks whose largest
    magnitude has exponent field 5 .. 9 or 253: the E2M1 plane encoder's
    scaled rounding holds from field 8 on, fields 6 and 7 take the integer
    rules, fields below 6 encode as zero.  (At field 254 the top digit
    plane's partial product, up to 2 * 2^127, would overflow FP32 in the
    tensor cores whatever the encoder does.)  Rows of lda = 545 floats are not
    16-byte aligned and run the general encoder instead of the specialised
    one; both must give the oracle's MXINT8 codes."""
    from hotarubi_b200 import capi
    rng = np.random.default_rng(300 + m + quant + lda)
    n = k = 544
    kb = k // 32
    x = rng.standard_normal((m, k)).astype(np.float32)
    fields = np.array([5, 6, 7, 8, 9, 253, 127, 100])
    f = fields[rng.integers(0, fields.size, (m, kb))]
    # Each block scaled so that its largest magnitude is 1.5 * 2^(f - 127).
    blocks = x.reshape(m, kb, 32).astype(np.float64)
    top = np.abs(blocks).max(axis=2, keepdims=True)
    blocks = blocks / top * 1.5 * np.ldexp(1.0, (f - 127)[..., None].astype(np.int64))
    x = blocks.reshape(m, k).astype(np.float32)
    xs = np.zeros((m, lda), np.float32)
    xs[:, :k] = x
    codes = np.zeros((n, k), np.uint8)
    codes[np.arange(n), np.arange(n)] = 2
    w = cpu.pack_nibbles(codes)
    ws = np.full((n, kb), 127, np.uint8)
    c = torch.zeros((m, n), dtype=torch.float32, device="cuda")
    keep = [dev(xs), dev(w), dev(ws)]
    d = capi.Library.desc(0, m, n, k, a=keep[0], lda=lda, w=keep[1], wscale=keep[2], c=c,
                          mode=capi.MODE_FAST, quant=quant)
    hrb.dense(d)
    hrb.sync()
    got = c.cpu().numpy()
    xb = x.view(np.uint32)
    q, s = cpu.quantize_vec(xb) if quant == 1 else cpu.encode_mxint8(xb)
    assert set(np.unique(s)) >= {5, 6, 7, 8, 9, 253}
    want = q.astype(np.float64) * np.repeat(np.ldexp(1.0, s.astype(np.int64) - 133), 32, axis=1)
    want[np.repeat(s < 6, 32, axis=1)] = 0.0
    want = want[:, :n].astype(np.float32)
    assert np.array_equal(got.view(np.uint32), want.view(np.uint32))


@pytest.mark.parametrize("wfmt,w8_kernel", [(0, 0), (1, 0), (1, 1), (2, 0)])
@pytest.mark.parametrize("m", [288, 64])
def test_fast_weight_operands_are_exact(hrb, wfmt, w8_kernel, m):
    """A = I (every block's largest value 1.0: q = 64, scale 2^0), so output
    C[r][n] is weight W[n][r] alone, which the tensor-core path must give
    exactly: MXFP4 and MXFP8 codes as they are, W8 as its three E2M1 digit
    planes with scales e - 6 + 3p or, with at most 64 tokens, converted to
    BF16 in the kernel.  Bit-equality pins the weight translation."""
    from hotarubi_b200 import capi
    rng = np.random.default_rng(90 + wfmt + m)
    k = 288                           # kb = 9: the second 256-element step is mostly padding
    n = 200
    x = np.eye(m, k, dtype=np.float32)
    kb = k // 32
    if wfmt == 1:
        w = rng.integers(-128, 128, (n, k)).astype(np.int8).view(np.uint8)
        ws = rng.integers(100, 140, (n, kb)).astype(np.uint8)
    else:
        w, ws = weights(rng, wfmt, n, kb)
    c = torch.zeros((m, n), dtype=torch.float32, device="cuda")
    keep = [dev(x), dev(w), dev(ws)]
    d = capi.Library.desc(wfmt, m, n, k, a=keep[0], w=keep[1], wscale=keep[2], c=c,
                          mode=capi.MODE_FAST, w8_kernel=w8_kernel)
    hrb.dense(d)
    hrb.sync()
    got = c.cpu().numpy()
    want = dequant_w(wfmt, w, ws, n, k).T[:m].astype(np.float32)  # [r][n] = W[n][r]
    assert np.array_equal(got.view(np.uint32), want.view(np.uint32))


def test_fast_w8_bf16_extreme_scales(hrb):
    """W8 with at most 64 tokens converts w * 2^(e - 133) to BF16 in the
    kernel by a fused multiply-add (e <= 237) or a subtract and multiply
    (e > 237), with subnormal multipliers for e < 7: A = I shows each
    converted weight exactly (outputs under 2^-126 may come out flushed)."""
    from hotarubi_b200 import capi
    rng = np.random.default_rng(123)
    m, k, n = 64, 256, 136
    kb = k // 32
    x = np.eye(m, k, dtype=np.float32)
    w = rng.integers(-128, 128, (n, k)).astype(np.int8).view(np.uint8)
    # Up to 253: with 254, -128 * 2^121 overflows, and 0 * inf in the other
    # products of a column would make it NaN.
    ws = np.where(rng.random((n, kb)) < 0.5, rng.integers(0, 12, (n, kb)),
                  rng.integers(226, 254, (n, kb))).astype(np.uint8)
    c = torch.zeros((m, n), dtype=torch.float32, device="cuda")
    keep = [dev(x), dev(w), dev(ws)]
    d = capi.Library.desc(1, m, n, k, a=keep[0], w=keep[1], wscale=keep[2], c=c,
                          mode=capi.MODE_FAST, w8_kernel=capi.W8_BF16)
    hrb.dense(d)
    hrb.sync()
    got = c.cpu().numpy()
    want = dequant_w(1, w, ws, n, k).T[:m].astype(np.float32)
    flushed = (got == 0) & (np.abs(want) < 2.0**-126)
    assert np.array_equal(np.where(flushed, 0, got.view(np.uint32)),
                          np.where(flushed, 0, want.view(np.uint32)))


@pytest.mark.parametrize("mixed", [False, True])
def test_plan_run_host_matches_device_run(hrb, mixed):
    """hrb_plan_run_host (host activations in, C out; pipelined in chunks
    over three streams when the plan is one kind::mxf4 group) gives the
    same bits as the plan run on device-resident operands."""
    from hotarubi_b200 import capi
    rng = np.random.default_rng(55 + mixed)
    n_gemm = 12
    m, n, k = 40, 136, 320
    wfmts = [2 if (mixed and i % 3 == 0) else 0 for i in range(n_gemm)]
    a_dev = torch.zeros((n_gemm, m, k), dtype=torch.float32, device="cuda")
    c_dev = torch.zeros((n_gemm, m, n), dtype=torch.float32, device="cuda")
    keep, descs = [], []
    for i, f in enumerate(wfmts):
        w, ws = weights(rng, f, n, k // 32)
        t = [dev(w), dev(ws)]
        keep += t
        descs.append(capi.Library.desc(f, m, n, k, a=a_dev[i], w=t[0], wscale=t[1],
                                       c=c_dev[i], mode=capi.MODE_FAST))
    plan = hrb.plan(descs)
    x = rng.standard_normal((n_gemm, m, k)).astype(np.float32)
    # Device run for the expected bits.
    a_dev.copy_(torch.from_numpy(x))
    plan.run()
    hrb.sync()
    want = c_dev.cpu().numpy().copy()
    c_dev.zero_()
    # Host run: one contiguous pinned block, except one GEMM from its own
    # buffer (breaks a coalesced copy) and one skipped output.
    a_pin = torch.from_numpy(x).pin_memory()
    lone = torch.from_numpy(x[5].copy()).pin_memory()
    c_pin = torch.zeros((n_gemm, m, n), dtype=torch.float32).pin_memory()
    a_host = [a_pin[i] for i in range(n_gemm)]
    a_host[5] = lone
    c_host = [c_pin[i] for i in range(n_gemm)]
    c_host[7] = None
    a_dev.zero_()
    torch.cuda.synchronize()
    for _ in range(2):  # twice: the second run reuses the plan's streams
        plan.run_host(a_host, c_host)
        hrb.sync()
    got = c_pin.numpy()
    for i in range(n_gemm):
        if i == 7:
            assert not got[i].any()
        else:
            assert np.array_equal(got[i].view(np.uint32), want[i].view(np.uint32)), i
    plan.close()
