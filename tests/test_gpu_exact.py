"""Parity of the CUDA path with the oracle and the reference's fixtures.

Every test here runs the product through its C ABI (libhrb_gemm.so, via
hotarubi_b200.capi) and compares FP32 bit patterns with the CPU checker:
the exact path must be bit-identical.  Device buffers come from torch.
"""
import numpy as np
import pytest

from oracle import cpu

pytestmark = pytest.mark.gpu

torch = pytest.importorskip("torch")


def dev(x: np.ndarray):
    return torch.from_numpy(np.ascontiguousarray(x)).cuda()


def host(t) -> np.ndarray:
    torch.cuda.synchronize()
    return t.cpu().numpy()


# --------------------------------------------------------------------------
# ISS drop-in

def _cmd(capi, fields):
    c = capi.GemmCmd()
    for name, v in zip(("a_base", "a_stride", "kb", "m", "w_base", "w_stride", "n8",
                        "c_base", "wmode", "acc"), fields):
        setattr(c, name, int(v))
    return c


def test_exec_on_gemm_array_test_cases(hrb, golden):
    from hotarubi_b200 import capi
    case = golden("iss_unit.npz")
    for name in case["names"]:
        abuf = np.zeros((8192, 132), np.uint8)
        wbuf = np.zeros((2048, 144), np.uint8)
        fbuf = np.zeros((4096, 32), np.uint32)
        abuf[case[f"{name}/a_idx"]] = case[f"{name}/a_words"]
        wbuf[case[f"{name}/w_idx"]] = case[f"{name}/w_words"]
        fbuf[case[f"{name}/c_idx"]] = case[f"{name}/c_before"]
        before = fbuf.copy()
        hrb.exec(_cmd(capi, case[f"{name}/cmd"]), abuf, wbuf, fbuf)
        idx = case[f"{name}/c_idx"]
        assert (fbuf[idx] == case[f"{name}/c_after"]).all(), name
        rest = np.setdiff1d(np.arange(4096), idx)
        assert (fbuf[rest] == before[rest]).all(), name


def test_exec_on_tb_gemm_test_cases(hrb, golden):
    from hotarubi_b200 import capi
    case = golden("tb_gemm.npz")
    for name in case["names"]:
        init = case[f"{name}/c_init"]
        fbuf = np.zeros((4096, 32), np.uint32)
        fbuf[:init.shape[0]] = init
        for i, cmd in enumerate(case[f"{name}/cmds"]):
            abuf = np.zeros((8192, 132), np.uint8)
            wbuf = np.zeros((2048, 144), np.uint8)
            a, w = case[f"{name}/a{i}"], case[f"{name}/w{i}"]
            abuf[:a.shape[0]] = a[:, :132]
            wbuf[:w.shape[0]] = w
            hrb.exec(_cmd(capi, cmd), abuf, wbuf, fbuf)
        assert (fbuf[:init.shape[0]] == case[f"{name}/c_expected"]).all(), name


def _random_memories(rng, scale_lo=118, scale_hi=137):
    abuf = rng.integers(0, 256, (8192, 132)).astype(np.uint8)
    abuf[:, 128:] = rng.integers(scale_lo, scale_hi, (8192, 4))
    wbuf = rng.integers(0, 256, (2048, 144)).astype(np.uint8)
    wbuf[:, 128:136] = rng.integers(scale_lo, scale_hi, (2048, 8))
    wbuf[:, 136:] = 0
    fbuf = (rng.standard_normal((4096, 32)).astype(np.float32) * 4).view(np.uint32)
    return abuf, wbuf, fbuf


def test_exec_random_commands_vs_oracle(hrb):
    from hotarubi_b200 import capi
    rng = np.random.default_rng(21)
    abuf, wbuf, fbuf = _random_memories(rng)
    for t in range(24):
        m = int(rng.integers(1, 32)) * 32
        kb = int(rng.integers(1, 40))
        n8 = int(rng.integers(1, 256)) if t % 3 == 0 else int(rng.integers(1, 24))
        fields = [int(rng.integers(0, 1 << 20)), kb + int(rng.integers(0, 3)), kb, m,
                  int(rng.integers(0, 1 << 20)), int(rng.integers(1, kb + 4)), n8,
                  int(rng.integers(0, 1 << 20)), t % 4, t % 2]
        want = fbuf.copy()
        assert cpu.execute_gemm(fields, abuf, wbuf, want) == 0
        got = fbuf.copy()
        hrb.exec(_cmd(capi, fields), abuf, wbuf, got)
        assert (got == want).all(), fields


def test_exec_aliasing_output_words_follow_iss_order(hrb):
    """m/4 * n8 > 4096: two (quad, group) pairs share FBUF words, so the ISS
    loop order (groups outer, quads inner) decides the result."""
    from hotarubi_b200 import capi
    rng = np.random.default_rng(22)
    abuf, wbuf, fbuf = _random_memories(rng)
    fields = [5, 3, 3, 992, 11, 3, 40, 77, 0, 1]
    want = fbuf.copy()
    assert cpu.execute_gemm(fields, abuf, wbuf, want) == 0
    got = fbuf.copy()
    hrb.exec(_cmd(capi, fields), abuf, wbuf, got)
    assert (got == want).all()


def test_exec_infinities_and_extreme_scales_vs_oracle(hrb):
    """Scale bytes near 0 and 255 make block values flush to +0 or overflow
    to +-inf; FBUF starts with infinities, NaNs, subnormals and -0.  The ISS
    reads exponent 255 as an ordinary exponent; the GPU matches it bit for
    bit (slow integer path)."""
    from hotarubi_b200 import capi
    rng = np.random.default_rng(23)
    abuf, wbuf, fbuf = _random_memories(rng, 0, 256)
    specials = np.array([0x7F800000, 0xFF800000, 0x7FC00000, 0x00000001, 0x80000000,
                         0x807FFFFF, 0x7F7FFFFF, 0xFF7FFFFF], np.uint32)
    fbuf[:, :8] = specials
    for t in range(12):
        kb = int(rng.integers(1, 12))
        fields = [int(rng.integers(0, 8192)), kb, kb, 64, int(rng.integers(0, 2048)), kb,
                  int(rng.integers(1, 9)), int(rng.integers(0, 4096)), t % 4, 1]
        want = fbuf.copy()
        assert cpu.execute_gemm(fields, abuf, wbuf, want) == 0
        got = fbuf.copy()
        hrb.exec(_cmd(capi, fields), abuf, wbuf, got)
        assert (got == want).all(), fields


def test_exec_rejects_what_execute_gemm_rejects(hrb):
    from hotarubi_b200 import capi
    abuf = np.zeros(8192 * 132, np.uint8)
    wbuf = np.zeros(2048 * 144, np.uint8)
    fbuf = np.zeros(4096 * 32, np.uint32)
    for fields, text in (([0, 1, 1, 16, 0, 1, 1, 0, 0, 0], "m = 16"),
                         ([0, 1, 2, 32, 0, 1, 1, 0, 0, 0], "kb = 2"),
                         ([0, 1, 1, 32, 0, 1, 0, 0, 0, 0], "n8 = 0")):
        with pytest.raises(capi.HrbError) as e:
            hrb.exec(_cmd(capi, fields), abuf, wbuf, fbuf)
        assert e.value.status == capi.HRB_EINVAL and text in e.value.message


def test_exec_device_memories(hrb, golden):
    from hotarubi_b200 import capi
    case = golden("iss_unit.npz")
    name = "every_mode_1"
    abuf = np.zeros((8192, 132), np.uint8)
    wbuf = np.zeros((2048, 144), np.uint8)
    fbuf = np.zeros((4096, 32), np.uint32)
    abuf[case[f"{name}/a_idx"]] = case[f"{name}/a_words"]
    wbuf[case[f"{name}/w_idx"]] = case[f"{name}/w_words"]
    fbuf[case[f"{name}/c_idx"]] = case[f"{name}/c_before"]
    da, dw, df = dev(abuf), dev(wbuf), dev(fbuf)
    hrb.exec_device(_cmd(capi, case[f"{name}/cmd"]), da, dw, df)
    hrb.sync()
    out = host(df)
    assert (out[case[f"{name}/c_idx"]] == case[f"{name}/c_after"]).all()


# --------------------------------------------------------------------------
# Quantizer

@pytest.mark.parametrize("name", ["q_64x96", "q_8x720", "q_4x40"])
def test_quantize_on_golden(hrb, golden, name):
    case = golden("quantize.npz")
    x = case[f"{name}/x"]
    rows, cols = x.shape
    kp = (cols + 31) // 32 * 32
    q = torch.zeros((rows, kp), dtype=torch.int8, device="cuda")
    s = torch.zeros((rows, kp // 32), dtype=torch.uint8, device="cuda")
    hrb.quantize(dev(x.view(np.float32)), rows, cols, q, s)
    hrb.sync()
    assert (host(q) == case[f"{name}/q"]).all()
    assert (host(s) == case[f"{name}/scale"]).all()


def test_quantize_vec_rule_and_strided_rows(hrb, golden):
    from hotarubi_b200 import capi
    case = golden("quantize.npz")
    x = case["vec/x"]
    want_q, want_s = cpu.quantize_vec(x)
    rows, cols = x.shape
    wide = np.zeros((rows, cols + 7), np.uint32)
    wide[:, :cols] = x
    q = torch.zeros((rows, cols), dtype=torch.int8, device="cuda")
    s = torch.zeros((rows, cols // 32), dtype=torch.uint8, device="cuda")
    hrb.quantize(dev(wide.view(np.float32)), rows, cols, q, s, ldx=cols + 7,
                 quant=capi.QUANT_VEC)
    hrb.sync()
    assert (host(q) == want_q).all() and (host(s) == want_s).all()


def test_quantize_flags_non_finite_input(hrb):
    from hotarubi_b200 import capi
    x = np.zeros((4, 64), np.float32)
    x[2, 5] = np.inf
    q = torch.zeros((4, 64), dtype=torch.int8, device="cuda")
    s = torch.zeros((4, 2), dtype=torch.uint8, device="cuda")
    hrb.quantize(dev(x), 4, 64, q, s)
    with pytest.raises(capi.HrbError) as e:
        hrb.sync()
    assert e.value.status == capi.HRB_EDATA
    hrb.sync()  # the flag clears


def test_quantize_large_random_vs_oracle(hrb):
    rng = np.random.default_rng(31)
    x = (rng.standard_normal((301, 1000)) * np.exp(rng.uniform(-30, 30, (301, 1)))).astype(
        np.float32)
    want_q, want_s = cpu.encode_mxint8(x.view(np.uint32))
    q = torch.zeros(want_q.shape, dtype=torch.int8, device="cuda")
    s = torch.zeros(want_s.shape, dtype=torch.uint8, device="cuda")
    hrb.quantize(dev(x), 301, 1000, q, s)
    hrb.sync()
    assert (host(q) == want_q).all() and (host(s) == want_s).all()


# --------------------------------------------------------------------------
# Dense exact GEMM

def _weights(rng, wfmt, n, kb):
    k = kb * 32
    if wfmt == cpu.WFMT_MXFP4:
        code = rng.integers(0, 16, (n, k)).astype(np.uint8)
        e = rng.integers(-10, -3, (n, kb))
        code, e = cpu.canonical_mxfp4(code, e)
        return cpu.pack_nibbles(code), (e + 127).astype(np.uint8)
    if wfmt == cpu.WFMT_W8:
        return (rng.integers(-128, 128, (n, k)).astype(np.int8).view(np.uint8),
                rng.integers(115, 125, (n, kb)).astype(np.uint8))
    code = rng.integers(0, 254, (n, k)).astype(np.uint8)
    code[code >= 0x7F] += 1
    return code, rng.integers(117, 124, (n, kb)).astype(np.uint8)


def _run_dense(hrb, wfmt, x, w, ws, n, *, bias=None, c_init=None, pieces=None,
               mode=0, fp32_input=True, colscale=None):
    from hotarubi_b200 import capi
    m, k = x.shape
    c = dev(c_init.view(np.float32)) if c_init is not None else torch.zeros(
        (m, n), dtype=torch.float32, device="cuda")
    kw = dict(w=dev(w), wscale=dev(ws), c=c, bias=None if bias is None else dev(bias),
              accumulate=c_init is not None, pieces=pieces, mode=mode,
              wcol_scale=None if colscale is None else dev(colscale))
    keep = [kw["w"], kw["wscale"], kw["bias"], kw["wcol_scale"]]
    if fp32_input:
        a = dev(x.view(np.float32))
        keep.append(a)
        d = capi.Library.desc(wfmt, m, n, k, a=a, **kw)
    else:
        q, s = cpu.encode_mxint8(x)
        aq, sq = dev(q), dev(s)
        keep += [aq, sq]
        d = capi.Library.desc(wfmt, m, n, k, aq=aq, ascale=sq, **kw)
    hrb.dense(d)
    hrb.sync()
    return host(c).view(np.uint32)


@pytest.mark.parametrize("wfmt", [0, 1, 2])
@pytest.mark.parametrize("shape", [(64, 96, 30), (1, 8, 1), (100, 130, 7), (33, 257, 80)])
def test_dense_exact_vs_oracle(hrb, wfmt, shape):
    m, n, kb = shape
    rng = np.random.default_rng(1000 + 10 * wfmt + kb)
    x = rng.standard_normal((m, kb * 32)).astype(np.float32).view(np.uint32)
    w, ws = _weights(rng, wfmt, n, kb)
    q, s = cpu.encode_mxint8(x)
    want = cpu.gemm_dense(wfmt, q, s, w, ws, n)
    got = _run_dense(hrb, wfmt, x, w, ws, n)
    assert (got == want).all()
    got2 = _run_dense(hrb, wfmt, x, w, ws, n, fp32_input=False)
    assert (got2 == want).all()


@pytest.mark.parametrize("wfmt", [0, 1, 2])
def test_dense_exact_bias_accumulate_pieces(hrb, wfmt):
    rng = np.random.default_rng(77 + wfmt)
    m, n, kb = 70, 72, 9
    x = rng.standard_normal((m, kb * 32 - 5)).astype(np.float32).view(np.uint32)
    w, ws = _weights(rng, wfmt, n, kb)
    bias = (rng.standard_normal(n).astype(np.float32) * 0.01).view(np.uint32)
    c0 = rng.standard_normal((m, n)).astype(np.float32).view(np.uint32)
    q, s = cpu.encode_mxint8(x)
    want = cpu.gemm_dense(wfmt, q, s, w, ws, n, bias_bits=bias, c_init=c0, pieces=[2, 4, 3])
    got = _run_dense(hrb, wfmt, x, w, ws, n, bias=bias, c_init=c0, pieces=[2, 4, 3])
    assert (got == want).all()


def _boundary_scales(rng, c, n):
    """Column scales: random magnitudes, zeros, ones that overflow, and ones
    that put row 0's product a few ulps either side of 2^-126 (where the
    ISS, rounding to 24 bits before it flushes, and an IEEE multiply with
    flush to zero part ways)."""
    cs = (rng.uniform(0.5, 2.0, n) * np.ldexp(1.0, rng.integers(-20, 20, n))).astype(np.float32)
    cs[rng.random(n) < 0.3] *= -1
    cs[5] = 0.0
    cs[6] = np.float32(3e38)
    v = c[0].view(np.float32).astype(np.float64)
    for j in range(8, min(n, 40)):
        if v[j] == 0 or not np.isfinite(v[j]):
            continue
        base = np.float32(2.0**-126 / abs(v[j]))
        cs[j] = np.frombuffer(np.array([base.view(np.uint32) + (j % 7) - 3], np.uint32).tobytes(),
                              np.float32)[0]
    return cs


@pytest.mark.parametrize("wfmt", [0, 1, 2])
def test_dense_exact_column_scales(hrb, wfmt):
    """wcol_scale in the exact mode: the ISS's FP32 multiply, then the bias
    add, bit for bit (FP32 and MXINT8 inputs, ragged sizes)."""
    rng = np.random.default_rng(300 + wfmt)
    for m, n, kb in ((70, 72, 9), (1, 40, 3), (130, 200, 17)):
        x = rng.standard_normal((m, kb * 32 - 3)).astype(np.float32).view(np.uint32)
        w, ws = _weights(rng, wfmt, n, kb)
        bias = (rng.standard_normal(n).astype(np.float32) * 0.01).view(np.uint32)
        q, s = cpu.encode_mxint8(x)
        plain = cpu.gemm_dense(wfmt, q, s, w, ws, n)
        cs = _boundary_scales(rng, plain, n)
        for b in (None, bias):
            want = cpu.gemm_dense(wfmt, q, s, w, ws, n, bias_bits=b,
                                  colscale_bits=cs.view(np.uint32))
            got = _run_dense(hrb, wfmt, x, w, ws, n, bias=b, colscale=cs)
            assert (got == want).all(), (m, n, kb, b is None)
            got = _run_dense(hrb, wfmt, x, w, ws, n, bias=b, colscale=cs, fp32_input=False)
            assert (got == want).all(), (m, n, kb, b is None)


def test_dense_exact_column_scales_with_special_chains(hrb):
    """Chains at infinity or NaN (block scales that overflow) through the
    column scale: the integer slow path applies the same multiply."""
    rng = np.random.default_rng(17)
    m, n, kb = 32, 64, 6
    for wfmt in (0, 1, 2):
        x = rng.standard_normal((m, kb * 32)).astype(np.float32).view(np.uint32)
        w, ws = _weights(rng, wfmt, n, kb)
        ws[::5, 2] = 254
        q, s = cpu.encode_mxint8(x)
        cs = (rng.standard_normal(n) * 4).astype(np.float32)
        cs[::9] = 0.0
        bias = (rng.standard_normal(n).astype(np.float32)).view(np.uint32)
        want = cpu.gemm_dense(wfmt, q, s, w, ws, n, bias_bits=bias, colscale_bits=cs.view(np.uint32))
        got = _run_dense(hrb, wfmt, x, w, ws, n, bias=bias, colscale=cs)
        assert (got == want).all(), wfmt


def test_dense_column_scales_host_entry_and_accumulate_refused(hrb):
    from hotarubi_b200 import capi
    rng = np.random.default_rng(23)
    m, n, kb = 48, 80, 7
    x = rng.standard_normal((m, kb * 32)).astype(np.float32)
    w, ws = _weights(rng, 1, n, kb)
    ws[:] = 133  # int8 weights: every code counts as its integer value
    bias = (rng.standard_normal(n) * 0.01).astype(np.float32)
    cs = (rng.uniform(0.5, 2.0, n) * 2.0**-10).astype(np.float32)
    q, s = cpu.encode_mxint8(x.view(np.uint32))
    want = cpu.gemm_dense(1, q, s, w, ws, n, bias_bits=bias.view(np.uint32),
                          colscale_bits=cs.view(np.uint32))
    c = np.zeros((m, n), np.float32)
    hrb.dense_host(capi.Library.desc(1, m, n, kb * 32, a=x, w=w, wscale=ws, bias=bias, c=c,
                                     wcol_scale=cs))
    assert (c.view(np.uint32) == want).all()
    t = [dev(x), dev(w), dev(ws), dev(bias), dev(cs)]
    cd = torch.zeros((m, n), dtype=torch.float32, device="cuda")
    d = capi.Library.desc(1, m, n, kb * 32, a=t[0], w=t[1], wscale=t[2], c=cd, wcol_scale=t[4],
                          accumulate=True)
    with pytest.raises(capi.HrbError):
        hrb.dense(d)


def test_dense_on_reference_iss_fixtures(hrb, golden):
    case = golden("dense.npz")
    for name in case["names"]:
        want = case[f"{name}/c"]
        got = _run_dense(hrb, int(case[f"{name}/wfmt"]), case[f"{name}/x"], case[f"{name}/w"],
                         case[f"{name}/wscale"], want.shape[1])
        assert (got == want).all(), name


def test_dense_mxfp8_fixture(hrb, golden):
    case = golden("dense_mxfp8.npz")
    got = _run_dense(hrb, 2, case["x"], case["w"], case["wscale"], case["c"].shape[1],
                     bias=case["bias"])
    assert (got == case["c"]).all()


def test_dense_extreme_scales_and_special_inputs(hrb):
    """Weight scales that overflow block values to infinity, accumulators that
    start at infinity or NaN: the integer slow path reproduces the chain."""
    rng = np.random.default_rng(5)
    m, n, kb = 32, 64, 6
    for wfmt in (0, 1, 2):
        x = rng.standard_normal((m, kb * 32)).astype(np.float32).view(np.uint32)
        w, ws = _weights(rng, wfmt, n, kb)
        ws[::5, 2] = 254
        ws[::7, 3] = 1
        c0 = rng.standard_normal((m, n)).astype(np.float32).view(np.uint32)
        c0[::3, ::4] = 0x7F800000
        c0[1::3, ::5] = 0x7FC00000
        c0[2::3, ::6] = 0x00000003
        q, s = cpu.encode_mxint8(x)
        want = cpu.gemm_dense(wfmt, q, s, w, ws, n, c_init=c0)
        got = _run_dense(hrb, wfmt, x, w, ws, n, c_init=c0)
        assert (got == want).all(), wfmt


def test_dense_host_entry_point(hrb):
    from hotarubi_b200 import capi
    rng = np.random.default_rng(8)
    m, n, kb = 64, 96, 12
    x = rng.standard_normal((m, kb * 32)).astype(np.float32)
    w, ws = _weights(rng, 1, n, kb)
    bias = (rng.standard_normal(n) * 0.01).astype(np.float32)
    c = np.zeros((m, n), np.float32)
    hrb.dense_host(capi.Library.desc(1, m, n, kb * 32, a=x, w=w, wscale=ws, bias=bias, c=c))
    q, s = cpu.encode_mxint8(x.view(np.uint32))
    want = cpu.gemm_dense(1, q, s, w, ws, n, bias_bits=bias.view(np.uint32))
    assert (c.view(np.uint32) == want).all()


def test_plan_batch_of_independent_gemms(hrb):
    from hotarubi_b200 import capi
    rng = np.random.default_rng(9)
    descs, keep, wants, outs = [], [], [], []
    for i in range(7):
        wfmt = i % 3
        m, n, kb = int(rng.integers(1, 90)), int(rng.integers(8, 140)), int(rng.integers(1, 20))
        x = rng.standard_normal((m, kb * 32)).astype(np.float32)
        w, ws = _weights(rng, wfmt, n, kb)
        q, s = cpu.encode_mxint8(x.view(np.uint32))
        wants.append(cpu.gemm_dense(wfmt, q, s, w, ws, n))
        a, dw, dws = dev(x), dev(w), dev(ws)
        c = torch.full((m, n), -1.0, device="cuda")
        keep += [a, dw, dws]
        outs.append(c)
        descs.append(capi.Library.desc(wfmt, m, n, kb * 32, a=a, w=dw, wscale=dws, c=c))
    plan = hrb.plan(descs)
    for _ in range(2):
        assert plan.run() >= 2
        hrb.sync()
        for c, want in zip(outs, wants):
            assert (host(c).view(np.uint32) == want).all()
    plan.close()


def test_dense_rejects_bad_descriptors(hrb):
    from hotarubi_b200 import capi
    w = torch.zeros(64, dtype=torch.uint8, device="cuda")
    c = torch.zeros(64, dtype=torch.float32, device="cuda")
    a = torch.zeros(64, dtype=torch.float32, device="cuda")
    for kw, text in ((dict(wfmt=7), "weight format"), (dict(K=0), "empty"),
                     (dict(pieces=[1, 2]), "cover")):
        args = dict(wfmt=0, M=1, N=8, K=64)
        args.update({k: v for k, v in kw.items() if k in args})
        d = capi.Library.desc(args["wfmt"], args["M"], args["N"], args["K"], a=a, w=w,
                              wscale=w, c=c, pieces=kw.get("pieces"))
        with pytest.raises(capi.HrbError) as e:
            hrb.dense(d)
        assert e.value.status == capi.HRB_EINVAL and text in e.value.message


# --------------------------------------------------------------------------
# Layout translation

def test_translation_round_trips(hrb, golden):
    case = golden("weights.npz")
    words = case["canonical_0_24/wbuf_words"]            # 3 groups x 4 blocks
    code = case["canonical_0_24/code"]
    e = case["canonical_0_24/e"]
    codes = torch.zeros((24, 4 * 16), dtype=torch.uint8, device="cuda")
    sc = torch.zeros((24, 4), dtype=torch.uint8, device="cuda")
    hrb.wbuf_to_dense(dev(words), 3, 4, codes, sc)
    hrb.sync()
    assert (host(codes) == cpu.pack_nibbles(code)).all()
    assert (host(sc) == (e + 127).astype(np.uint8)).all()

    rng = np.random.default_rng(4)
    q = rng.integers(-128, 128, (16, 64)).astype(np.int8)
    qs = rng.integers(100, 140, (16, 2)).astype(np.uint8)
    hi, lo = cpu.split_w8(q)
    hw = cpu.pack_wbuf(hi, qs)
    lw = cpu.pack_wbuf(lo, qs)
    dq = torch.zeros((16, 64), dtype=torch.int8, device="cuda")
    ds = torch.zeros((16, 2), dtype=torch.uint8, device="cuda")
    hrb.w8_planes_to_dense(dev(hw), dev(lw), 2, 2, dq, ds)
    hrb.sync()
    assert (host(dq) == q).all() and (host(ds) == qs).all()

    qa = case_q = golden("quantize.npz")
    words = qa["q_64x96/abuf_words"]
    aq = torch.zeros((64, 96), dtype=torch.int8, device="cuda")
    asc = torch.zeros((64, 3), dtype=torch.uint8, device="cuda")
    hrb.abuf_to_dense(dev(words), 16, 3, aq, asc)
    hrb.sync()
    assert (host(aq) == case_q["q_64x96/q"]).all()
    assert (host(asc) == case_q["q_64x96/scale"]).all()

    cmat = rng.standard_normal((8, 16)).astype(np.float32)
    fw = torch.zeros((4, 32), dtype=torch.float32, device="cuda")
    hrb.dense_to_fbuf(dev(cmat), 8, 16, fw)
    hrb.sync()
    assert (host(fw).view(np.uint32) == cpu.pack_fbuf(cmat.view(np.uint32))).all()


# --------------------------------------------------------------------------
# Full benchmark sizes

def test_c2_full_size_exact(hrb):
    from hotarubi_b200 import workloads
    x = workloads.activations(0, 64, 2560)
    w, ws = workloads.mxfp4_weights(1, 960, 2560)
    q, s = cpu.encode_mxint8(x.view(np.uint32))
    want = cpu.gemm_dense(0, q, s, w, ws, 960)
    got = _run_dense(hrb, 0, x.view(np.uint32), w, ws, 960)
    assert (got == want).all()
