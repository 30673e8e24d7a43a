"""GEMMs whose activations the library reads in the DMA row format
(hrb_gemm_rows): ROW and ROW_INDEXED units of a DDR window on the device,
null entries included, several planes chained as K pieces.

* HRB_MODE_EXACT bit for bit against the reference's own LoadRows +
  ExecuteGemm over the same window (tests/golden/rows.npz, made by
  make_golden.py from oracle/ref_bridge.cpp hrbref_rows_gemm_iss);
* HRB_MODE_FAST (the units encoded straight into the tensor-core operand
  blocks) within the stated bound (K/16 + 4) 2^-23 sum|a w| of the float64
  product of the gathered operands, MXFP8 weights included, and at a size
  that takes the large-tile kernels;
* the errors: a ROW window too small (at the call), an index entry outside
  the window and a scale byte of 255 in fast mode (at hrb_sync).
"""
import numpy as np
import pytest

from oracle import cpu

pytestmark = pytest.mark.gpu

torch = pytest.importorskip("torch")

from test_oracle_rows import CASES  # noqa: E402

E2M1 = np.array([0, .5, 1, 1.5, 2, 3, 4, 6], np.float64)


def dev(x):
    return torch.from_numpy(np.ascontiguousarray(x)).cuda()


def load_case(g, name):
    lay = {k: int(g[f"{name}/{k}"]) for k in ("ddr_base", "ddr_addr", "tok", "planes",
                                               "plane_stride", "row_tokens", "row_stride")}
    lay["index"] = g.get(f"{name}/index")
    return g[f"{name}/window"], lay


def rows_desc(capi, win_dev, win_bytes, lay, index_dev):
    return capi.rows(win_dev, lay["ddr_base"], win_bytes, lay["tok"], lay["planes"],
                     lay["plane_stride"], ddr_addr=lay.get("ddr_addr", 0),
                     row_tokens=lay.get("row_tokens", 0), row_stride=lay.get("row_stride", 0),
                     index=index_dev)


def dequant_weights(wfmt, w, ws, n, kp):
    sc = np.repeat(np.ldexp(1.0, ws.astype(np.int64) - 127), 32, axis=1)
    if wfmt == cpu.WFMT_MXFP4:
        code = np.zeros((n, kp), np.uint8)
        code[:, 0::2] = w & 0xF
        code[:, 1::2] = w >> 4
        v = E2M1[code & 7] * np.where(code & 8, -1.0, 1.0)
    elif wfmt == cpu.WFMT_W8:
        v = w.view(np.int8).astype(np.float64) * 2.0**-6
    else:
        v = np.array([cpu.oracle().hrbo_e4m3_units(int(c)) for c in range(256)],
                     np.float64)[w] * 2.0**-9
    return v * sc


def within_bound(got, aq, asc, wd, k):
    a = aq.astype(np.float64) * np.repeat(np.ldexp(1.0, asc.astype(np.int64) - 133), 32, axis=1)
    ref = a @ wd.T
    absref = np.abs(a) @ np.abs(wd).T
    err = np.abs(got.astype(np.float64) - ref)
    tol = (k / 16 + 4) * 2.0**-23
    return bool((err <= tol * absref + 1e-30).all()), float((err / (absref + 1e-30)).max())


def run(hrb, capi, wfmt, m, n, k, win, lay, w, ws, mode):
    win_d = dev(win)
    idx_d = None if lay.get("index") is None else dev(lay["index"].view(np.int32))
    c = torch.zeros((m, n), dtype=torch.float32, device="cuda")
    d = capi.Library.desc(wfmt, m, n, k, w=dev(w), wscale=dev(ws), c=c, mode=mode)
    torch.cuda.synchronize()  # torch's fills come before the library's stream reads them
    d._keep = (win_d, idx_d)
    hrb.gemm_rows(d, rows_desc(capi, win_d, win.size, lay, idx_d))
    hrb.sync()
    return c


@pytest.mark.parametrize("case", CASES, ids=[c[0] for c in CASES])
def test_rows_exact_equals_reference_loads_and_chain(hrb, golden, case):
    from hotarubi_b200 import capi
    g = golden("rows.npz")
    name, m, tok, planes, _, _, _, wfmt, n = case
    win, lay = load_case(g, name)
    c = run(hrb, capi, wfmt, m, n, planes * tok * 32, win, lay, g[f"{name}/w"],
            g[f"{name}/wscale"], capi.MODE_EXACT)
    got = c.cpu().numpy().view(np.uint32)
    want = g[f"{name}/c"]
    assert (got == want).all(), f"{int((got != want).sum())} of {got.size} outputs differ"


@pytest.mark.parametrize("case", CASES, ids=[c[0] for c in CASES])
def test_rows_fast_within_bound(hrb, golden, case):
    from hotarubi_b200 import capi
    g = golden("rows.npz")
    name, m, tok, planes, _, _, _, wfmt, n = case
    win, lay = load_case(g, name)
    k = planes * tok * 32
    c = run(hrb, capi, wfmt, m, n, k, win, lay, g[f"{name}/w"], g[f"{name}/wscale"],
            capi.MODE_FAST)
    aq, asc = cpu.rows_to_dense(win, lay["ddr_base"], lay["ddr_addr"], tok, planes,
                                lay["plane_stride"], lay["row_tokens"], lay["row_stride"],
                                lay["index"], m)
    wd = dequant_weights(wfmt, g[f"{name}/w"], g[f"{name}/wscale"], n, k)
    ok, worst = within_bound(c.cpu().numpy(), aq, asc, wd, k)
    assert ok, f"worst relative error {worst:.3e}"


@pytest.mark.parametrize("wfmt", [0, 1, 2], ids=["mxfp4", "w8", "mxfp8"])
@pytest.mark.parametrize("m,tok,planes,indexed", [(2048, 30, 1, False), (1200, 16, 5, True),
                                                  (40, 8, 4, False)])
def test_rows_fast_sizes_and_formats(hrb, wfmt, m, tok, planes, indexed):
    """MXFP8 weights (no reference counterpart, so no golden) and sizes that
    take the 128-token tiles; every row checked."""
    from hotarubi_b200 import capi
    rng = np.random.default_rng(m + wfmt)
    rt = 0 if indexed else 32
    win, lay, aq, asc = cpu.make_rows_window(rng, m, tok, planes, indexed, rt, 0.05)
    kb = planes * tok
    n = 264
    if wfmt == 0:
        code = rng.integers(0, 16, (n, kb * 32)).astype(np.uint8)
        code, e = cpu.canonical_mxfp4(code, rng.integers(-10, -3, (n, kb)))
        w, ws = cpu.pack_nibbles(code), (e + 127).astype(np.uint8)
    elif wfmt == 1:
        w = rng.integers(-127, 128, (n, kb * 32)).astype(np.int8).view(np.uint8)
        ws = rng.integers(116, 124, (n, kb)).astype(np.uint8)
    else:
        w = rng.integers(0, 254, (n, kb * 32)).astype(np.uint8)
        w[w >= 0x7F] += 1
        ws = rng.integers(117, 124, (n, kb)).astype(np.uint8)
    c = run(hrb, capi, wfmt, m, n, kb * 32, win, lay, w, ws, capi.MODE_FAST)
    ok, worst = within_bound(c.cpu().numpy(), aq, asc, dequant_weights(wfmt, w, ws, n, kb * 32),
                             kb * 32)
    assert ok, f"worst relative error {worst:.3e}"
    # The exact mode of the same GEMM against the oracle's chain (MXFP4, W8).
    if wfmt != 2:
        ce = run(hrb, capi, wfmt, m, n, kb * 32, win, lay, w, ws, capi.MODE_EXACT)
        want = cpu.gemm_dense(wfmt, aq, asc, w, ws, n, pieces=[tok] * planes)
        assert (ce.cpu().numpy().view(np.uint32) == want).all()


def test_rows_errors(hrb):
    from hotarubi_b200 import capi
    rng = np.random.default_rng(5)
    m, tok, n = 32, 8, 16
    win, lay, aq, asc = cpu.make_rows_window(rng, m, tok, 1, False, 16)
    w = np.zeros((n, tok * 16), np.uint8)
    ws = np.full((n, tok), 127, np.uint8)
    # A window one byte short of the last unit: refused at the call.
    ub = cpu.row_unit_bytes(tok)
    far = (lay["ddr_addr"] * 16 - lay["ddr_base"] + ((m - 1) // 16) * lay["row_stride"]
           + ((m - 1) % 16) * ub + ub)
    with pytest.raises(capi.HrbError) as e:
        run(hrb, capi, 0, m, n, tok * 32, win[:far - 1], lay, w, ws, capi.MODE_EXACT)
    assert e.value.status == capi.HRB_EINVAL
    # An index entry past the window: skipped on the device, reported by sync.
    win2, lay2, _, _ = cpu.make_rows_window(rng, m, tok, 1, True)
    lay2 = dict(lay2)
    lay2["index"] = lay2["index"].copy()
    lay2["index"][3] = (lay2["ddr_base"] + win2.size + 4096) // 16
    with pytest.raises(capi.HrbError) as e:
        run(hrb, capi, 0, m, n, tok * 32, win2, lay2, w, ws, capi.MODE_FAST)
    assert e.value.status == capi.HRB_EDATA
    # A scale byte of 255 has no E2M1 digit-plane encoding in fast mode.
    win3 = win.copy()
    off = (lay["ddr_addr"] * 16 - lay["ddr_base"]) + tok * 32
    win3[off] = 255
    with pytest.raises(capi.HrbError) as e:
        run(hrb, capi, 0, m, n, tok * 32, win3, lay, w, ws, capi.MODE_FAST)
    assert e.value.status == capi.HRB_EDATA
