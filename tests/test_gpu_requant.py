"""The MXINT8 copy of a GEMM's output (hrb_gemm_desc.cq / cscale): the VEC
'q' pass that follows GEMM + ADDP on the NPU (QuantizeBlock,
tools/iss/lane.cpp:406-423), or the host rule (EncodeMxint8,
tools/runtime/formats.cpp:138-162), fused into the tensor-core epilogue
(fast mode) or run after the exact GEMM.

The copy must equal the oracle's encoding of the FP32 output of the same
call bit for bit, padding columns (N up to a multiple of 32) included.
"""
import numpy as np
import pytest

from oracle import cpu

pytestmark = pytest.mark.gpu

torch = pytest.importorskip("torch")


def dev(x):
    return torch.from_numpy(np.ascontiguousarray(x)).cuda()


def operands(rng, wfmt, m, n, k):
    from hotarubi_b200 import workloads
    x = (rng.standard_normal((m, k)) * 3).astype(np.float32)
    kb = (k + 31) // 32
    if wfmt == 0:
        w, ws = workloads.mxfp4_weights(int(rng.integers(1 << 30)), n, k)
    elif wfmt == 1:
        w = rng.integers(-128, 128, (n, kb * 32)).astype(np.int8).view(np.uint8)
        ws = rng.integers(115, 125, (n, kb)).astype(np.uint8)
    else:
        w, ws = workloads.mxfp8_weights(int(rng.integers(1 << 30)), n, kb * 32)
    b = (rng.standard_normal(n) * 0.5).astype(np.float32)
    return x, w, ws, b


def encode(c, rule):
    bits = np.ascontiguousarray(c).view(np.uint32)
    return cpu.quantize_vec(bits) if rule == 1 else cpu.encode_mxint8(bits)


@pytest.mark.parametrize("mode", [0, 1])
@pytest.mark.parametrize("rule", [0, 1])
@pytest.mark.parametrize("wfmt", [0, 1, 2])
def test_copy_equals_encoding_of_output(hrb, wfmt, rule, mode):
    from hotarubi_b200 import capi
    rng = np.random.default_rng(100 + 10 * wfmt + 2 * rule + mode)
    m, n, k = 70, 200, 320             # N = 200: the last block holds 24 padding columns
    x, w, ws, b = operands(rng, wfmt, m, n, k)
    kbq = (n + 31) // 32
    c = torch.zeros((m, n), dtype=torch.float32, device="cuda")
    cq = torch.full((m, kbq * 32), 77, dtype=torch.int8, device="cuda")
    cs = torch.zeros((m, kbq), dtype=torch.uint8, device="cuda")
    keep = [dev(x), dev(w), dev(ws), dev(b)]
    d = capi.Library.desc(wfmt, m, n, k, a=keep[0], w=keep[1], wscale=keep[2], bias=keep[3],
                          c=c, mode=mode, cq=cq, cscale=cs, cquant=rule)
    hrb.dense(d)
    hrb.sync()
    got_c = c.cpu().numpy()
    q, s = encode(got_c, rule)
    assert np.array_equal(cq.cpu().numpy(), q)
    assert np.array_equal(cs.cpu().numpy(), s)
    if mode == 1:
        # The copy alone (no FP32 output) is the same copy.
        cq2 = torch.zeros_like(cq)
        cs2 = torch.zeros_like(cs)
        d2 = capi.Library.desc(wfmt, m, n, k, a=keep[0], w=keep[1], wscale=keep[2],
                               bias=keep[3], c=None, mode=mode, cq=cq2, cscale=cs2, cquant=rule)
        hrb.dense(d2)
        hrb.sync()
        assert torch.equal(cq2, cq) and torch.equal(cs2, cs)


def test_copy_through_a_plan_and_host_entry_points(hrb):
    from hotarubi_b200 import capi
    rng = np.random.default_rng(7)
    descs, keep, outs = [], [], []
    for i, (wfmt, mode) in enumerate([(0, 1), (1, 0), (2, 1), (0, 0), (1, 1)]):
        m, n, k = int(rng.integers(1, 150)), int(rng.integers(8, 300)), 32 * int(rng.integers(1, 20))
        x, w, ws, b = operands(rng, wfmt, m, n, k)
        kbq = (n + 31) // 32
        t = [dev(x), dev(w), dev(ws), dev(b)]
        keep += t
        c = torch.zeros((m, n), dtype=torch.float32, device="cuda")
        cq = torch.zeros((m, kbq * 32), dtype=torch.int8, device="cuda")
        cs = torch.zeros((m, kbq), dtype=torch.uint8, device="cuda")
        outs.append((c, cq, cs, i % 2))
        descs.append(capi.Library.desc(wfmt, m, n, k, a=t[0], w=t[1], wscale=t[2], bias=t[3],
                                       c=c, mode=mode, cq=cq, cscale=cs, cquant=i % 2))
    plan = hrb.plan(descs)
    plan.run()
    hrb.sync()
    for c, cq, cs, rule in outs:
        q, s = encode(c.cpu().numpy(), rule)
        assert np.array_equal(cq.cpu().numpy(), q) and np.array_equal(cs.cpu().numpy(), s)
    plan.close()
    # Host pointers.
    x, w, ws, b = operands(rng, 0, 33, 100, 256)
    c = np.zeros((33, 100), np.float32)
    cq = np.zeros((33, 128), np.int8)
    cs = np.zeros((33, 4), np.uint8)
    d = capi.Library.desc(0, 33, 100, 256, a=x, w=w, wscale=ws, bias=b, c=c, mode=1,
                          cq=cq, cscale=cs, cquant=1)
    hrb.dense_host(d)
    q, s = encode(c, 1)
    assert np.array_equal(cq, q) and np.array_equal(cs, s)


def test_copy_needs_an_output_unless_fused(hrb):
    from hotarubi_b200 import capi
    rng = np.random.default_rng(3)
    x, w, ws, b = operands(rng, 0, 16, 64, 64)
    cq = torch.zeros((16, 64), dtype=torch.int8, device="cuda")
    cs = torch.zeros((16, 2), dtype=torch.uint8, device="cuda")
    keep = [dev(x), dev(w), dev(ws)]
    for mode, acc in ((0, False), (1, True)):
        d = capi.Library.desc(0, 16, 64, 64, a=keep[0], w=keep[1], wscale=keep[2], c=None,
                              mode=mode, cq=cq, cscale=cs, accumulate=acc)
        with pytest.raises(capi.HrbError) as e:
            hrb.dense(d)
        assert e.value.status == capi.HRB_EINVAL


@pytest.mark.parametrize("mode", [0, 1])
@pytest.mark.parametrize("wfmt", [0, 1])
def test_copy_with_a_row_stride(hrb, wfmt, mode):
    """hrb_gemm_desc.ldcq: the copy of a GEMM over a column slice lands in a
    wider matrix's layout (cq and cscale pointing at the slice's first
    column), bit-equal to the packed copy, with the wider rows' other columns
    untouched; device and host entry points."""
    from hotarubi_b200 import capi
    rng = np.random.default_rng(300 + 10 * wfmt + mode)
    m, n, k = 70, 200, 320
    wide, n0 = 512, 96                  # the slice's columns [96, 296) of 512
    x, w, ws, b = operands(rng, wfmt, m, n, k)
    kbq = (n + 31) // 32
    keep = [dev(x), dev(w), dev(ws), dev(b)]
    common = dict(a=keep[0], w=keep[1], wscale=keep[2], bias=keep[3], mode=mode, cquant=1)
    c = torch.zeros((m, n), dtype=torch.float32, device="cuda")
    q0 = torch.zeros((m, kbq * 32), dtype=torch.int8, device="cuda")
    s0 = torch.zeros((m, kbq), dtype=torch.uint8, device="cuda")
    qw = torch.full((m, wide), 77, dtype=torch.int8, device="cuda")
    sw = torch.full((m, wide // 32), 99, dtype=torch.uint8, device="cuda")
    torch.cuda.synchronize()
    hrb.dense(capi.Library.desc(wfmt, m, n, k, c=c, cq=q0, cscale=s0, **common))
    hrb.dense(capi.Library.desc(wfmt, m, n, k, c=c, cq=qw[:, n0:], cscale=sw[:, n0 // 32:],
                                ldcq=wide, **common))
    hrb.sync()
    got_q, got_s = qw.cpu().numpy(), sw.cpu().numpy()
    assert (got_q[:, n0:n0 + kbq * 32] == q0.cpu().numpy()).all()
    assert (got_s[:, n0 // 32:n0 // 32 + kbq] == s0.cpu().numpy()).all()
    assert (got_q[:, :n0] == 77).all() and (got_q[:, n0 + kbq * 32:] == 77).all()
    assert (got_s[:, :n0 // 32] == 99).all() and (got_s[:, n0 // 32 + kbq:] == 99).all()
    # The host entry point: a pitched copy of the slice's columns only.
    hq = np.full((m, wide), 55, np.int8)
    hs = np.full((m, wide // 32), 44, np.uint8)
    hc = np.zeros((m, n), np.float32)
    hrb.dense_host(capi.Library.desc(wfmt, m, n, k, a=x, w=w, wscale=ws, bias=b, c=hc,
                                     mode=mode, cquant=1, cq=hq[:, n0:], cscale=hs[:, n0 // 32:],
                                     ldcq=wide))
    assert (hq[:, n0:n0 + kbq * 32] == q0.cpu().numpy()).all()
    assert (hs[:, n0 // 32:n0 // 32 + kbq] == s0.cpu().numpy()).all()
    assert (hq[:, :n0] == 55).all() and (hq[:, n0 + kbq * 32:] == 55).all()
    assert (hs[:, :n0 // 32] == 44).all() and (hs[:, n0 // 32 + kbq:] == 44).all()


def test_row_stride_checks(hrb):
    from hotarubi_b200 import capi
    rng = np.random.default_rng(7)
    m, n, k = 8, 200, 64
    x, w, ws, b = operands(rng, 0, m, n, k)
    keep = [dev(x), dev(w), dev(ws)]
    c = torch.zeros((m, n), dtype=torch.float32, device="cuda")
    q = torch.zeros((m, 512), dtype=torch.int8, device="cuda")
    s = torch.zeros((m, 16), dtype=torch.uint8, device="cuda")
    for ldcq, cq in ((100, q), (192, q), (256, None)):
        d = capi.Library.desc(0, m, n, k, a=keep[0], w=keep[1], wscale=keep[2], c=c,
                              cq=cq, cscale=None if cq is None else s, ldcq=ldcq)
        with pytest.raises(capi.HrbError):
            hrb.dense(d)
