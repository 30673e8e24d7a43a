"""hrb_gemm_dense_noalloc: the dense GEMM entry point that allocates nothing.

It is for callers that cannot call cudaMalloc themselves or have the library
do it (a simulator plugin inside a process whose device memory is owned by
someone else, code running while a CUDA graph is captured, a real-time
loop).  They pass device buffers for every input and output; the only
scratch is a fixed device array inside the library.

The test calls it through the C ABI twice in a row, with different shapes
and data, and checks each result against hrb_gemm_dense (the allocating
entry point) bit for bit, as the exact path is bit-exact.  It also checks
that a request larger than the fixed scratch is refused.  This file sorts
last so that a failure here leaves every other test already run; it needs
nothing from the other tests and passes in a fresh process on its own.
"""
import ctypes

import numpy as np
import pytest

pytestmark = pytest.mark.gpu

torch = pytest.importorskip("torch")


def _operands(rng, m, n, k):
    from hotarubi_b200 import workloads
    x = rng.standard_normal((m, k)).astype(np.float32)
    kp = (k + 31) // 32 * 32          # weights are stored with K padded to 32
    w, ws = workloads.mxfp4_weights(int(rng.integers(0, 1 << 30)), n, kp)
    bias = (rng.standard_normal(n) * 0.01).astype(np.float32)
    return [torch.from_numpy(v).cuda() for v in (x, w, ws, bias)]


def test_noalloc_matches_the_allocating_entry_point_on_two_calls():
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    from hotarubi_b200 import capi
    lib = capi.load()
    ctx = capi.Library(0)
    torch.cuda.set_device(0)
    rng = np.random.default_rng(2024)
    for m, n, k in ((64, 960, 2560), (32, 200, 720)):
        x, w, ws, bias = _operands(rng, m, n, k)
        want = torch.zeros((m, n), dtype=torch.float32, device="cuda")
        got = torch.full((m, n), 7.0, dtype=torch.float32, device="cuda")
        ctx.dense(capi.Library.desc(capi.WFMT_MXFP4, m, n, k, a=x, w=w, wscale=ws,
                                    bias=bias, c=want))
        ctx.sync()
        d = capi.Library.desc(capi.WFMT_MXFP4, m, n, k, a=x, w=w, wscale=ws, bias=bias, c=got)
        assert lib.hrb_gemm_dense_noalloc(ctypes.byref(d), None) == capi.HRB_OK
        torch.cuda.synchronize()
        assert torch.equal(got.view(torch.int32), want.view(torch.int32)), (m, n, k)
    ctx.close()


def test_noalloc_refuses_more_than_its_scratch():
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    from hotarubi_b200 import capi
    lib = capi.load()
    m, n, k = 1024, 8, 4096          # 4 MiB of codes + scales: over the limit
    x = torch.zeros((m, k), dtype=torch.float32, device="cuda")
    w = torch.zeros((n, k // 2), dtype=torch.uint8, device="cuda")
    ws = torch.zeros((n, k // 32), dtype=torch.uint8, device="cuda")
    c = torch.zeros((m, n), dtype=torch.float32, device="cuda")
    d = capi.Library.desc(capi.WFMT_MXFP4, m, n, k, a=x, w=w, wscale=ws, c=c)
    assert lib.hrb_gemm_dense_noalloc(ctypes.byref(d), None) == capi.HRB_EINVAL


@pytest.mark.gpu
def test_no_alloc_mxint8_copy_of_the_output(hrb):
    """hrb_gemm_dense_noalloc with cq: the encoder over C after the GEMM,
    equal to the oracle's VEC encoding of C."""
    from hotarubi_b200 import capi
    from oracle import cpu
    rng = np.random.default_rng(12)
    m, n, k = 40, 90, 256
    x = torch.from_numpy(rng.standard_normal((m, k)).astype(np.float32)).cuda()
    w = torch.from_numpy(rng.integers(0, 256, (n, k // 2)).astype(np.uint8)).cuda()
    ws = torch.from_numpy(rng.integers(118, 124, (n, k // 32)).astype(np.uint8)).cuda()
    c = torch.zeros((m, n), dtype=torch.float32, device="cuda")
    cq = torch.zeros((m, 96), dtype=torch.int8, device="cuda")
    cs = torch.zeros((m, 3), dtype=torch.uint8, device="cuda")
    d = capi.Library.desc(0, m, n, k, a=x, w=w, wscale=ws, c=c, cq=cq, cscale=cs, cquant=1)
    st = capi.load().hrb_gemm_dense_noalloc(ctypes.byref(d), None)
    assert st == capi.HRB_OK
    torch.cuda.synchronize()
    q, s = cpu.quantize_vec(c.cpu().numpy().view(np.uint32))
    assert np.array_equal(cq.cpu().numpy(), q) and np.array_equal(cs.cpu().numpy(), s)


def test_noalloc_column_scales_match_the_oracle():
    """wcol_scale through the no-alloc entry: int8 weights (W8 block scale
    bytes 133) with a per-column FP32 scale, bit for bit with the oracle."""
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    from hotarubi_b200 import capi
    from oracle import cpu
    torch.cuda.set_device(0)
    rng = np.random.default_rng(99)
    m, n, kb = 48, 80, 7
    x = rng.standard_normal((m, kb * 32)).astype(np.float32)
    w = rng.integers(-128, 128, (n, kb * 32)).astype(np.int8).view(np.uint8)
    ws = np.full((n, kb), 133, np.uint8)
    bias = (rng.standard_normal(n) * 0.01).astype(np.float32)
    cs = (rng.uniform(0.5, 2.0, n) * 2.0**-10).astype(np.float32)
    q, s = cpu.encode_mxint8(x.view(np.uint32))
    want = cpu.gemm_dense(1, q, s, w, ws, n, bias_bits=bias.view(np.uint32),
                          colscale_bits=cs.view(np.uint32))
    t = [torch.from_numpy(v).cuda() for v in (x, w, ws, bias, cs)]
    got = torch.zeros((m, n), dtype=torch.float32, device="cuda")
    d = capi.Library.desc(capi.WFMT_W8, m, n, kb * 32, a=t[0], w=t[1], wscale=t[2], bias=t[3],
                          c=got, wcol_scale=t[4])
    assert capi.load().hrb_gemm_dense_noalloc(ctypes.byref(d), None) == capi.HRB_OK
    torch.cuda.synchronize()
    assert (got.cpu().numpy().view(np.uint32) == want).all()


def test_noalloc_mxint8_input_on_a_caller_stream():
    """Pre-encoded MXINT8 activations (aq/ascale: the scratch is not used) on
    a caller-supplied stream, bit for bit with hrb_gemm_dense."""
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    from hotarubi_b200 import capi, workloads
    from oracle import cpu
    lib = capi.load()
    ctx = capi.Library(0)
    torch.cuda.set_device(0)
    rng = np.random.default_rng(77)
    m, n, k = 96, 136, 640
    x = rng.standard_normal((m, k)).astype(np.float32)
    q, s = cpu.encode_mxint8(x.view(np.uint32))
    w, ws = workloads.mxfp4_weights(5, n, k)
    aq, asc, dw, dws = (torch.from_numpy(v).cuda() for v in (q, s, w, ws))
    want = torch.zeros((m, n), dtype=torch.float32, device="cuda")
    ctx.dense(capi.Library.desc(capi.WFMT_MXFP4, m, n, k, aq=aq, ascale=asc, w=dw, wscale=dws,
                                c=want))
    ctx.sync()
    stream = torch.cuda.Stream()
    got = torch.full((m, n), -1.0, dtype=torch.float32, device="cuda")
    torch.cuda.synchronize()
    d = capi.Library.desc(capi.WFMT_MXFP4, m, n, k, aq=aq, ascale=asc, w=dw, wscale=dws, c=got)
    assert lib.hrb_gemm_dense_noalloc(ctypes.byref(d), ctypes.c_void_p(stream.cuda_stream)) \
        == capi.HRB_OK
    stream.synchronize()
    assert torch.equal(got.view(torch.int32), want.view(torch.int32))
    ctx.close()


def test_noalloc_encoding_that_just_fits_the_scratch():
    """M = 992 at K = 4096 needs 4,190,208 of the scratch's 4,194,304 bytes
    (codes and scales, each rounded up to 256): accepted and equal to
    hrb_gemm_dense; M = 993 needs 4,194,560 and is refused with a message."""
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    from hotarubi_b200 import capi, workloads
    lib = capi.load()
    ctx = capi.Library(0)
    torch.cuda.set_device(0)
    n, k = 24, 4096
    w, ws = workloads.mxfp4_weights(9, n, k)
    dw, dws = torch.from_numpy(w).cuda(), torch.from_numpy(ws).cuda()
    x = torch.from_numpy(np.random.default_rng(3).standard_normal((993, k))
                         .astype(np.float32)).cuda()
    m = 992
    want = torch.zeros((m, n), dtype=torch.float32, device="cuda")
    ctx.dense(capi.Library.desc(capi.WFMT_MXFP4, m, n, k, a=x[:m], w=dw, wscale=dws, c=want))
    ctx.sync()
    got = torch.zeros((m, n), dtype=torch.float32, device="cuda")
    d = capi.Library.desc(capi.WFMT_MXFP4, m, n, k, a=x[:m], w=dw, wscale=dws, c=got)
    assert lib.hrb_gemm_dense_noalloc(ctypes.byref(d), None) == capi.HRB_OK
    torch.cuda.synchronize()
    assert torch.equal(got.view(torch.int32), want.view(torch.int32))
    over = torch.zeros((993, n), dtype=torch.float32, device="cuda")
    d = capi.Library.desc(capi.WFMT_MXFP4, 993, n, k, a=x, w=dw, wscale=dws, c=over)
    assert lib.hrb_gemm_dense_noalloc(ctypes.byref(d), None) == capi.HRB_EINVAL
    msg = lib.hrb_last_error(None).decode()
    assert "4194560" in msg and "4194304" in msg, msg
    ctx.close()
