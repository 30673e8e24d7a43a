"""Weights straight from a compiled program (hrb_image_*, hrb_gemm_image).

The image is built the way hotarubi's compiler builds one: weight matrices
packed into WBUF words by the reference's own PackWbuf (W8 split by its own
SplitW8 into "<name>_hi" and "<name>_lo" regions, PlaceW8), placed at page
offsets among other regions, and a meta.json written by the reference's own
Json writer in MetaJson's layout (tools/compiler/output.cpp:57-89).

CPU: hrb_image_region finds every region where the reference's loader
(Json::Parse + regions, tools/runtime/runtime.cpp:132-150) finds it, also in
a pretty-printed meta.json, and refuses a missing one.
GPU: hrb_gemm_image on the uploaded image equals hrb_gemm_dense on the dense
weights bit for bit (exact mode also equals the CPU oracle), twice in a row
(the second call reuses the cached dense weights); hrb_image_weights gives
the dense weights back; misuse is refused.
"""
import ctypes
import json

import numpy as np
import pytest

from oracle import cpu

PAGE = 4096


def reference_meta(ref, regions: dict[str, tuple[int, int]], image_bytes: int) -> str:
    names = [n.encode() for n in regions]
    arr = (ctypes.c_char_p * len(names))(*names)
    offs = (ctypes.c_uint64 * len(names))(*[regions[n][0] for n in regions])
    sizes = (ctypes.c_uint64 * len(names))(*[regions[n][1] for n in regions])
    buf = ctypes.create_string_buffer(1 << 16)
    ref.hrbref_meta_json.restype = ctypes.c_int64
    ref.hrbref_meta_json.argtypes = [ctypes.c_void_p, ctypes.c_void_p, ctypes.c_void_p,
                                     ctypes.c_uint32, ctypes.c_uint64, ctypes.c_char_p,
                                     ctypes.c_size_t]
    n = ref.hrbref_meta_json(arr, offs, sizes, len(names), image_bytes, buf, len(buf))
    assert n > 0
    return buf.value.decode()


def reference_find(ref, meta: str, name: str):
    ref.hrbref_find_region.restype = ctypes.c_int
    ref.hrbref_find_region.argtypes = [ctypes.c_char_p, ctypes.c_char_p,
                                       ctypes.POINTER(ctypes.c_uint64),
                                       ctypes.POINTER(ctypes.c_uint64)]
    off, size = ctypes.c_uint64(), ctypes.c_uint64()
    rc = ref.hrbref_find_region(meta.encode(), name.encode(), ctypes.byref(off),
                                ctypes.byref(size))
    return (off.value, size.value) if rc == 0 else None


def test_region_lookup_matches_the_reference_loader(ref_lib):
    from hotarubi_b200 import capi
    regions = {"instr": (0, 4 * PAGE), "layers.0.q_hi": (4 * PAGE, 276480),
               "layers.0.q_lo": (72 * PAGE, 276480), "fc": (140 * PAGE, 1382400),
               "trace": (2 ** 33, 65536), "x": (3 * 2 ** 30, 16)}
    meta = reference_meta(ref_lib, regions, 2 ** 34)
    pretty = json.dumps(json.loads(meta), indent=2)
    for text in (meta, pretty):
        for name, want in regions.items():
            assert reference_find(ref_lib, text, name) == want
            assert capi.image_region(text, name) == want
    assert reference_find(ref_lib, meta, "missing") is None
    with pytest.raises(capi.HrbError):
        capi.image_region(meta, "missing")
    with pytest.raises(capi.HrbError):
        capi.image_region('{"base": 0}', "fc")


def build_image(ref, rng):
    """An image with an MXFP4 matrix (region fc) and a W8 matrix (w8_hi,
    w8_lo) among other regions; returns (bytes, meta, dense weights)."""
    n4, k4 = 136, 320
    code = rng.integers(0, 16, (n4, k4)).astype(np.uint8)
    e4 = rng.integers(-10, -3, (n4, k4 // 32)).astype(np.int32)
    code, e4 = cpu.canonical_mxfp4(code, e4)
    e4 = np.ascontiguousarray(e4, np.int32)
    fc = np.zeros(n4 // 8 * k4 // 32 * 144, np.uint8)
    ref.hrbref_pack_wbuf(np.ascontiguousarray(code), e4, n4, k4, fc)
    n8, k8 = 96, 256
    q = rng.integers(-128, 128, (n8, k8)).astype(np.int8)
    e8 = rng.integers(-12, -2, (n8, k8 // 32)).astype(np.int32)
    hi = np.zeros((n8, k8), np.uint8)
    lo = np.zeros((n8, k8), np.uint8)
    ref.hrbref_split_w8(q, n8, k8, hi, lo)
    whi = np.zeros(n8 // 8 * k8 // 32 * 144, np.uint8)
    wlo = np.zeros_like(whi)
    ref.hrbref_pack_wbuf(hi, e8, n8, k8, whi)
    ref.hrbref_pack_wbuf(lo, e8, n8, k8, wlo)
    layout = {"instr": (0, PAGE), "fc": (PAGE, fc.size)}
    at = PAGE + (fc.size + PAGE - 1) // PAGE * PAGE
    layout["bias"] = (at, 999)
    at += PAGE
    layout["w8_hi"] = (at, whi.size)
    at += (whi.size + PAGE - 1) // PAGE * PAGE
    layout["w8_lo"] = (at, wlo.size)
    at += (wlo.size + PAGE - 1) // PAGE * PAGE
    image = rng.integers(0, 256, at, dtype=np.uint8)  # other regions: any bytes
    for name, words in (("fc", fc), ("w8_hi", whi), ("w8_lo", wlo)):
        off, size = layout[name]
        image[off:off + size] = words
    meta = reference_meta(ref, layout, at)
    dense = {"fc": (cpu.pack_nibbles(code), (e4 + 127).astype(np.uint8), n4, k4),
             "w8": (q.view(np.uint8), (e8 + 127).astype(np.uint8), n8, k8)}
    return image, meta, dense


@pytest.mark.gpu
@pytest.mark.parametrize("mode", [0, 1], ids=["exact", "fast"])
def test_gemm_image_equals_the_dense_gemm(hrb, ref_lib, mode):
    torch = pytest.importorskip("torch")
    from hotarubi_b200 import capi
    rng = np.random.default_rng(17 + mode)
    image, meta, dense = build_image(ref_lib, rng)
    img = capi.Image(hrb, image)
    try:
        for key, wfmt in (("fc", capi.WFMT_MXFP4), ("w8", capi.WFMT_W8)):
            w, ws, n, k = dense[key]
            m = 70
            x = rng.standard_normal((m, k)).astype(np.float32)
            bias = (rng.standard_normal(n) * 0.01).astype(np.float32)
            xd, bd = torch.from_numpy(x).cuda(), torch.from_numpy(bias).cuda()
            want = torch.zeros((m, n), dtype=torch.float32, device="cuda")
            # The library's stream does not wait for torch's: its fills first.
            torch.cuda.synchronize()
            hrb.dense(capi.Library.desc(wfmt, m, n, k, a=xd, w=torch.from_numpy(w).cuda(),
                                        wscale=torch.from_numpy(ws).cuda(), bias=bd, c=want,
                                        mode=mode))
            hrb.sync()
            if key == "fc":
                off, lo = capi.image_region(meta, "fc")[0], 0
            else:
                off, lo = capi.image_region(meta, "w8_hi")[0], capi.image_region(meta, "w8_lo")[0]
            for _ in range(2):  # the second call reuses the cached dense weights
                got = torch.full((m, n), 3.0, dtype=torch.float32, device="cuda")
                torch.cuda.synchronize()
                img.gemm(capi.Library.desc(wfmt, m, n, k, a=xd, bias=bd, c=got, mode=mode),
                         off, lo)
                hrb.sync()
                assert torch.equal(got.view(torch.int32), want.view(torch.int32)), key
            if mode == capi.MODE_EXACT:
                q, s = cpu.encode_mxint8(x.view(np.uint32))
                oracle = cpu.gemm_dense(wfmt, q, s, w, ws, n, bias_bits=bias.view(np.uint32))
                assert (want.cpu().numpy().view(np.uint32) == oracle).all(), key
            # The dense weights themselves.
            wd = torch.zeros(w.shape, dtype=torch.uint8, device="cuda")
            wsd = torch.zeros(ws.shape, dtype=torch.uint8, device="cuda")
            torch.cuda.synchronize()
            img.weights(wfmt, off, n, k, wd, wsd, offset_lo=lo)
            hrb.sync()
            assert np.array_equal(wd.cpu().numpy(), w) and np.array_equal(wsd.cpu().numpy(), ws)
        # Misuse: weights given as well, a region past the end, MXFP8.
        n, k = 8, 32
        c = torch.zeros((4, n), dtype=torch.float32, device="cuda")
        xd = torch.zeros((4, k), dtype=torch.float32, device="cuda")
        with pytest.raises(capi.HrbError) as e:
            img.gemm(capi.Library.desc(0, 4, n, k, a=xd, w=xd, wscale=xd, c=c), 0)
        assert e.value.status == capi.HRB_EINVAL
        with pytest.raises(capi.HrbError) as e:
            img.gemm(capi.Library.desc(0, 4, n, k, a=xd, c=c), len(image) - 100)
        assert e.value.status == capi.HRB_EINVAL
        with pytest.raises(capi.HrbError) as e:
            img.gemm(capi.Library.desc(2, 4, n, k, a=xd, c=c), 0)
        assert e.value.status == capi.HRB_ENOTSUP
    finally:
        img.close()
