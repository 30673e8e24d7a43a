"""ctypes bindings to the two CPU checkers, plus numpy restatements of the
reference's operand layouts — TEST INFRASTRUCTURE ONLY (see oracle/__init__).

Layout functions cite the reference function they restate:

* ``pack_abuf``      tools/runtime/formats.cpp:114-136 (PackAbuf)
* ``pack_wbuf``      tools/compiler/tensors.cpp:66-90 (PackWbuf)
* ``pack_fbuf`` /
  ``unpack_fbuf``    tools/runtime/formats.cpp:72-112
* ``canonical_mxfp4`` tools/compiler/weights.cpp:39-70 (CanonicalMxfp4)
* ``split_w8``       tools/compiler/weights.cpp:72-88 (SplitW8)
* ``unpack_wbuf``    the inverse of PackWbuf
* ``t32_split8``     tools/iss/dma_engine.cpp:336-405 (LoadT32), in dense form
"""
from __future__ import annotations

import ctypes
import os
import subprocess

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
ORACLE_SO = os.path.join(HERE, "_build", "libhrb_oracle.so")
REF_SO = os.path.join(HERE, "_ref", "libhrb_ref.so")

_u8p = np.ctypeslib.ndpointer(np.uint8, flags="C_CONTIGUOUS")
_i8p = np.ctypeslib.ndpointer(np.int8, flags="C_CONTIGUOUS")
_u32p = np.ctypeslib.ndpointer(np.uint32, flags="C_CONTIGUOUS")
_i32p = np.ctypeslib.ndpointer(np.int32, flags="C_CONTIGUOUS")
_i64p = np.ctypeslib.ndpointer(np.int64, flags="C_CONTIGUOUS")

_oracle = None
_ref = None

WFMT_MXFP4, WFMT_W8, WFMT_MXFP8 = 0, 1, 2


def build() -> None:
    """Builds the C restatement (and the reference checker where the
    reference checkout exists)."""
    subprocess.run(["make", "-s", "-C", HERE, "all"], check=True)


def oracle() -> ctypes.CDLL:
    global _oracle
    if _oracle is None:
        if not os.path.exists(ORACLE_SO):
            subprocess.run(["make", "-s", "-C", HERE, "oracle"], check=True)
        lib = ctypes.CDLL(ORACLE_SO)
        lib.hrbo_fp32_add.restype = ctypes.c_uint32
        lib.hrbo_fp32_add.argtypes = [ctypes.c_uint32, ctypes.c_uint32]
        lib.hrbo_round_scaled.restype = ctypes.c_uint32
        lib.hrbo_round_scaled.argtypes = [ctypes.c_int64, ctypes.c_int32]
        lib.hrbo_block_value.restype = ctypes.c_uint32
        lib.hrbo_block_value.argtypes = [ctypes.c_int64, ctypes.c_uint32,
                                         ctypes.c_uint32, ctypes.c_uint32]
        lib.hrbo_weight_value.restype = ctypes.c_int32
        lib.hrbo_weight_value.argtypes = [ctypes.c_uint32, ctypes.c_uint32]
        lib.hrbo_e4m3_units.restype = ctypes.c_int32
        lib.hrbo_e4m3_units.argtypes = [ctypes.c_uint32]
        lib.hrbo_execute_gemm.restype = ctypes.c_int
        lib.hrbo_execute_gemm.argtypes = [_u32p, _u8p, _u8p, _u32p]
        lib.hrbo_encode_mxint8.restype = ctypes.c_int
        lib.hrbo_encode_mxint8.argtypes = [_u32p, ctypes.c_uint32, ctypes.c_uint32,
                                           _i8p, _u8p]
        lib.hrbo_quantize_vec.restype = None
        lib.hrbo_quantize_vec.argtypes = [_u32p, ctypes.c_uint32, ctypes.c_uint32,
                                          _i8p, _u8p]
        lib.hrbo_gemm_dense.restype = None
        lib.hrbo_gemm_dense.argtypes = [
            ctypes.c_uint32, ctypes.c_uint32, ctypes.c_uint32, ctypes.c_uint32,
            _i8p, _u8p, _u8p, _u8p, ctypes.c_void_p, ctypes.c_uint32,
            ctypes.c_void_p, _u32p, ctypes.c_int, ctypes.c_uint32, ctypes.c_uint32]
        lib.hrbo_abs_chain.restype = ctypes.c_double
        lib.hrbo_abs_chain.argtypes = [
            ctypes.c_uint32, ctypes.c_uint32, ctypes.c_uint32, ctypes.c_void_p,
            ctypes.c_void_p, _u8p, _u8p, ctypes.c_uint32]
        lib.hrbo_fp32_add_n.restype = None
        lib.hrbo_fp32_add_n.argtypes = [_u32p, _u32p, _u32p, ctypes.c_size_t]
        lib.hrbo_fp32_mul_n.restype = None
        lib.hrbo_fp32_mul_n.argtypes = [_u32p, _u32p, _u32p, ctypes.c_size_t]
        lib.hrbo_round_scaled_n.restype = None
        lib.hrbo_round_scaled_n.argtypes = [_i64p, _i32p, _u32p, ctypes.c_size_t]
        lib.hrbo_align_element.restype = ctypes.c_uint8
        lib.hrbo_align_element.argtypes = [ctypes.c_uint8, ctypes.c_uint32]
        lib.hrbo_conv_im2col.restype = ctypes.c_int
        lib.hrbo_conv_im2col.argtypes = [ctypes.c_uint32] * 7 + [_i8p, _u8p, _i8p, _u8p]
        lib.hrbo_conv_weights.restype = None
        lib.hrbo_conv_weights.argtypes = [ctypes.c_uint32] * 4 + [_u8p, _u8p, _u8p, _u8p]
        lib.hrbo_relu_n.restype = None
        lib.hrbo_relu_n.argtypes = [_u32p, ctypes.c_size_t]
        lib.hrbo_fp32_mul.restype = ctypes.c_uint32
        lib.hrbo_fp32_mul.argtypes = [ctypes.c_uint32, ctypes.c_uint32]
        lib.hrbo_gacc_dense.restype = None
        lib.hrbo_gacc_dense.argtypes = [ctypes.c_uint32] * 4 + [
            np.ctypeslib.ndpointer(np.uint64, flags="C_CONTIGUOUS"), _u32p, _u8p, ctypes.c_uint64,
            _u32p, ctypes.c_int]
        lib.hrbo_t32_split8.restype = ctypes.c_int
        lib.hrbo_t32_split8.argtypes = [_i8p, _u8p, ctypes.c_uint32, ctypes.c_uint32,
                                        ctypes.c_uint32, _i8p, _u8p]
        _oracle = lib
    return _oracle


def ref() -> ctypes.CDLL | None:
    """The reference's own sources built into oracle/_ref, or None."""
    global _ref
    if _ref is None and os.path.exists(REF_SO):
        lib = ctypes.CDLL(REF_SO)
        for name in ("hrbref_fp32_add", "hrbref_tb_fp32_add", "hrbref_exact_add"):
            getattr(lib, name).restype = ctypes.c_uint32
            getattr(lib, name).argtypes = [ctypes.c_uint32, ctypes.c_uint32]
        lib.hrbref_exact_round.restype = ctypes.c_uint32
        lib.hrbref_exact_round.argtypes = [ctypes.c_int64, ctypes.c_int64]
        lib.hrbref_weight_value.restype = ctypes.c_int32
        lib.hrbref_weight_value.argtypes = [ctypes.c_uint32, ctypes.c_uint32]
        lib.hrbref_block_value.restype = ctypes.c_uint32
        lib.hrbref_block_value.argtypes = [ctypes.c_int32, ctypes.c_uint32,
                                           ctypes.c_uint32, ctypes.c_uint32]
        lib.hrbref_execute_gemm.restype = None
        lib.hrbref_execute_gemm.argtypes = [_u32p, _u8p, _u8p, _u32p, ctypes.c_void_p]
        lib.hrbref_reference_gemm.restype = None
        lib.hrbref_reference_gemm.argtypes = [_u32p, _u8p, ctypes.c_uint32, _u8p,
                                              ctypes.c_uint32, _u32p, ctypes.c_uint32]
        lib.hrbref_encode_mxint8.restype = None
        lib.hrbref_encode_mxint8.argtypes = [_u32p, ctypes.c_uint32, ctypes.c_uint32,
                                             _i8p, _i32p]
        lib.hrbref_pack_abuf.restype = None
        lib.hrbref_pack_abuf.argtypes = [_i8p, _i32p, ctypes.c_uint32, ctypes.c_uint32, _u8p]
        lib.hrbref_quantize_block.restype = None
        lib.hrbref_quantize_block.argtypes = [_u32p, _u8p]
        lib.hrbref_canonical_mxfp4.restype = None
        lib.hrbref_canonical_mxfp4.argtypes = [_u8p, _i32p, ctypes.c_uint32,
                                               ctypes.c_uint32, ctypes.c_int32,
                                               ctypes.c_uint32, _u8p, _i32p]
        lib.hrbref_split_w8.restype = None
        lib.hrbref_split_w8.argtypes = [_i8p, ctypes.c_uint32, ctypes.c_uint32, _u8p, _u8p]
        lib.hrbref_pack_wbuf.restype = None
        lib.hrbref_pack_wbuf.argtypes = [_u8p, _i32p, ctypes.c_uint32, ctypes.c_uint32, _u8p]
        for name in ("hrbref_fp32_add_n", "hrbref_tb_fp32_add_n", "hrbref_exact_add_n",
                     "hrbref_fp32_mul_n"):
            getattr(lib, name).restype = None
            getattr(lib, name).argtypes = [_u32p, _u32p, _u32p, ctypes.c_size_t]
        lib.hrbref_exact_round_n.restype = None
        lib.hrbref_exact_round_n.argtypes = [_i64p, _i32p, _u32p, ctypes.c_size_t]
        lib.hrbref_fill_gemm_array_test.restype = None
        lib.hrbref_fill_gemm_array_test.argtypes = [ctypes.c_uint32, _u8p, _u8p, _u32p]
        lib.hrbref_tb_rng_new.restype = ctypes.c_void_p
        lib.hrbref_tb_rng_new.argtypes = [ctypes.c_uint32]
        lib.hrbref_tb_rng_free.restype = None
        lib.hrbref_tb_rng_free.argtypes = [ctypes.c_void_p]
        for name, ptr in (("hrbref_tb_random_abuf", _u8p), ("hrbref_tb_random_wbuf", _u8p),
                          ("hrbref_tb_random_fbuf", _u32p)):
            getattr(lib, name).restype = None
            getattr(lib, name).argtypes = [ctypes.c_void_p, ctypes.c_uint32, ptr]
        lib.hrbref_align_element.restype = ctypes.c_uint8
        lib.hrbref_align_element.argtypes = [ctypes.c_uint8, ctypes.c_uint32]
        lib.hrbref_dma_load_wbuf.restype = None
        lib.hrbref_dma_load_wbuf.argtypes = [ctypes.c_uint32, _u8p, ctypes.c_uint32,
                                             ctypes.c_uint32, ctypes.c_uint32,
                                             ctypes.c_uint32, ctypes.c_uint32, _u8p]
        lib.hrbref_conv_iss.restype = ctypes.c_int
        lib.hrbref_conv_iss.argtypes = [ctypes.c_uint32] * 6 + [
            _i8p, _u8p, _u8p, _i32p, _u32p, ctypes.c_void_p, ctypes.c_int, _u32p]
        lib.hrbref_rows_gemm_iss.restype = ctypes.c_int
        lib.hrbref_rows_gemm_iss.argtypes = [
            _u8p, ctypes.c_uint64, ctypes.c_uint64, ctypes.c_uint32, ctypes.c_uint32,
            ctypes.c_uint32, ctypes.c_uint64, ctypes.c_uint32, ctypes.c_uint64, ctypes.c_void_p,
            ctypes.c_uint32, ctypes.c_uint32, ctypes.c_uint32, _u8p, _u32p]
        lib.hrbref_conv_iss_w8.restype = ctypes.c_int
        lib.hrbref_conv_iss_w8.argtypes = [ctypes.c_uint32] * 6 + [
            _i8p, _u8p, _u8p, _u8p, _i32p, _u32p, ctypes.c_void_p, ctypes.c_int, _u32p]
        lib.hrbref_gemm_cycles.restype = ctypes.c_uint64
        lib.hrbref_gemm_cycles.argtypes = [_u32p, ctypes.c_void_p]
        lib.hrbref_dense_gemm_cycles.restype = ctypes.c_uint64
        lib.hrbref_dense_gemm_cycles.argtypes = [ctypes.c_uint32] * 4
        lib.hrbref_gacc_iss.restype = ctypes.c_int
        lib.hrbref_gacc_iss.argtypes = [ctypes.c_uint32] * 3 + [
            np.ctypeslib.ndpointer(np.uint64, flags="C_CONTIGUOUS"), _u32p, _u8p,
            ctypes.c_uint32, ctypes.c_uint32, _u32p]
        lib.hrbref_dense_gemm_iss.restype = ctypes.c_int
        lib.hrbref_dense_gemm_iss.argtypes = [
            ctypes.c_uint32, ctypes.c_uint32, ctypes.c_uint32, ctypes.c_uint32,
            _u8p, _u8p, _u32p, ctypes.c_uint32, ctypes.c_uint32, ctypes.c_uint32]
        _ref = lib
    return _ref


# ---------------------------------------------------------------------------
# Scalar / array arithmetic

def fp32_add(a, b) -> np.ndarray:
    a = np.ascontiguousarray(a, dtype=np.uint32).ravel()
    b = np.ascontiguousarray(b, dtype=np.uint32).ravel()
    out = np.empty_like(a)
    oracle().hrbo_fp32_add_n(a, b, out, a.size)
    return out


def fp32_mul(a, b) -> np.ndarray:
    a = np.ascontiguousarray(a, dtype=np.uint32).ravel()
    b = np.ascontiguousarray(b, dtype=np.uint32).ravel()
    out = np.empty_like(a)
    oracle().hrbo_fp32_mul_n(a, b, out, a.size)
    return out


def round_scaled(sums, exponents) -> np.ndarray:
    s = np.ascontiguousarray(sums, dtype=np.int64).ravel()
    e = np.ascontiguousarray(exponents, dtype=np.int32).ravel()
    out = np.empty(s.size, dtype=np.uint32)
    oracle().hrbo_round_scaled_n(s, e, out, s.size)
    return out


# ---------------------------------------------------------------------------
# Quantization

def encode_mxint8(x_bits: np.ndarray) -> tuple[np.ndarray, np.ndarray]:
    """EncodeMxint8 on a [rows, cols] FP32 bit matrix -> (q [rows, kp] int8,
    scale bytes [rows, kp/32])."""
    x = np.ascontiguousarray(x_bits, dtype=np.uint32)
    rows, cols = x.shape
    kp = (cols + 31) // 32 * 32
    q = np.empty((rows, kp), dtype=np.int8)
    s = np.empty((rows, kp // 32), dtype=np.uint8)
    if oracle().hrbo_encode_mxint8(x.ravel(), rows, cols, q.ravel(), s.ravel()) != 0:
        raise ValueError("MXINT8 input is infinite or NaN")
    return q, s


def quantize_vec(x_bits: np.ndarray) -> tuple[np.ndarray, np.ndarray]:
    x = np.ascontiguousarray(x_bits, dtype=np.uint32)
    rows, cols = x.shape
    kp = (cols + 31) // 32 * 32
    q = np.empty((rows, kp), dtype=np.int8)
    s = np.empty((rows, kp // 32), dtype=np.uint8)
    oracle().hrbo_quantize_vec(x.ravel(), rows, cols, q.ravel(), s.ravel())
    return q, s


# ---------------------------------------------------------------------------
# GEMM

def execute_gemm(fields, abuf: np.ndarray, wbuf: np.ndarray, fbuf: np.ndarray) -> int:
    """ExecuteGemm on full memories; fbuf (4096 x 32 uint32) updated in place."""
    f = np.ascontiguousarray(fields, dtype=np.uint32)
    return oracle().hrbo_execute_gemm(f, abuf.reshape(-1), wbuf.reshape(-1), fbuf.reshape(-1))


def gemm_dense(wfmt: int, aq: np.ndarray, ascale: np.ndarray, w: np.ndarray,
               wscale: np.ndarray, n: int, bias_bits=None, c_init=None,
               pieces=None, rows=None, colscale_bits=None) -> np.ndarray:
    """The dense chain of hrbo_gemm_dense; returns [M, N] FP32 bits.

    colscale_bits ([N] FP32 bits, hrb_gemm_desc.wcol_scale) multiplies each
    finished chain with the ISS's FP32 multiply (tools/iss/fp32.hpp:77-92)
    before the bias is added with its FP32 add, as a VEC MUL then ADDP would."""
    if colscale_bits is not None:
        assert c_init is None, "per-column scales do not combine with accumulate"
        c = gemm_dense(wfmt, aq, ascale, w, wscale, n, pieces=pieces, rows=rows)
        m = c.shape[0]
        cs = np.broadcast_to(np.asarray(colscale_bits, dtype=np.uint32).reshape(1, n), (m, n))
        c = fp32_mul(c, cs).reshape(m, n)
        if bias_bits is not None:
            b = np.broadcast_to(np.asarray(bias_bits, dtype=np.uint32).reshape(1, n), (m, n))
            c = fp32_add(c, b).reshape(m, n)
        if rows is not None:  # rows outside the range stay zero, as in the chain
            r0, r1 = rows
            c[:r0] = 0
            c[r1:] = 0
        return c
    m, kp = aq.shape
    kb = kp // 32
    c = (np.ascontiguousarray(c_init, dtype=np.uint32).copy() if c_init is not None
         else np.zeros((m, n), dtype=np.uint32))
    bias = None if bias_bits is None else np.ascontiguousarray(bias_bits, dtype=np.uint32)
    pc = None if pieces is None else np.ascontiguousarray(pieces, dtype=np.uint32)
    r0, r1 = (0, m) if rows is None else rows
    oracle().hrbo_gemm_dense(
        wfmt, m, n, kb, np.ascontiguousarray(aq).ravel(), np.ascontiguousarray(ascale).ravel(),
        np.ascontiguousarray(w).ravel(), np.ascontiguousarray(wscale).ravel(),
        None if pc is None else pc.ctypes.data, 0 if pc is None else pc.size,
        None if bias is None else bias.ctypes.data, c.ravel(),
        1 if c_init is not None else 0, r0, r1)
    return c


NULL_ENTRY = 0xFFFFFFFF


def row_unit_bytes(tok: int) -> int:
    """Bytes of one token's unit in the MXINT8 row format (MakeRowFormat,
    tools/iss/dma_engine.cpp:156-183): tok x 32 codes, then tok scale bytes
    in one 16-byte beat (two when tok > 16)."""
    return tok * 32 + (32 if tok > 16 else 16)


def rows_to_dense(ddr: np.ndarray, ddr_base: int, first_unit: int, tok: int, planes: int,
                  plane_stride: int, row_tokens: int, row_stride: int, index, m: int):
    """The activations a GEMM reads from DDR in the row format, as dense
    MXINT8 (aq [m][planes * tok * 32] int8, ascale [m][planes * tok]): what
    LoadRows (dma_engine.cpp:231-262) puts in ABUF, plane by plane.  Token t's
    unit of plane 0 is at byte first_unit * 16 + (t // row_tokens) *
    row_stride + (t % row_tokens) * unit (ROW) or index[t] * 16 (ROW_INDEXED,
    NULL_ENTRY: zero codes, scale bytes 127); plane p adds p * plane_stride.
    Addresses are DDR byte addresses; ddr[0] is at ddr_base."""
    ub = row_unit_bytes(tok)
    kb = planes * tok
    aq = np.zeros((m, kb * 32), np.int8)
    asc = np.full((m, kb), 127, np.uint8)
    ddr = np.asarray(ddr, np.uint8)
    for t in range(m):
        if index is not None:
            if int(index[t]) == NULL_ENTRY:
                continue
            off0 = int(index[t]) * 16 - ddr_base
        else:
            off0 = first_unit * 16 - ddr_base + (t // row_tokens) * row_stride + \
                (t % row_tokens) * ub
        for p in range(planes):
            off = off0 + p * plane_stride
            aq[t, p * tok * 32:(p + 1) * tok * 32] = ddr[off:off + tok * 32].view(np.int8)
            asc[t, p * tok:(p + 1) * tok] = ddr[off + tok * 32:off + tok * 32 + tok]
    return aq, asc


def make_rows_window(rng, m: int, tok: int, planes: int, indexed: bool, row_tokens: int = 0,
                     nulls: float = 0.0, ddr_base: int = 0x20000000):
    """A DDR window holding m tokens' MXINT8 activations in the row format,
    for tests: units of encoded N(0,1) rows (EncodeMxint8) with junk in the
    padding and between units.  ROW: rows of row_tokens tokens, a gap after
    each row, planes one after another; ROW_INDEXED: every (token, plane 0)
    unit at a shuffled slot, the planes plane_stride apart, a share `nulls`
    of null entries.  Returns (window uint8, layout dict of the hrb_rows
    fields, aq, ascale) with aq/ascale the dense view (rows_to_dense)."""
    ub = row_unit_bytes(tok)
    kb = planes * tok
    x = rng.standard_normal((m, kb * 32)).astype(np.float32)
    x[:, : 32] *= 64.0          # a spread of block scales
    q, s = encode_mxint8(x.view(np.uint32))
    if indexed:
        slots = m + 5
        plane_stride = slots * ub + 48
        size = planes * plane_stride + 64
        order = rng.permutation(slots)[:m]
        first = 32
        index = (ddr_base + first + order * ub) // 16
        index = index.astype(np.uint32)
        index[rng.random(m) < nulls] = NULL_ENTRY
        layout = dict(tok=tok, planes=planes, plane_stride=plane_stride, index=index)
        unit_off = [None if index[t] == NULL_ENTRY else first + int(order[t]) * ub
                    for t in range(m)]
    else:
        rows_n = (m + row_tokens - 1) // row_tokens
        row_stride = row_tokens * ub + 16 * int(rng.integers(0, 4))
        plane_stride = rows_n * row_stride + 32
        first = 48
        size = first + planes * plane_stride + 64
        layout = dict(tok=tok, planes=planes, plane_stride=plane_stride,
                      ddr_addr=(ddr_base + first) // 16, row_tokens=row_tokens,
                      row_stride=row_stride)
        unit_off = [first + (t // row_tokens) * row_stride + (t % row_tokens) * ub
                    for t in range(m)]
    win = rng.integers(0, 256, size).astype(np.uint8)    # junk everywhere else
    for t in range(m):
        if unit_off[t] is None:
            continue
        for p in range(planes):
            o = unit_off[t] + p * plane_stride
            win[o:o + tok * 32] = q[t, p * tok * 32:(p + 1) * tok * 32].view(np.uint8)
            win[o + tok * 32:o + tok * 32 + tok] = s[t, p * tok:(p + 1) * tok]
    layout.update(ddr_base=ddr_base, window_bytes=size)
    aq, asc = rows_to_dense(win, ddr_base, layout.get("ddr_addr", 0), tok, planes,
                            plane_stride, layout.get("row_tokens", 0),
                            layout.get("row_stride", 0), layout.get("index"), m)
    return win, layout, aq, asc


def abs_chain(wfmt: int, aq_row: np.ndarray, ascale_row: np.ndarray, w: np.ndarray,
              wscale: np.ndarray, n: int) -> float:
    kb = aq_row.size // 32
    aq_row = np.ascontiguousarray(aq_row, dtype=np.int8)
    ascale_row = np.ascontiguousarray(ascale_row, dtype=np.uint8)
    return oracle().hrbo_abs_chain(wfmt, 0, kb, aq_row.ctypes.data, ascale_row.ctypes.data,
                                   np.ascontiguousarray(w).ravel(),
                                   np.ascontiguousarray(wscale).ravel(), n)


# ---------------------------------------------------------------------------
# Operand layouts (numpy restatements)

def pack_abuf(q: np.ndarray, scale: np.ndarray) -> np.ndarray:
    """PackAbuf: [rows, cols] int8 + [rows, blocks] scale bytes -> words of
    144 bytes ordered (quad, block): bytes j*32+k = token j element k,
    128..131 = the four scales, 132..143 = 0.  Returns [quads*blocks, 144]."""
    rows, cols = q.shape
    assert rows % 4 == 0 and cols % 32 == 0
    blocks = cols // 32
    quads = rows // 4
    out = np.zeros((quads, blocks, 144), dtype=np.uint8)
    qv = q.view(np.uint8).reshape(quads, 4, blocks, 32).transpose(0, 2, 1, 3)
    out[:, :, :128] = qv.reshape(quads, blocks, 128)
    out[:, :, 128:132] = scale.reshape(quads, 4, blocks).transpose(0, 2, 1)
    return out.reshape(quads * blocks, 144)


def pack_wbuf(code: np.ndarray, scale: np.ndarray) -> np.ndarray:
    """PackWbuf: [rows, cols] 4-bit codes + [rows, blocks] scale bytes -> words
    of 144 bytes ordered (group of 8 rows, block): byte c*16+m holds elements
    2m (low nibble) and 2m+1 (high nibble) of column c, 128..135 = scales.
    Returns [groups*blocks, 144]."""
    rows, cols = code.shape
    assert rows % 8 == 0 and cols % 32 == 0
    blocks = cols // 32
    groups = rows // 8
    c = (code.astype(np.uint8) & 0xF).reshape(groups, 8, blocks, 16, 2)
    packed = (c[..., 0] | (c[..., 1] << 4)).transpose(0, 2, 1, 3)  # g, b, col, 16
    out = np.zeros((groups, blocks, 144), dtype=np.uint8)
    out[:, :, :128] = packed.reshape(groups, blocks, 128)
    out[:, :, 128:136] = scale.reshape(groups, 8, blocks).transpose(0, 2, 1)
    return out.reshape(groups * blocks, 144)


def unpack_wbuf(words: np.ndarray, groups: int, blocks: int) -> tuple[np.ndarray, np.ndarray]:
    """The inverse of pack_wbuf: [groups*blocks, 144] words ordered (group,
    block) -> ([8*groups, 32*blocks] 4-bit codes, [8*groups, blocks] scales)."""
    w = np.asarray(words, dtype=np.uint8).reshape(groups, blocks, 144)
    packed = w[:, :, :128].reshape(groups, blocks, 8, 16)
    code = np.stack([packed & 0xF, packed >> 4], axis=-1)        # g, b, col, 16, 2
    code = code.transpose(0, 2, 1, 3, 4).reshape(8 * groups, 32 * blocks)
    scale = w[:, :, 128:136].transpose(0, 2, 1).reshape(8 * groups, blocks)
    return code.astype(np.uint8), scale.copy()


def mxint8_rows_to_dense(ddr: np.ndarray, rows: int, row_words: int, stride: int,
                         offset: int = 0) -> tuple[np.ndarray, np.ndarray]:
    """MXINT8 cache rows as the DMA engine reads them (dma_engine.cpp:54-58,
    303-334): DDR row r holds tokens 4r..4r+3 as ``row_words`` 144-byte words
    ``stride`` bytes apart (word w: bytes j*32+d = token j, dim 32w+d; 128+j =
    token j's scale).  Returns (codes [4*rows, 32*row_words] int8, scales
    [4*rows, row_words])."""
    d = np.asarray(ddr, dtype=np.uint8)
    words = np.stack([d[offset + r * stride: offset + r * stride + row_words * 144]
                      .reshape(row_words, 144) for r in range(rows)])   # r, w, 144
    q = words[:, :, :128].reshape(rows, row_words, 4, 32).transpose(0, 2, 1, 3)
    s = words[:, :, 128:132].transpose(0, 2, 1)
    return (q.reshape(4 * rows, 32 * row_words).view(np.int8).copy(),
            s.reshape(4 * rows, row_words).copy())


def w8_planes_from_wbuf(wbuf: np.ndarray, onchip: int, groups: int,
                        blocks: int) -> tuple[np.ndarray, np.ndarray]:
    """The two planes a SPLIT8 or T32_SPLIT8 load leaves in WBUF (HI words from
    ``onchip``, LO words ``groups*blocks`` later, both in PackWbuf order,
    dma_engine.cpp:326-331,394-401) joined back into MXINT8 weights
    [8*groups, 32*blocks] and their scales.  Raises if the planes' scales
    differ."""
    n = groups * blocks
    idx = (onchip + np.arange(2 * n)) % wbuf.shape[0]
    hi, hs = unpack_wbuf(wbuf[idx[:n]], groups, blocks)
    lo, ls = unpack_wbuf(wbuf[idx[n:]], groups, blocks)
    assert (hs == ls).all(), "HI and LO planes carry different scales"
    return ((hi << 4) | lo).astype(np.uint8).view(np.int8), hs


def pack_fbuf(c_bits: np.ndarray) -> np.ndarray:
    """PackFbuf: [rows, cols] -> [rows/4 * cols/8, 32] words, element t*8+c."""
    rows, cols = c_bits.shape
    return (c_bits.reshape(rows // 4, 4, cols // 8, 8).transpose(0, 2, 1, 3)
            .reshape(-1, 32).copy())


def unpack_fbuf(words: np.ndarray, rows: int, cols: int) -> np.ndarray:
    return (words.reshape(rows // 4, cols // 8, 4, 8).transpose(0, 2, 1, 3)
            .reshape(rows, cols).copy())


_HALF_UNITS = np.array([0, 1, 2, 3, 4, 6, 8, 12], dtype=np.int32)
_FLOOR_LOG2 = np.array([0, -1, 0, 0, 1, 1, 2, 2], dtype=np.int32)


def canonical_mxfp4(code: np.ndarray, e: np.ndarray, shift: int = 0,
                    rows: int | None = None) -> tuple[np.ndarray, np.ndarray]:
    """CanonicalMxfp4: per nonzero block, rescale the codes so the largest
    magnitude index is in 4..7 (value >= 2) and move the difference into the
    exponent, plus ``shift``.  All-zero blocks get e = 0 and plain +0 codes;
    rows beyond the input are zero padding."""
    r, cols = code.shape
    rows = r if rows is None else rows
    blocks = cols // 32
    c = code.reshape(r, blocks, 32).astype(np.int32)
    mag = c & 7
    top = mag.max(axis=2)
    up = 2 - _FLOOR_LOG2[top]                      # left shift of half units
    half = _HALF_UNITS[mag] << up[..., None]
    lut = np.full(13, -1, dtype=np.int32)
    lut[_HALF_UNITS] = np.arange(8)
    assert (half <= 12).all()
    index = lut[half]
    assert (index >= 0).all()
    out_code = np.where((index != 0) & ((c & 8) != 0), index | 8, index)
    out_e = e.reshape(r, blocks).astype(np.int32) + _FLOOR_LOG2[top] - 2 + shift
    zero = top == 0
    out_code[zero] = 0
    out_e[zero] = 0
    code_out = np.zeros((rows, cols), dtype=np.uint8)
    e_out = np.zeros((rows, blocks), dtype=np.int32)
    code_out[:r] = out_code.reshape(r, cols)
    e_out[:r] = out_e
    return code_out, e_out


def align_element(value: int, shift: int) -> int:
    """AlignElement (dma_engine.cpp:532-544) through the C restatement."""
    return int(oracle().hrbo_align_element(value & 0xFF, shift))


def t32_split8(vq: np.ndarray, vs: np.ndarray, hd: int | None = None) -> tuple[np.ndarray, np.ndarray]:
    """T32_SPLIT8 in dense form (hrbo_t32_split8): V codes [tokens, ldv] and
    scales [tokens, ldv/32] -> W8 operand codes [hd, tokens], scales
    [hd, tokens/32]."""
    vq = np.ascontiguousarray(vq, dtype=np.int8)
    vs = np.ascontiguousarray(vs, dtype=np.uint8)
    tokens, ldv = vq.shape
    hd = ldv if hd is None else hd
    wq = np.empty((hd, tokens), dtype=np.int8)
    ws = np.empty((hd, tokens // 32), dtype=np.uint8)
    if oracle().hrbo_t32_split8(vq.ravel(), vs.ravel(), tokens, hd, ldv, wq.ravel(),
                                ws.ravel()) != 0:
        raise ValueError(f"T32_SPLIT8 shape {tokens} x {hd} (ldv {ldv}) is not whole 32 x 32 blocks")
    return wq, ws


# ---------------------------------------------------------------------------
# Convolution (ConvEmitter, tools/compiler/sparsedrive_encoder.cpp)

def conv_geometry(H: int, W: int, cin: int, kh: int, stride: int):
    """(Ho, Wo, planes, K' blocks per output) of a conv the emitter accepts."""
    plane = min(cin, 256)
    return H // stride, W // stride, cin // plane, kh * kh * cin // 32


def conv_im2col(aq: np.ndarray, ascale: np.ndarray, images: int, H: int, W: int, cin: int,
                kh: int, stride: int, order: int = 0) -> tuple[np.ndarray, np.ndarray]:
    """hrbo_conv_im2col: the gathered activations [images*Ho*Wo, kh*kh*cin]
    in chain order (plane, tap, channel) and their scales."""
    ho, wo, _, kbo = conv_geometry(H, W, cin, kh, stride)
    m = images * ho * wo
    q = np.empty((m, kbo * 32), np.int8)
    sc = np.empty((m, kbo), np.uint8)
    if oracle().hrbo_conv_im2col(images, H, W, cin, kh, stride, order,
                                 np.ascontiguousarray(aq, np.int8).ravel(),
                                 np.ascontiguousarray(ascale, np.uint8).ravel(),
                                 q.ravel(), sc.ravel()) != 0:
        raise ValueError("conv shape not supported")
    return q, sc


def conv_weights(wfmt: int, w: np.ndarray, wscale: np.ndarray, cout: int, cin: int,
                 kh: int) -> tuple[np.ndarray, np.ndarray]:
    """hrbo_conv_weights: the [cout, kh*kh*cin] weight matrix in chain order."""
    bpb = 16 if wfmt == WFMT_MXFP4 else 32
    w = np.ascontiguousarray(w, np.uint8)
    out = np.empty_like(w)
    osc = np.empty_like(np.ascontiguousarray(wscale, np.uint8))
    oracle().hrbo_conv_weights(cout, cin, kh, bpb, w.ravel(),
                               np.ascontiguousarray(wscale, np.uint8).ravel(), out.ravel(),
                               osc.ravel())
    return out, osc


def relu(bits: np.ndarray) -> np.ndarray:
    out = np.ascontiguousarray(bits, np.uint32).copy()
    oracle().hrbo_relu_n(out.ravel(), out.size)
    return out


def conv_dense(wfmt: int, aq, ascale, images, H, W, cin, cout, kh, stride, w, wscale,
               order=0, bias_bits=None, c_init=None, relu_out=False) -> np.ndarray:
    """The conv chain: gathered activations x reordered weights, one K
    piece per (plane, tap) job (W8: HI then LO per job), bias, RELU."""
    q, sc = conv_im2col(aq, ascale, images, H, W, cin, kh, stride, order)
    wq, ws = conv_weights(wfmt, w, wscale, cout, cin, kh)
    _, _, planes, _ = conv_geometry(H, W, cin, kh, stride)
    pieces = [min(cin, 256) // 32] * (planes * kh * kh)
    c = gemm_dense(wfmt, q, sc, wq, ws, cout, bias_bits=bias_bits, c_init=c_init,
                   pieces=pieces)
    return relu(c) if relu_out else c


def gacc_dense(entries: np.ndarray, w: np.ndarray, rows: np.ndarray, blocks: int,
               out_init=None) -> np.ndarray:
    """hrbo_gacc_dense: entries uint64 [tokens, slots, corners], w FP32 bits
    [tokens, slots, blocks], rows uint8 [nrows, row_stride]; returns FP32
    bits [tokens, blocks * 32]."""
    entries = np.ascontiguousarray(entries, np.uint64)
    tokens, slots, corners = entries.shape
    out = (np.zeros((tokens, blocks * 32), np.uint32) if out_init is None
           else np.ascontiguousarray(out_init, np.uint32).copy())
    rows = np.ascontiguousarray(rows, np.uint8)
    oracle().hrbo_gacc_dense(tokens, slots, corners, blocks, entries.ravel(),
                             np.ascontiguousarray(w, np.uint32).ravel(), rows.ravel(),
                             rows.shape[1], out.ravel(), 0 if out_init is None else 1)
    return out


def split_w8(q: np.ndarray) -> tuple[np.ndarray, np.ndarray]:
    """SplitW8: int8 -> (high nibble, low nibble) codes."""
    b = q.view(np.uint8)
    return (b >> 4).astype(np.uint8), (b & 0xF).astype(np.uint8)


def pack_nibbles(code: np.ndarray) -> np.ndarray:
    """[rows, cols] 4-bit codes -> [rows, cols/2] bytes, low nibble = even
    column (the nibble order of a WBUF word)."""
    c = code.astype(np.uint8) & 0xF
    return (c[:, 0::2] | (c[:, 1::2] << 4)).astype(np.uint8)
