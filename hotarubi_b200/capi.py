"""ctypes binding of libhrb_gemm.so (include/hrb_gemm.h).

The library is the product: this module only loads it and converts
arguments.  Device buffers are passed as integer addresses (for example
``torch.Tensor.data_ptr()``), host buffers as numpy arrays.  Every call that
returns a status other than HRB_OK raises :class:`HrbError` carrying the
status and the library's message.
"""
from __future__ import annotations

import ctypes
import os
import re

import numpy as np

PKG = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(PKG, "lib", "libhrb_gemm.so")
HEADER = os.path.join(os.path.dirname(PKG), "include", "hrb_gemm.h")

HRB_OK, HRB_EINVAL, HRB_ECUDA, HRB_ENOMEM, HRB_ENOTSUP, HRB_EDATA = range(6)
WFMT_MXFP4, WFMT_W8, WFMT_MXFP8 = 0, 1, 2
MODE_EXACT, MODE_FAST = 0, 1
QUANT_HOST, QUANT_VEC = 0, 1
ABUF_WORDS, ABUF_WORD_BYTES = 8192, 132
WBUF_WORDS, WBUF_WORD_BYTES = 2048, 144
FBUF_WORDS = 4096


class HrbError(RuntimeError):
    def __init__(self, status: int, message: str):
        super().__init__(f"hrb status {status}: {message}")
        self.status = status
        self.message = message


class GemmCmd(ctypes.Structure):
    """hrb_gemm_cmd: GemmCommand of tools/iss/gemm_array.hpp:16-27."""
    _fields_ = [(n, ctypes.c_uint32) for n in (
        "a_base", "a_stride", "kb", "m", "w_base", "w_stride", "n8", "c_base", "wmode", "acc")]


class IpcHandle(ctypes.Structure):
    _fields_ = [("bytes", ctypes.c_uint8 * 64)]


class CommId(ctypes.Structure):
    """hrb_comm_id: the 128-byte bootstrap id of a communicator."""
    _fields_ = [("bytes", ctypes.c_uint8 * 128)]


class GemmDesc(ctypes.Structure):
    """hrb_gemm_desc."""
    _fields_ = [
        ("wfmt", ctypes.c_uint32), ("mode", ctypes.c_uint32),
        ("M", ctypes.c_uint32), ("N", ctypes.c_uint32), ("K", ctypes.c_uint32),
        ("a", ctypes.c_void_p), ("lda", ctypes.c_uint32), ("quant", ctypes.c_uint32),
        ("aq", ctypes.c_void_p), ("ascale", ctypes.c_void_p),
        ("w", ctypes.c_void_p), ("wscale", ctypes.c_void_p),
        ("bias", ctypes.c_void_p), ("c", ctypes.c_void_p), ("ldc", ctypes.c_uint32),
        ("accumulate", ctypes.c_uint32),
        ("pieces", ctypes.c_void_p), ("npieces", ctypes.c_uint32),
        ("cq", ctypes.c_void_p), ("cscale", ctypes.c_void_p), ("cquant", ctypes.c_uint32),
        ("wcol_scale", ctypes.c_void_p), ("w8_kernel", ctypes.c_uint32),
        ("ldcq", ctypes.c_uint32),
    ]


class ConvDesc(ctypes.Structure):
    """hrb_conv_desc."""
    _fields_ = [
        ("wfmt", ctypes.c_uint32), ("mode", ctypes.c_uint32),
        ("images", ctypes.c_uint32), ("H", ctypes.c_uint32), ("W", ctypes.c_uint32),
        ("cin", ctypes.c_uint32), ("cout", ctypes.c_uint32),
        ("kh", ctypes.c_uint32), ("stride", ctypes.c_uint32), ("order", ctypes.c_uint32),
        ("a", ctypes.c_void_p), ("quant", ctypes.c_uint32),
        ("aq", ctypes.c_void_p), ("ascale", ctypes.c_void_p),
        ("w", ctypes.c_void_p), ("wscale", ctypes.c_void_p),
        ("bias", ctypes.c_void_p), ("c", ctypes.c_void_p),
        ("accumulate", ctypes.c_uint32), ("relu", ctypes.c_uint32),
        ("cq", ctypes.c_void_p), ("cscale", ctypes.c_void_p), ("cquant", ctypes.c_uint32),
    ]


CONV_XMAJOR, CONV_YMAJOR = 0, 1
W8_DIGIT_PLANES, W8_BF16 = 0, 1


class GaccDesc(ctypes.Structure):
    """hrb_gacc_desc."""
    _fields_ = [
        ("tokens", ctypes.c_uint32), ("slots", ctypes.c_uint32), ("corners", ctypes.c_uint32),
        ("blocks", ctypes.c_uint32), ("entries", ctypes.c_void_p), ("w", ctypes.c_void_p),
        ("rows", ctypes.c_void_p), ("row_stride", ctypes.c_uint64), ("nrows", ctypes.c_uint32),
        ("out", ctypes.c_void_p), ("accumulate", ctypes.c_uint32),
    ]


class Rows(ctypes.Structure):
    """hrb_rows: activations in the DMA row format (ROW, or ROW_INDEXED with
    `index`)."""
    _fields_ = [
        ("window", ctypes.c_void_p), ("ddr_base", ctypes.c_uint64),
        ("window_bytes", ctypes.c_uint64), ("tok", ctypes.c_uint32), ("planes", ctypes.c_uint32),
        ("plane_stride", ctypes.c_uint64), ("ddr_addr", ctypes.c_uint32),
        ("row_tokens", ctypes.c_uint32), ("row_stride", ctypes.c_uint64),
        ("index", ctypes.c_void_p),
    ]


NULL_ENTRY = 0xFFFFFFFF


def row_unit_bytes(tok: int) -> int:
    """Bytes of one MXINT8 row-format unit (tok x 32 codes, tok scale bytes
    padded to 16, or to 32 when tok > 16)."""
    return tok * 32 + (32 if tok > 16 else 16)


def rows(window, ddr_base: int, window_bytes: int, tok: int, planes: int, plane_stride: int,
         *, ddr_addr: int = 0, row_tokens: int = 0, row_stride: int = 0, index=None) -> Rows:
    r = Rows()
    r.window = _ptr(window)
    r.ddr_base, r.window_bytes = ddr_base, window_bytes
    r.tok, r.planes, r.plane_stride = tok, planes, plane_stride
    r.ddr_addr, r.row_tokens, r.row_stride = ddr_addr, row_tokens, row_stride
    r.index = _ptr(index)
    return r


def header_functions() -> list[str]:
    """Every function include/hrb_gemm.h declares."""
    text = open(HEADER).read()
    return re.findall(r"^HRB_API [^(]*?\b(hrb_\w+)\(", text, flags=re.M)


_lib = None


def load() -> ctypes.CDLL:
    """Loads libhrb_gemm.so; raises if it has not been built."""
    global _lib
    if _lib is None:
        if not os.path.exists(LIB_PATH):
            raise RuntimeError(f"{LIB_PATH} is missing: build it with "
                               "`python -m hotarubi_b200.build`")
        lib = ctypes.CDLL(LIB_PATH)
        P = ctypes.c_void_p
        u32 = ctypes.c_uint32
        sigs = {
            "hrb_create": (ctypes.c_int, [ctypes.c_int, ctypes.POINTER(P)]),
            "hrb_destroy": (ctypes.c_int, [P]),
            "hrb_sync": (ctypes.c_int, [P]),
            "hrb_last_error": (ctypes.c_char_p, [P]),
            "hrb_status_string": (ctypes.c_char_p, [ctypes.c_int]),
            "hrb_get_stream": (P, [P]),
            "hrb_set_stream": (ctypes.c_int, [P, P]),
            "hrb_launch_count": (ctypes.c_uint64, [P]),
            "hrb_gemm_decode": (ctypes.c_int, [P, ctypes.POINTER(GemmCmd)]),
            "hrb_gemm_check": (ctypes.c_int, [P, ctypes.POINTER(GemmCmd)]),
            "hrb_gemm_exec": (ctypes.c_int, [P, ctypes.POINTER(GemmCmd), P, P, P]),
            "hrb_gemm_exec_device": (ctypes.c_int, [P, ctypes.POINTER(GemmCmd), P, P, P, P]),
            "hrb_gemm_accesses": (ctypes.c_int, [ctypes.POINTER(GemmCmd), P, P, P, P]),
            "hrb_gemm_dense": (ctypes.c_int, [P, ctypes.POINTER(GemmDesc), P]),
            "hrb_gemm_dense_host": (ctypes.c_int, [P, ctypes.POINTER(GemmDesc)]),
            "hrb_gemm_rows": (ctypes.c_int, [P, ctypes.POINTER(GemmDesc), ctypes.POINTER(Rows),
                                             P]),
            "hrb_gemm_dense_noalloc": (ctypes.c_int, [ctypes.POINTER(GemmDesc), P]),
            "hrb_quantize_mxint8": (ctypes.c_int, [P, P, u32, u32, u32, u32, P, P, P]),
            "hrb_plan_create": (ctypes.c_int, [P, ctypes.POINTER(GemmDesc), u32,
                                               ctypes.POINTER(P)]),
            "hrb_plan_run": (ctypes.c_int, [P, P, ctypes.POINTER(u32)]),
            "hrb_plan_run_host": (ctypes.c_int, [P, P, ctypes.POINTER(P), ctypes.POINTER(P),
                                                 ctypes.POINTER(P)]),
            "hrb_plan_destroy": (ctypes.c_int, [P]),
            "hrb_plan_profile": (ctypes.c_int, [P, P, u32, ctypes.POINTER(ctypes.c_float), u32,
                                                ctypes.POINTER(u32)]),
            "hrb_wbuf_to_dense": (ctypes.c_int, [P, P, u32, u32, P, P, P]),
            "hrb_w8_planes_to_dense": (ctypes.c_int, [P, P, P, u32, u32, P, P, P]),
            "hrb_abuf_to_dense": (ctypes.c_int, [P, P, u32, u32, P, P, P]),
            "hrb_t32_split8_dense": (ctypes.c_int, [P, P, P, u32, u32, u32, P, P, P]),
            "hrb_dense_to_fbuf": (ctypes.c_int, [P, P, u32, u32, P, P]),
            "hrb_gemm_npu_cycles": (ctypes.c_uint64, [ctypes.POINTER(GemmCmd)]),
            "hrb_dense_npu_cycles": (ctypes.c_uint64, [u32, u32, u32, u32]),
            "hrb_conv_dense": (ctypes.c_int, [P, ctypes.POINTER(ConvDesc), P]),
            "hrb_gacc_dense": (ctypes.c_int, [P, ctypes.POINTER(GaccDesc), P]),
            "hrb_conv_plan_create": (ctypes.c_int, [P, ctypes.POINTER(ConvDesc),
                                                    ctypes.POINTER(P)]),
            "hrb_conv_plan_run": (ctypes.c_int, [P, P, ctypes.POINTER(u32)]),
            "hrb_conv_plan_destroy": (ctypes.c_int, [P]),
            "hrb_conv_plan_profile": (ctypes.c_int, [P, P, u32, ctypes.POINTER(ctypes.c_float),
                                                     u32, ctypes.POINTER(u32)]),
            "hrb_shared_alloc": (ctypes.c_int, [P, ctypes.c_size_t, ctypes.POINTER(P),
                                                ctypes.POINTER(IpcHandle)]),
            "hrb_shared_free": (ctypes.c_int, [P, P]),
            "hrb_peer_open": (ctypes.c_int, [P, ctypes.POINTER(IpcHandle), ctypes.POINTER(P)]),
            "hrb_peer_close": (ctypes.c_int, [P, P]),
            "hrb_shard_columns": (None, [u32, u32, u32, ctypes.POINTER(u32), ctypes.POINTER(u32)]),
            "hrb_plan_set_peers": (ctypes.c_int, [P, P, ctypes.POINTER(P), u32]),
            "hrb_conv_plan_set_peers": (ctypes.c_int, [P, P, ctypes.POINTER(P), u32]),
            "hrb_comm_id_new": (ctypes.c_int, [ctypes.POINTER(CommId)]),
            "hrb_comm_create": (ctypes.c_int, [P, ctypes.POINTER(CommId), u32, u32,
                                               ctypes.POINTER(P)]),
            "hrb_comm_destroy": (ctypes.c_int, [P]),
            "hrb_comm_exchange": (ctypes.c_int, [P, P, P, ctypes.c_size_t]),
            "hrb_comm_barrier": (ctypes.c_int, [P]),
            "hrb_comm_fence": (ctypes.c_int, [P, P]),
            "hrb_comm_allgather": (ctypes.c_int, [P, P, ctypes.POINTER(ctypes.c_uint64), P]),
            "hrb_shard_rows": (None, [u32, u32, u32, ctypes.POINTER(u32), ctypes.POINTER(u32)]),
            "hrb_image_region": (ctypes.c_int, [ctypes.c_char_p, ctypes.c_char_p,
                                                ctypes.POINTER(ctypes.c_uint64),
                                                ctypes.POINTER(ctypes.c_uint64)]),
            "hrb_image_upload": (ctypes.c_int, [P, P, ctypes.c_size_t, ctypes.POINTER(P)]),
            "hrb_image_destroy": (ctypes.c_int, [P]),
            "hrb_image_data": (P, [P]),
            "hrb_image_weights": (ctypes.c_int, [P, P, u32, ctypes.c_uint64, ctypes.c_uint64,
                                                 u32, u32, P, P, P]),
            "hrb_gemm_image": (ctypes.c_int, [P, P, ctypes.POINTER(GemmDesc), ctypes.c_uint64,
                                              ctypes.c_uint64, P]),
        }
        for name, (res, args) in sigs.items():
            f = getattr(lib, name, None)
            if f is None:  # an older build; tests/test_capi_host.py checks the exports
                continue
            f.restype = res
            f.argtypes = args
        _lib = lib
    return _lib


def _ptr(x) -> int | None:
    if x is None:
        return None
    if isinstance(x, int):
        return x
    if isinstance(x, np.ndarray):
        return x.ctypes.data
    return x.data_ptr()  # torch tensor


def shard_columns(n: int, rank: int, ranks: int) -> tuple[int, int]:
    """hrb_shard_columns: output columns [n0, n1) of `rank` of `ranks`, in
    whole 128-column tiles (no device needed)."""
    n0, n1 = ctypes.c_uint32(), ctypes.c_uint32()
    load().hrb_shard_columns(n, rank, ranks, ctypes.byref(n0), ctypes.byref(n1))
    return n0.value, n1.value


def shard_rows(units: int, rank: int, ranks: int) -> tuple[int, int]:
    """hrb_shard_rows: units (e.g. images) [u0, u1) of `rank` of `ranks`."""
    u0, u1 = ctypes.c_uint32(), ctypes.c_uint32()
    load().hrb_shard_rows(units, rank, ranks, ctypes.byref(u0), ctypes.byref(u1))
    return u0.value, u1.value


def image_region(meta_json: str, name: str) -> tuple[int, int]:
    """hrb_image_region: [offset, size] of region `name` in meta.json text."""
    off, size = ctypes.c_uint64(), ctypes.c_uint64()
    st = load().hrb_image_region(meta_json.encode(), name.encode(), ctypes.byref(off),
                                 ctypes.byref(size))
    if st != HRB_OK:
        raise HrbError(st, (load().hrb_last_error(None) or b"").decode())
    return off.value, size.value


class Image:
    """An hrb_image: a compiled program's image.bin on the context's device."""

    def __init__(self, owner: "Library", data: bytes | np.ndarray):
        self.owner = owner
        buf = np.frombuffer(bytes(data), np.uint8) if isinstance(data, bytes) else data
        buf = np.ascontiguousarray(buf, np.uint8)
        h = ctypes.c_void_p()
        owner._check(owner.lib.hrb_image_upload(owner.ctx, buf.ctypes.data, buf.size,
                                                ctypes.byref(h)))
        self.h = h

    def weights(self, wfmt, offset, N, K, w, wscale, offset_lo=0, stream=0) -> None:
        self.owner._check(self.owner.lib.hrb_image_weights(
            self.owner.ctx, self.h, wfmt, offset, offset_lo, N, K, _ptr(w), _ptr(wscale),
            stream or None))

    def gemm(self, d: "GemmDesc", offset: int, offset_lo: int = 0, stream: int = 0) -> None:
        self.owner._check(self.owner.lib.hrb_gemm_image(self.owner.ctx, self.h, ctypes.byref(d),
                                                        offset, offset_lo, stream or None))

    def close(self) -> None:
        if self.h:
            self.owner.lib.hrb_image_destroy(self.h)
            self.h = None


def comm_id_new() -> bytes:
    """hrb_comm_id_new: a fresh bootstrap id (rank 0 makes it)."""
    cid = CommId()
    st = load().hrb_comm_id_new(ctypes.byref(cid))
    if st != HRB_OK:
        raise HrbError(st, (load().hrb_last_error(None) or b"").decode())
    return bytes(cid.bytes)


class Comm:
    """An hrb_comm over a context: NCCL among the ranks of one node."""

    def __init__(self, owner: "Library", comm_id: bytes, rank: int, ranks: int):
        self.owner = owner
        self.rank, self.ranks = rank, ranks
        cid = CommId.from_buffer_copy(comm_id)
        h = ctypes.c_void_p()
        owner._check(owner.lib.hrb_comm_create(owner.ctx, ctypes.byref(cid), rank, ranks,
                                               ctypes.byref(h)))
        self.h = h

    def exchange(self, mine: bytes) -> list[bytes]:
        """Every rank's record (all the same length), in rank order."""
        n = len(mine)
        src = ctypes.create_string_buffer(mine, n)
        dst = ctypes.create_string_buffer(n * self.ranks)
        self.owner._check(self.owner.lib.hrb_comm_exchange(self.h, src, dst, n))
        raw = dst.raw
        return [raw[i * n:(i + 1) * n] for i in range(self.ranks)]

    def barrier(self) -> None:
        self.owner._check(self.owner.lib.hrb_comm_barrier(self.h))

    def fence(self, stream: int = 0) -> None:
        """hrb_comm_fence: later work on `stream` waits for every rank's
        earlier work on its stream."""
        self.owner._check(self.owner.lib.hrb_comm_fence(self.h, stream or None))

    def allgather(self, buf, offsets: list[int], stream: int = 0) -> None:
        """In place: rank r's bytes [offsets[r], offsets[r + 1]) of `buf`
        to every rank."""
        arr = (ctypes.c_uint64 * len(offsets))(*offsets)
        self.owner._check(self.owner.lib.hrb_comm_allgather(self.h, _ptr(buf), arr,
                                                            stream or None))

    def close(self) -> None:
        if self.h:
            self.owner.lib.hrb_comm_destroy(self.h)
            self.h = None


def gemm_check(cmd: GemmCmd) -> tuple[int, str]:
    """hrb_gemm_check without a context (host only)."""
    lib = load()
    return lib.hrb_gemm_check(None, ctypes.byref(cmd)), ""


def gemm_decode(instruction: bytes) -> GemmCmd:
    lib = load()
    cmd = GemmCmd()
    buf = (ctypes.c_uint8 * 16).from_buffer_copy(instruction)
    st = lib.hrb_gemm_decode(buf, ctypes.byref(cmd))
    if st != HRB_OK:
        raise HrbError(st, "decode")
    return cmd


def gemm_accesses(cmd: GemmCmd):
    lib = load()
    a = np.zeros(ABUF_WORDS, np.uint8)
    w = np.zeros(WBUF_WORDS, np.uint8)
    fr = np.zeros(FBUF_WORDS, np.uint8)
    fw = np.zeros(FBUF_WORDS, np.uint8)
    st = lib.hrb_gemm_accesses(ctypes.byref(cmd), a.ctypes.data, w.ctypes.data,
                               fr.ctypes.data, fw.ctypes.data)
    if st != HRB_OK:
        raise HrbError(st, "invalid command")
    return a, w, fr, fw


class Library:
    """One hrb_ctx on a CUDA device."""

    def __init__(self, device: int = 0):
        self.lib = load()
        ctx = ctypes.c_void_p()
        st = self.lib.hrb_create(device, ctypes.byref(ctx))
        if st != HRB_OK:
            raise HrbError(st, "hrb_create failed")
        self.ctx = ctx
        self.device = device

    def close(self) -> None:
        if self.ctx:
            self.lib.hrb_destroy(self.ctx)
            self.ctx = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass

    # -- helpers ----------------------------------------------------------
    def _check(self, st: int) -> None:
        if st != HRB_OK:
            raise HrbError(st, self.lib.hrb_last_error(self.ctx).decode())

    def last_error(self) -> str:
        return self.lib.hrb_last_error(self.ctx).decode()

    def sync(self) -> None:
        self._check(self.lib.hrb_sync(self.ctx))

    def stream(self) -> int:
        return self.lib.hrb_get_stream(self.ctx) or 0

    def set_stream(self, stream: int) -> None:
        self._check(self.lib.hrb_set_stream(self.ctx, stream))

    def launches(self) -> int:
        return int(self.lib.hrb_launch_count(self.ctx))

    # -- ISS drop-in ------------------------------------------------------
    def check(self, cmd: GemmCmd) -> int:
        return self.lib.hrb_gemm_check(self.ctx, ctypes.byref(cmd))

    def exec(self, cmd: GemmCmd, abuf: np.ndarray, wbuf: np.ndarray, fbuf: np.ndarray) -> None:
        assert abuf.dtype == np.uint8 and abuf.size == ABUF_WORDS * ABUF_WORD_BYTES
        assert wbuf.dtype == np.uint8 and wbuf.size == WBUF_WORDS * WBUF_WORD_BYTES
        assert fbuf.dtype == np.uint32 and fbuf.size == FBUF_WORDS * 32
        assert abuf.flags.c_contiguous and wbuf.flags.c_contiguous and fbuf.flags.c_contiguous
        self._check(self.lib.hrb_gemm_exec(self.ctx, ctypes.byref(cmd), abuf.ctypes.data,
                                           wbuf.ctypes.data, fbuf.ctypes.data))

    def exec_device(self, cmd: GemmCmd, abuf, wbuf, fbuf, stream: int = 0) -> None:
        self._check(self.lib.hrb_gemm_exec_device(self.ctx, ctypes.byref(cmd), _ptr(abuf),
                                                  _ptr(wbuf), _ptr(fbuf), stream or None))

    # -- dense ------------------------------------------------------------
    @staticmethod
    def desc(wfmt, M, N, K, *, a=None, lda=None, quant=QUANT_HOST, aq=None, ascale=None,
             w=None, wscale=None, bias=None, c=None, ldc=None, accumulate=False,
             pieces=None, mode=MODE_EXACT, cq=None, cscale=None, cquant=QUANT_VEC,
             wcol_scale=None, w8_kernel=0, ldcq=0):
        d = GemmDesc()
        d.wfmt, d.mode, d.M, d.N, d.K = wfmt, mode, M, N, K
        d.a = _ptr(a)
        d.lda = lda if lda is not None else (K if a is not None else 0)
        d.quant = quant
        d.aq, d.ascale = _ptr(aq), _ptr(ascale)
        d.w, d.wscale = _ptr(w), _ptr(wscale)
        d.bias = _ptr(bias)
        d.c = _ptr(c)
        d.ldc = ldc if ldc is not None else N
        d.accumulate = 1 if accumulate else 0
        d.cq, d.cscale, d.cquant = _ptr(cq), _ptr(cscale), cquant
        d.wcol_scale = _ptr(wcol_scale)
        d.w8_kernel = w8_kernel
        d.ldcq = ldcq
        if pieces is not None:
            arr = np.ascontiguousarray(pieces, dtype=np.uint32)
            d._pieces_keep = arr  # keep alive
            d.pieces = arr.ctypes.data
            d.npieces = arr.size
        return d

    def dense(self, d: GemmDesc, stream: int = 0) -> None:
        self._check(self.lib.hrb_gemm_dense(self.ctx, ctypes.byref(d), stream or None))

    def gemm_rows(self, d: GemmDesc, r: Rows, stream: int = 0) -> None:
        """hrb_gemm_rows: d's activations from the row-format source r."""
        self._check(self.lib.hrb_gemm_rows(self.ctx, ctypes.byref(d), ctypes.byref(r),
                                           stream or None))

    def dense_host(self, d: GemmDesc) -> None:
        self._check(self.lib.hrb_gemm_dense_host(self.ctx, ctypes.byref(d)))

    def quantize(self, x, rows, cols, q, scale, ldx=None, quant=QUANT_HOST, stream=0) -> None:
        self._check(self.lib.hrb_quantize_mxint8(self.ctx, _ptr(x), rows, cols,
                                                 ldx if ldx is not None else cols, quant,
                                                 _ptr(q), _ptr(scale), stream or None))

    def plan(self, descs: list[GemmDesc]) -> "Plan":
        return Plan(self, descs)

    # -- translation ------------------------------------------------------
    def shared_alloc(self, nbytes: int) -> tuple[int, bytes]:
        """hrb_shared_alloc: (device pointer, 64-byte IPC handle)."""
        ptr = ctypes.c_void_p()
        h = IpcHandle()
        self._check(self.lib.hrb_shared_alloc(self.ctx, nbytes, ctypes.byref(ptr), ctypes.byref(h)))
        return ptr.value, bytes(h.bytes)

    def shared_free(self, ptr: int) -> None:
        self._check(self.lib.hrb_shared_free(self.ctx, ptr))

    def peer_open(self, handle: bytes) -> int:
        h = IpcHandle()
        ctypes.memmove(h.bytes, handle, 64)
        ptr = ctypes.c_void_p()
        self._check(self.lib.hrb_peer_open(self.ctx, ctypes.byref(h), ctypes.byref(ptr)))
        return ptr.value

    def peer_close(self, ptr: int) -> None:
        self._check(self.lib.hrb_peer_close(self.ctx, ptr))

    def wbuf_to_dense(self, words, groups, kb, codes, scales, stream=0):
        self._check(self.lib.hrb_wbuf_to_dense(self.ctx, _ptr(words), groups, kb, _ptr(codes),
                                               _ptr(scales), stream or None))

    def w8_planes_to_dense(self, hi, lo, groups, kb, q, scales, stream=0):
        self._check(self.lib.hrb_w8_planes_to_dense(self.ctx, _ptr(hi), _ptr(lo), groups, kb,
                                                    _ptr(q), _ptr(scales), stream or None))

    def abuf_to_dense(self, words, quads, kb, q, scales, stream=0):
        self._check(self.lib.hrb_abuf_to_dense(self.ctx, _ptr(words), quads, kb, _ptr(q),
                                               _ptr(scales), stream or None))

    def t32_split8(self, vq, vscale, tokens, hd, wq, wscale, ldv=None, stream=0):
        """T32_SPLIT8 in dense form: V cache codes [tokens][ldv] + scales ->
        the W8 operand of P.V, codes [hd][tokens] + scales [hd][tokens/32]."""
        self._check(self.lib.hrb_t32_split8_dense(self.ctx, _ptr(vq), _ptr(vscale), tokens, hd,
                                                  hd if ldv is None else ldv, _ptr(wq),
                                                  _ptr(wscale), stream or None))

    def gacc(self, entries, w, rows, out, *, tokens, slots, corners, blocks, row_stride, nrows,
             accumulate=False, stream: int = 0) -> None:
        """hrb_gacc_dense on device buffers."""
        d = GaccDesc(tokens, slots, corners, blocks, _ptr(entries), _ptr(w), _ptr(rows),
                     row_stride, nrows, _ptr(out), 1 if accumulate else 0)
        self._check(self.lib.hrb_gacc_dense(self.ctx, ctypes.byref(d), stream or None))

    def conv(self, d: ConvDesc, stream: int = 0) -> None:
        self._check(self.lib.hrb_conv_dense(self.ctx, ctypes.byref(d), stream or None))

    def conv_plan(self, d: ConvDesc) -> ConvPlan:
        return ConvPlan(self, d)

    def dense_to_fbuf(self, c, rows, cols, words, stream=0):
        self._check(self.lib.hrb_dense_to_fbuf(self.ctx, _ptr(c), rows, cols, _ptr(words),
                                               stream or None))


def conv_desc(wfmt, images, H, W, cin, cout, kh, stride, *, order=CONV_XMAJOR, a=None,
              quant=QUANT_HOST, aq=None, ascale=None, w=None, wscale=None, bias=None, c=None,
              accumulate=False, relu=False, mode=MODE_EXACT, cq=None, cscale=None,
              cquant=QUANT_VEC) -> ConvDesc:
    d = ConvDesc()
    d.wfmt, d.mode = wfmt, mode
    d.images, d.H, d.W, d.cin, d.cout, d.kh, d.stride, d.order = (
        images, H, W, cin, cout, kh, stride, order)
    d.a, d.quant = _ptr(a), quant
    d.aq, d.ascale = _ptr(aq), _ptr(ascale)
    d.w, d.wscale = _ptr(w), _ptr(wscale)
    d.bias, d.c = _ptr(bias), _ptr(c)
    d.accumulate = 1 if accumulate else 0
    d.relu = 1 if relu else 0
    d.cq, d.cscale, d.cquant = _ptr(cq), _ptr(cscale), cquant
    return d


class ConvPlan:
    def __init__(self, owner: "Library", desc: ConvDesc):
        self.owner = owner
        self.desc = desc
        h = ctypes.c_void_p()
        owner._check(owner.lib.hrb_conv_plan_create(owner.ctx, ctypes.byref(desc),
                                                    ctypes.byref(h)))
        self.handle = h

    def run(self, stream: int = 0) -> int:
        n = ctypes.c_uint32()
        self.owner._check(self.owner.lib.hrb_conv_plan_run(self.handle, stream or None,
                                                           ctypes.byref(n)))
        return n.value

    def profile(self, reps: int = 20, stream: int = 0) -> list[float]:
        """Mean ms of each launch of a run (hrb_conv_plan_profile)."""
        ms = (ctypes.c_float * 8)()
        n = ctypes.c_uint32()
        self.owner._check(self.owner.lib.hrb_conv_plan_profile(self.handle, stream or None, reps,
                                                               ms, 8, ctypes.byref(n)))
        return [ms[i] for i in range(n.value)]

    def set_peers(self, local_base: int, peer_bases: list[int]) -> None:
        """hrb_conv_plan_set_peers: every output byte also goes to each peer
        base + (its address - local_base)."""
        arr = (ctypes.c_void_p * max(1, len(peer_bases)))(*peer_bases)
        self.owner._check(self.owner.lib.hrb_conv_plan_set_peers(self.handle, local_base, arr,
                                                                 len(peer_bases)))

    def close(self) -> None:
        if self.handle:
            self.owner.lib.hrb_conv_plan_destroy(self.handle)
            self.handle = None


class Plan:
    def __init__(self, owner: Library, descs: list[GemmDesc]):
        self.owner = owner
        arr = (GemmDesc * len(descs))(*descs)
        h = ctypes.c_void_p()
        owner._check(owner.lib.hrb_plan_create(owner.ctx, arr, len(descs), ctypes.byref(h)))
        self.h = h

    def run(self, stream: int = 0) -> int:
        n = ctypes.c_uint32()
        self.owner._check(self.owner.lib.hrb_plan_run(self.h, stream or None, ctypes.byref(n)))
        return n.value

    def run_host(self, a_host=None, c_host=None, ascale_host=None, stream: int = 0) -> None:
        """hrb_plan_run_host: per GEMM (creation order) host activations in,
        plan run, C out, asynchronous on `stream`.  Entries are host pointers
        (ints), arrays/tensors, or None to skip."""
        def arr(xs):
            if xs is None:
                return None
            return (ctypes.c_void_p * len(xs))(*[_ptr(x) for x in xs])
        self._host_args = (arr(a_host), arr(ascale_host), arr(c_host))  # alive until the call ends
        a, sc, c = self._host_args
        self.owner._check(self.owner.lib.hrb_plan_run_host(self.h, stream or None, a, sc, c))

    def set_peers(self, local_base: int, peer_bases: list[int]) -> None:
        """hrb_plan_set_peers: every output also goes to each peer base +
        (its address - local_base)."""
        arr = (ctypes.c_void_p * max(1, len(peer_bases)))(*peer_bases)
        self.owner._check(self.owner.lib.hrb_plan_set_peers(self.h, local_base, arr,
                                                            len(peer_bases)))

    def profile(self, reps: int = 10, stream: int = 0) -> list[float]:
        """Mean milliseconds of each kernel launch of the plan."""
        cap = 16
        ms = (ctypes.c_float * cap)()
        n = ctypes.c_uint32()
        self.owner._check(self.owner.lib.hrb_plan_profile(self.h, stream or None, reps, ms, cap,
                                                          ctypes.byref(n)))
        return [float(ms[i]) for i in range(n.value)]

    def close(self) -> None:
        if self.h:
            self.owner.lib.hrb_plan_destroy(self.h)
            self.h = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass


NPU_CLOCK_HZ = 250e6  # the NPU's PL clock (the reference's docs/design.md:27)


def npu_cycles(cmd_fields) -> int:
    """hrb_gemm_npu_cycles of one GEMM instruction (10 fields)."""
    return int(load().hrb_gemm_npu_cycles(ctypes.byref(GemmCmd(*[int(v) for v in cmd_fields]))))


def dense_npu_cycles(wfmt: int, M: int, N: int, K: int) -> int:
    """hrb_dense_npu_cycles: NPU cycles of a dense GEMM as GEMM instructions."""
    return int(load().hrb_dense_npu_cycles(wfmt, M, N, K))
