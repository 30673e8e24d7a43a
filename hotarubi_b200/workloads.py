"""Seeded synthetic operands for the benchmark configurations.

No public dataset is involved: the reference quotes no benchmark data for
this path, and its calibration sets are not needed.  Each tensor draws from
``numpy.random.default_rng(seed)`` with its own seed, with the shapes and
distributions of the five configurations:

* C1  W8 GEMM 64 x 960 -> 2560: activations N(0,1); int8 weights uniform in
  [-127, 127] with a per-output-channel FP32 scale |N(0, 0.02)| / 127; bias
  N(0, 0.01).  The reference runs per-channel weights as hotarubi's compiler
  places any float matrix (PlaceW8, tools/compiler/smolvla_common.cpp:95-103):
  dequantize (q * s, FP32), EncodeMxint8, SplitW8.
* C2  MXFP4 GEMM 64 x 2560 -> 960: activations N(0,1); E2M1 codes uniform
  over the 16 codes, one E8M0 scale per 32-block with exponent uniform in
  [-10, -4], passed through CanonicalMxfp4 (tools/compiler/weights.cpp:39-70)
  as the compiler does before packing; no bias.
* MXFP8 weights: E4M3 codes uniform over the finite codes, E8M0 exponent
  uniform in [-10, -4].

Weights come out in the dense formats of include/hrb_gemm.h.
"""
from __future__ import annotations

import numpy as np

_HALF_UNITS = np.array([0, 1, 2, 3, 4, 6, 8, 12], dtype=np.int32)
_FLOOR_LOG2 = np.array([0, -1, 0, 0, 1, 1, 2, 2], dtype=np.int32)
_HALF_TO_INDEX = np.full(13, -1, dtype=np.int32)
_HALF_TO_INDEX[_HALF_UNITS] = np.arange(8)


def activations(seed: int, m: int, k: int) -> np.ndarray:
    return np.random.default_rng(seed).standard_normal((m, k), dtype=np.float32)


def canonical_mxfp4(code: np.ndarray, e: np.ndarray, shift: int = 0):
    """hotarubi's CanonicalMxfp4 on [N, K] 4-bit codes and [N, K/32] block
    exponents: every nonzero block is rescaled so that its largest magnitude
    code has value >= 2 (index 4..7), the exponent absorbing the change, plus
    ``shift``; all-zero blocks become exponent 0 with +0 codes."""
    n, k = code.shape
    blocks = k // 32
    c = code.reshape(n, blocks, 32).astype(np.int32)
    mag = c & 7
    top = mag.max(axis=2)
    up = 2 - _FLOOR_LOG2[top]
    index = _HALF_TO_INDEX[_HALF_UNITS[mag] << up[..., None]]
    out = np.where((index != 0) & ((c & 8) != 0), index | 8, index).astype(np.uint8)
    e_out = e.astype(np.int32) + _FLOOR_LOG2[top] - 2 + shift
    zero = top == 0
    out[zero] = 0
    e_out[zero] = 0
    return out.reshape(n, k), e_out


def pack_nibbles(code: np.ndarray) -> np.ndarray:
    """[N, K] codes -> [N, K/2] bytes, element 2j in the low nibble of byte j."""
    c = code.astype(np.uint8) & 0xF
    return (c[:, 0::2] | (c[:, 1::2] << 4)).astype(np.uint8)


def mxfp4_weights(seed: int, n: int, k: int):
    """C2 weights: (packed codes [N, K/2], scale bytes [N, K/32])."""
    rng = np.random.default_rng(seed)
    code = rng.integers(0, 16, (n, k), dtype=np.int32).astype(np.uint8)
    e = rng.integers(-10, -3, (n, k // 32), dtype=np.int32)
    code, e = canonical_mxfp4(code, e)
    return pack_nibbles(code), (e + 127).astype(np.uint8)


def w8_per_channel(seed: int, n: int, k: int):
    """C1 weights before placement: int8 [N, K], FP32 per-channel scale [N]."""
    rng = np.random.default_rng(seed)
    q = rng.integers(-127, 128, (n, k), dtype=np.int32).astype(np.int8)
    s = (np.abs(rng.standard_normal(n)) * 0.02 / 127.0).astype(np.float32)
    return q, s


def dequantize_per_channel(q: np.ndarray, s: np.ndarray) -> np.ndarray:
    """q * s rounded once to FP32 (the product of an int8 and an FP32 is
    exact in double, so the float32 cast is the single rounding)."""
    return (q.astype(np.float64) * s.astype(np.float64)[:, None]).astype(np.float32)


def mxfp8_weights(seed: int, n: int, k: int):
    """E4M3 codes [N, K] (no NaN codes) and scale bytes [N, K/32]."""
    rng = np.random.default_rng(seed)
    code = rng.integers(0, 254, (n, k), dtype=np.int32).astype(np.uint8)
    code[code >= 0x7F] += 1            # skip 0x7F; 0xFF is out of range too
    e = rng.integers(-10, -3, (n, k // 32), dtype=np.int32)
    return code, (e + 127).astype(np.uint8)


def bias(seed: int, n: int, sigma: float = 0.01) -> np.ndarray:
    return (np.random.default_rng(seed).standard_normal(n) * sigma).astype(np.float32)


CONFIGS = {
    "c1_w8_64x960x2560": dict(wfmt=1, M=64, K=960, N=2560, bias=True),
    "c2_mxfp4_64x2560x960": dict(wfmt=0, M=64, K=2560, N=960, bias=False),
}
