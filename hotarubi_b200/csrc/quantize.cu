// FP32 -> MXINT8 on the device: the prologue of every hotarubi GEMM (the VEC
// 'q' pass that writes ABUF on the NPU; EncodeMxint8 on the host).
//
//   host rule  tools/runtime/formats.cpp:35-56 (QuantizeInt8),
//              :138-162 (EncodeMxint8)
//   VEC rule   tools/iss/lane.cpp:384-423 (QuantizeElement, QuantizeBlock)
//
// Both rules: the block exponent is the FP32 exponent field of the block's
// largest magnitude; q = x * 2^(6 - e) rounded to nearest even and clamped to
// [-128, 127].  They differ on subnormal inputs (the VEC pass reads them as
// zero) and on all-zero blocks' scale bytes only when those hold subnormals.
//
// Layout: a thread owns four consecutive elements of a row, eight lanes own a
// 32-element block, a warp covers 128 elements (4 blocks) of one row.  The
// block maximum is an integer max over the magnitude bits across 8 lanes.
// Traffic is the compulsory 4 bytes in and 1 + 1/32 bytes out per element.
#include <algorithm>
#include <cstdint>

#include "hrb_kernels.cuh"
#include "hrb_quant.cuh"
#include "hrb_tc.cuh"
#include "sm100.cuh"

namespace hrb {
namespace {

// One unit of work: 128 consecutive elements (four blocks) of one row.
struct Unit {
  const QuantJob* job;
  uint32_t row, chunk, col0;
};

// Loads the unit's four elements of this lane.
__device__ __forceinline__ void load_unit(const Unit& t, uint32_t v[4]) {
  const QuantJob& job = *t.job;
  const float* src = job.x + static_cast<size_t>(t.row) * job.ldx;
  if (t.col0 + 3u < job.cols && job.vec4) {
    const float4 f = __ldcs(reinterpret_cast<const float4*>(src + t.col0));
    v[0] = __float_as_uint(f.x);
    v[1] = __float_as_uint(f.y);
    v[2] = __float_as_uint(f.z);
    v[3] = __float_as_uint(f.w);
  } else {
#pragma unroll
    for (int i = 0; i < 4; ++i) v[i] = t.col0 + i < job.cols ? __float_as_uint(src[t.col0 + i]) : 0u;
  }
}

// q of four elements of one block.  Normal case: x * 2^(6 - e) is an exact
// FP32 scaling (|result| < 2^7), and adding 1.5 * 2^23 rounds it to the
// nearest integer, ties to even, exactly as QuantizeInt8 / QuantizeElement do;
// the integer rules above handle blocks whose scale 2^(6 - e) leaves the FP32
// range.  The VEC rule reads subnormal inputs as zero.
__device__ __forceinline__ void quantize4(const uint32_t v[4], uint32_t key, bool vec_rule,
                                          int32_t q[4], uint32_t& scale) {
  int32_t e;  // block exponent, value scale 2^(e - 6)
  if (vec_rule) {
    e = static_cast<int32_t>(key) - 127;
    scale = key == 0 ? 127u : key;
  } else {
    e = key != 0 ? static_cast<int32_t>(key >> 23) - 127 : 0;
    scale = static_cast<uint32_t>(e + 127);
  }
  if (e >= -120 && e < 128) {
    const float sc = __uint_as_float(static_cast<uint32_t>(133 - e) << 23);  // 2^(6 - e)
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      const float y = __uint_as_float(v[i]) * sc;
      int32_t r = __float_as_int(y + 12582912.0f) - 0x4B400000;
      r = r < -128 ? -128 : (r > 127 ? 127 : r);
      if (vec_rule && ((v[i] >> 23) & 0xFFu) == 0) r = 0;
      q[i] = r;
    }
  } else if (vec_rule) {
#pragma unroll
    for (int i = 0; i < 4; ++i) q[i] = quantize_vec_rule(v[i], key);
  } else {
#pragma unroll
    for (int i = 0; i < 4; ++i) q[i] = quantize_host_rule(v[i], e);
  }
}

// Block maximum, encoding and stores of one unit.
__device__ __forceinline__ void finish_unit(const Unit& t, const uint32_t v[4], uint32_t lane,
                                            uint32_t* error_flag) {
  const QuantJob& job = *t.job;
  const bool vec_rule = job.vec_rule != 0;
  uint32_t key = 0;  // host rule: max magnitude; VEC rule: max exponent field
  bool bad = false;
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const uint32_t mag = v[i] & 0x7FFFFFFFu;
    bad |= (mag >> 23) == 0xFFu;
    const uint32_t k = vec_rule ? (mag >> 23) : mag;
    key = k > key ? k : key;
  }
  key = max(key, __shfl_xor_sync(0xFFFFFFFFu, key, 1));
  key = max(key, __shfl_xor_sync(0xFFFFFFFFu, key, 2));
  key = max(key, __shfl_xor_sync(0xFFFFFFFFu, key, 4));
  if (!vec_rule && __any_sync(0xFFFFFFFFu, bad) && lane == 0) atomicOr(error_flag, 1u);
  const uint32_t block = t.chunk * 4u + (lane >> 3);
  if (block >= job.kb) return;  // past the last block of the row
  int32_t q[4];
  uint32_t scale;
  quantize4(v, key, vec_rule, q, scale);
  if (job.q != nullptr) {
    const uint32_t packed = (static_cast<uint32_t>(q[0]) & 0xFFu) |
                            ((static_cast<uint32_t>(q[1]) & 0xFFu) << 8) |
                            ((static_cast<uint32_t>(q[2]) & 0xFFu) << 16) |
                            ((static_cast<uint32_t>(q[3]) & 0xFFu) << 24);
    const size_t ldq = job.ldq != 0 ? job.ldq : job.kb;
    *reinterpret_cast<uint32_t*>(job.q + static_cast<size_t>(t.row) * ldq * 32u + t.col0) = packed;
    if ((lane & 7u) == 0) job.scale[static_cast<size_t>(t.row) * ldq + block] = static_cast<uint8_t>(scale);
  }

}

// Each warp walks a contiguous range of units, so the job a unit belongs to
// is found by one binary search and then by stepping forward; the next
// unit's load is issued before the current one is encoded.
__global__ void __launch_bounds__(256)
k_quantize(const QuantJob* jobs, uint32_t njobs, const __grid_constant__ QuantJob inline_job,
           uint32_t* error_flag) {
  const uint32_t lane = threadIdx.x & 31u;
  const uint32_t warp = (blockIdx.x * blockDim.x + threadIdx.x) >> 5;
  const uint32_t nwarps = (gridDim.x * blockDim.x) >> 5;
  const uint64_t total = jobs != nullptr ? jobs[njobs - 1].unit_begin + jobs[njobs - 1].units
                                         : inline_job.units;
  const uint64_t per = (total + nwarps - 1) / nwarps;
  const uint64_t begin = static_cast<uint64_t>(warp) * per;
  const uint64_t end = begin + per < total ? begin + per : total;
  if (begin >= end) return;
  uint32_t j = 0;
  if (jobs != nullptr) {
    uint32_t lo = 0, hi = njobs - 1;
    while (lo < hi) {
      const uint32_t mid = (lo + hi + 1) >> 1;
      if (jobs[mid].unit_begin <= begin) lo = mid; else hi = mid - 1;
    }
    j = lo;
  }
  // Position of a unit inside its job: found once by division, then stepped
  // (consecutive units are consecutive 128-element chunks of a row).
  const QuantJob* job = jobs != nullptr ? &jobs[j] : &inline_job;
  uint64_t job_end = job->unit_begin + job->units;
  uint32_t chunks = (job->cover_blocks + 3u) / 4u;
  uint32_t row, chunk;
  {
    const uint32_t u = static_cast<uint32_t>(begin - job->unit_begin);
    row = u / chunks;
    chunk = u % chunks;
  }
  auto locate = [&](uint64_t unit) {
    if (unit >= job_end) {  // next job (only with a job array)
      job = &jobs[++j];
      job_end = job->unit_begin + job->units;
      chunks = (job->cover_blocks + 3u) / 4u;
      row = 0;
      chunk = 0;
    }
    Unit t;
    t.job = job;
    t.row = row;
    t.chunk = chunk;
    t.col0 = chunk * 128u + lane * 4u;
    if (++chunk == chunks) {
      chunk = 0;
      ++row;
    }
    return t;
  };
  Unit cur = locate(begin);
  uint32_t v[4];
  load_unit(cur, v);
  for (uint64_t unit = begin; unit < end; ++unit) {
    Unit nxt = cur;
    uint32_t w[4] = {0u, 0u, 0u, 0u};
    const bool more = unit + 1 < end;
    if (more) {
      nxt = locate(unit + 1);
      load_unit(nxt, w);
    }
    finish_unit(cur, v, lane, error_flag);
    cur = nxt;
#pragma unroll
    for (int i = 0; i < 4; ++i) v[i] = w[i];
  }
}


// ---------------------------------------------------------------------------
// Activations for the kind::mxf4 kernel: MXINT8 codes as three E2M1 digit
// planes (layout: mx_act_block_bytes / mx_act_sf_offset in hrb_tc.cuh).
//
// A unit is one (row, 256-element K step); lane l of the unit's warp owns
// elements 8l .. 8l+7 (four lanes per 32-element block), so each plane's row
// of the step is one 32-bit store per lane.  In FP32, all exact:
//   q  = RNE(x * 2^(6 - e))           (1.5 * 2^23 added and subtracted)
//   d2 = RNE(q / 64), r = q - 64 d2   (|r| <= 32)
//   d1 = RNE(r / 8),  d0 = r - 8 d1   (all digits in [-4, 4])
// and cvt.rn.satfinite.e2m1x2 packs the digits, which E2M1 holds exactly.
// Blocks whose scale 2^(6 - e) leaves the FP32 range take the integer rules
// of QuantizeInt8 / QuantizeElement for q.  A block whose scale byte is below
// 6 (largest magnitude under 2^-121) has no E8M0 scale for its lowest plane
// and is encoded as zero: its products, below 2^-121 |w|, are dropped.

__device__ __forceinline__ float rint_exact(float v) {
  return __fadd_rn(__fadd_rn(v, 12582912.0f), -12582912.0f);
}

__device__ __forceinline__ uint32_t pack_e2m1x8(const float d[8]) {
  uint32_t out;
  asm("{\n\t.reg .b8 b0, b1, b2, b3;\n\t"
      "cvt.rn.satfinite.e2m1x2.f32 b0, %2, %1;\n\t"
      "cvt.rn.satfinite.e2m1x2.f32 b1, %4, %3;\n\t"
      "cvt.rn.satfinite.e2m1x2.f32 b2, %6, %5;\n\t"
      "cvt.rn.satfinite.e2m1x2.f32 b3, %8, %7;\n\t"
      "mov.b32 %0, {b0, b1, b2, b3};\n\t}"
      : "=r"(out)
      : "f"(d[0]), "f"(d[1]), "f"(d[2]), "f"(d[3]), "f"(d[4]), "f"(d[5]), "f"(d[6]), "f"(d[7]));
  return out;
}

// The job fields the plane encoder reads, kept in registers.
struct PlaneJob {
  const float* x;
  uint8_t* tiles;
  uint32_t rows, cols, ldx, tile_rows, vec4, vec_rule;
  uint32_t f8;        // E4M3 planes (tiles_kind 3), else E2M1 planes
  uint32_t bf16;      // BF16 values (tiles_kind 4)
  uint32_t steps;     // operand K steps per row tile (256 elements E2M1, 128 E4M3 or BF16)
  uint32_t k_steps;   // units per row: 256-element groups
  uint32_t block_bytes, plane_bytes;  // the activation block, tile_rows * 128
  uint64_t unit_begin, units;
};

__device__ __forceinline__ PlaneJob plane_job(const QuantJob& j) {
  PlaneJob p;
  p.x = j.x;
  p.tiles = j.tiles;
  p.rows = j.rows;
  p.cols = j.cols;
  p.ldx = j.ldx;
  p.f8 = j.tiles_kind == 3;
  p.bf16 = j.tiles_kind == 4;
  p.steps = j.k_steps;
  p.k_steps = p.f8 || p.bf16 ? (j.k_steps + 1u) / 2u : j.k_steps;
  p.tile_rows = j.tile_rows;
  p.vec4 = j.vec4;
  p.vec_rule = j.vec_rule;
  p.block_bytes = p.f8     ? mx8_act_block_bytes(j.tile_rows)
                  : p.bf16 ? mxbf_act_block_bytes(j.tile_rows)
                           : mx_act_block_bytes(j.tile_rows);
  p.plane_bytes = j.tile_rows * 128u;
  p.unit_begin = j.unit_begin;
  p.units = j.units;
  return p;
}

// Where lane `lane`'s outputs for one row go (fixed while the row lasts):
// the row's tile block of step 0, the lane's plane-word offset in a block,
// and the offsets of its block's three scale bytes.
struct PlaneOut {
  uint8_t* blk0;
  uint32_t off;
  uint32_t sf[3];
};

__device__ __forceinline__ PlaneOut plane_out(const PlaneJob& j, uint32_t row, uint32_t lane) {
  const uint32_t shift = j.tile_rows == 64 ? 6u : 7u;
  const uint32_t rt = row >> shift, r = row & (j.tile_rows - 1u);
  PlaneOut o;
  o.blk0 = j.tiles + static_cast<size_t>(rt) * j.steps * j.block_bytes;
  if (j.bf16) {
    // BF16: lane l's eight values (16 bytes) are logical chunk l % 8 of row
    // r of atom (l / 8) % 2 of step 2 u + l / 16.
    o.off = ((lane >> 3) & 1u) * j.plane_bytes + r * 128u + (((lane & 7u) ^ (r & 7u)) << 4);
    o.sf[0] = o.sf[1] = o.sf[2] = 0;
  } else if (j.f8) {
    // E4M3: lane l's eight bytes are bytes 8 (l % 16) .. of the row of step
    // 2 u + l / 16: logical 16-byte chunk (l % 16) / 2, half l % 2.
    o.off = r * 128u + ((((lane & 15u) >> 1) ^ (r & 7u)) << 4) + (lane & 1u) * 8u;
#pragma unroll
    for (uint32_t p = 0; p < 2; ++p) {
      o.sf[p] = mx8_act_sf_offset(j.tile_rows, p * j.tile_rows + r, (lane >> 2) & 3u);
    }
    o.sf[2] = 0;
  } else {
    // E2M1: lane l's four bytes sit in logical 16-byte chunk l / 4 of the row;
    // lanes l % 4 = p < 3 of a block write plane p's scale byte.
    o.off = r * 128u + (((lane >> 2) ^ (r & 7u)) << 4) + (lane & 3u) * 4u;
    const uint32_t p = lane & 3u;
    o.sf[0] = p < 3u ? mx_act_sf_offset(j.tile_rows, p * j.tile_rows + r, lane >> 2) : 0u;
    o.sf[1] = o.sf[2] = 0;
  }
  return o;
}

__device__ __forceinline__ uint32_t pack_e4m3x4(float a0, float a1, float a2, float a3) {
  uint32_t out;
  asm("{\n\t.reg .b16 lo, hi;\n\t"
      "cvt.rn.satfinite.e4m3x2.f32 lo, %2, %1;\n\t"
      "cvt.rn.satfinite.e4m3x2.f32 hi, %4, %3;\n\t"
      "mov.b32 %0, {lo, hi};\n\t}"
      : "=r"(out)
      : "f"(a0), "f"(a1), "f"(a2), "f"(a3));
  return out;
}

// max(|a|, |b|) of two FP32 bit patterns with NaN propagation (the sign of
// the result is not used).
__device__ __forceinline__ float max_nan_abs(uint32_t a, uint32_t b) {
  float r;
  asm("max.NaN.xorsign.abs.f32 %0, %1, %2;" : "=f"(r) : "f"(__uint_as_float(a)),
      "f"(__uint_as_float(b)));
  return r;
}

__device__ __forceinline__ void write_planes(const PlaneJob& j, const PlaneOut& o, uint32_t step,
                                             const float (&t)[8], uint32_t scale, uint32_t lane,
                                             const uint32_t* lut);

template <bool kVec>
__device__ __forceinline__ void encode_planes(const PlaneJob& j, const PlaneOut& o, uint32_t step,
                                              uint32_t v[8], uint32_t lane, uint32_t& bad,
                                              const uint32_t* lut) {
  constexpr float kMagic = 12582912.0f;  // 1.5 * 2^23
  // The largest magnitude as an FP32 max of magnitudes (NaN-propagating, so
  // a NaN or an Inf still shows in the key); the VEC rule's key is its
  // exponent field (subnormals have field 0 either way).
  float m[4];
#pragma unroll
  for (uint32_t i = 0; i < 4; ++i) m[i] = max_nan_abs(v[2 * i], v[2 * i + 1]);
  uint32_t key =
      __float_as_uint(max_nan_abs(__float_as_uint(max_nan_abs(__float_as_uint(m[0]),
                                                              __float_as_uint(m[1]))),
                                  __float_as_uint(max_nan_abs(__float_as_uint(m[2]),
                                                              __float_as_uint(m[3]))))) &
      0x7FFFFFFFu;
  if (kVec) {
    key >>= 23;
#pragma unroll
    for (uint32_t i = 0; i < 8; ++i) {
      if (((v[i] >> 23) & 0xFFu) == 0) v[i] = 0;  // the VEC pass reads subnormals as zero
    }
  }
  key = max(key, __shfl_xor_sync(0xFFFFFFFFu, key, 1));
  key = max(key, __shfl_xor_sync(0xFFFFFFFFu, key, 2));
  int32_t e;
  uint32_t scale;
  if (kVec) {
    e = static_cast<int32_t>(key) - 127;
    scale = key == 0 ? 127u : key;
  } else {
    bad |= key >= 0x7F800000u;  // an Inf or NaN in the block
    e = key != 0 ? static_cast<int32_t>(key >> 23) - 127 : 0;
    scale = static_cast<uint32_t>(e + 127);
  }
  // t = q + 1.5 * 2^23: q in the low byte of its bits (two's complement).
  float t[8];
  if (scale < 6u && !j.bf16) {
    // The planes' scales 2^(e - 6 + 3p) start below E8M0's 2^-127: such a
    // block (largest magnitude under 2^-121) is encoded as zero.
#pragma unroll
    for (uint32_t i = 0; i < 8; ++i) t[i] = kMagic;
  } else if (e >= -120 && e < 128) {
    // x * 2^(6 - e) is exact, so the fused add of 1.5 * 2^23 rounds it once;
    // q >= -128 always, and 128 clamps to 127.
    const float sc = __uint_as_float(static_cast<uint32_t>(133 - e) << 23);  // 2^(6 - e)
#pragma unroll
    for (uint32_t i = 0; i < 8; ++i) {
      t[i] = fminf(__fmaf_rn(__uint_as_float(v[i]), sc, kMagic), kMagic + 127.0f);
    }
  } else {
#pragma unroll
    for (uint32_t i = 0; i < 8; ++i) {
      t[i] = kMagic + static_cast<float>(kVec ? quantize_vec_rule(v[i], key)
                                               : quantize_host_rule(v[i], e));
    }
  }
  write_planes(j, o, step, t, scale, lane, lut);
}

// The lane's eight codes of one unit, t[i] = q + 1.5 * 2^23 (q in the low
// byte of the bits), with their block's scale byte, into the operand blocks:
// BF16 values, two E4M3 digit planes or three E2M1 digit planes.
__device__ __forceinline__ void write_planes(const PlaneJob& j, const PlaneOut& o, uint32_t step,
                                             const float (&t)[8], uint32_t scale, uint32_t lane,
                                             const uint32_t* lut) {
  constexpr float kMagic = 12582912.0f;  // 1.5 * 2^23
  if (j.bf16) {
    // q * 2^(scale - 133) in FP32, exact (a power-of-two multiple of an
    // integer below 2^8, at least 2^-133: a subnormal at worst, with the
    // IEEE multiply), whose low 16 bits are then zero: the high half is
    // the exact BF16 value.
    const float sc = __uint_as_float(scale >= 7u ? (scale - 6u) << 23 : 1u << (scale + 16u));
    uint32_t h[8];
#pragma unroll
    for (uint32_t i = 0; i < 8; ++i) {
      float y;
      asm("mul.rn.f32 %0, %1, %2;" : "=f"(y) : "f"(__fadd_rn(t[i], -kMagic)), "f"(sc));
      h[i] = __float_as_uint(y);
    }
    const uint32_t st = 2u * step + (lane >> 4);  // this lane's 128-element step
    if (st < j.steps) {
      *reinterpret_cast<uint4*>(o.blk0 + st * j.block_bytes + o.off) =
          make_uint4(__byte_perm(h[0], h[1], 0x7632u), __byte_perm(h[2], h[3], 0x7632u),
                     __byte_perm(h[4], h[5], 0x7632u), __byte_perm(h[6], h[7], 0x7632u));
    }
    return;
  }
  if (j.f8) {
    // Two E4M3 digits: h = RNE(q / 16), l = q - 16 h, both in [-8, 8].
    float h[8], l[8];
#pragma unroll
    for (uint32_t i = 0; i < 8; ++i) {
      const float qf = __fadd_rn(t[i], -kMagic);
      h[i] = __fadd_rn(__fmaf_rn(qf, 0.0625f, kMagic), -kMagic);
      l[i] = __fmaf_rn(h[i], -16.0f, qf);
    }
    const uint32_t st = 2u * step + (lane >> 4);  // this lane's 128-element step
    if (st < j.steps) {
      uint8_t* blk = o.blk0 + st * j.block_bytes;
      *reinterpret_cast<uint2*>(blk + o.off) =
          make_uint2(pack_e4m3x4(l[0], l[1], l[2], l[3]), pack_e4m3x4(l[4], l[5], l[6], l[7]));
      *reinterpret_cast<uint2*>(blk + j.plane_bytes + o.off) =
          make_uint2(pack_e4m3x4(h[0], h[1], h[2], h[3]), pack_e4m3x4(h[4], h[5], h[6], h[7]));
      if ((lane & 3u) == 0) {
#pragma unroll
        for (uint32_t p = 0; p < 2; ++p) {
          int32_t se = static_cast<int32_t>(scale) - 6 + 4 * static_cast<int32_t>(p);
          se = se > 254 ? 254 : se;  // scale >= 6 here or the block is zero
          blk[o.sf[p]] = static_cast<uint8_t>(se < 0 ? 0 : se);
        }
      }
    }
    return;
  }
  // The three E2M1 digit codes of each q from the table (bytes 0, 1, 2 of
  // lut[q & 0xFF]); pairs of elements merge into one word whose byte p is
  // plane p's byte for the pair (low nibble the even element), and byte
  // permutes gather each plane's four bytes.
  uint32_t pair[4];
#pragma unroll
  for (uint32_t k = 0; k < 4; ++k) {
    const uint32_t lo = lut[__float_as_uint(t[2 * k]) & 0xFFu];
    const uint32_t hi = lut[__float_as_uint(t[2 * k + 1]) & 0xFFu];
    pair[k] = lo | (hi << 4);
  }
  const uint32_t a01 = __byte_perm(pair[0], pair[1], 0x5140u);  // p0: 0,4  p1: 1,5
  const uint32_t a23 = __byte_perm(pair[2], pair[3], 0x5140u);
  const uint32_t b01 = __byte_perm(pair[0], pair[1], 0x0062u);  // p2: 2,6
  const uint32_t b23 = __byte_perm(pair[2], pair[3], 0x0062u);
  uint8_t* blk = o.blk0 + step * j.block_bytes;
  *reinterpret_cast<uint32_t*>(blk + o.off) = __byte_perm(a01, a23, 0x5410u);
  *reinterpret_cast<uint32_t*>(blk + j.plane_bytes + o.off) = __byte_perm(a01, a23, 0x7632u);
  *reinterpret_cast<uint32_t*>(blk + 2u * j.plane_bytes + o.off) = __byte_perm(b01, b23, 0x5410u);
  if ((lane & 3u) < 3u) {
    int32_t se = static_cast<int32_t>(scale) - 6 + 3 * static_cast<int32_t>(lane & 3u);
    se = se > 254 ? 254 : se;  // scale >= 6 here or the block is zero
    blk[o.sf[0]] = static_cast<uint8_t>(se < 0 ? 0 : se);
  }
}

// Position of a unit: its job (fields in registers), row and K step.
struct PlaneCursor {
  PlaneJob job;
  uint32_t jx, row, step;
};

// Moves to the next unit; returns true when the row changed.
__device__ __forceinline__ bool plane_cursor_next(PlaneCursor& c, const QuantJob* jobs,
                                                  uint32_t njobs) {
  if (++c.step < c.job.k_steps) return false;
  c.step = 0;
  if (++c.row == c.job.rows && jobs != nullptr && c.jx + 1 < njobs) {
    c.job = plane_job(jobs[++c.jx]);
    c.row = 0;
  }
  return true;
}

// Lane `lane`'s eight elements of a unit into its 32 bytes of the ring slot
// with cp.async (16-byte pieces, zero-filled past the row's end); rows that
// are not 16-byte aligned take plain loads.
__device__ __forceinline__ void stage8(const PlaneCursor& c, uint32_t lane, uint32_t* slot) {
  const uint32_t col0 = c.step * 256u + lane * 8u;
  const float* src = c.job.x + static_cast<size_t>(c.row) * c.job.ldx + col0;
  const uint32_t dst = static_cast<uint32_t>(__cvta_generic_to_shared(slot));
  if (c.job.vec4 && col0 + 8u <= c.job.cols) {
    asm volatile("cp.async.cg.shared.global [%0], [%1], 16;\n\t"
                 "cp.async.cg.shared.global [%2], [%3], 16;" ::"r"(dst), "l"(src), "r"(dst + 16u),
                 "l"(src + 4)
                 : "memory");
  } else if (c.job.vec4) {
#pragma unroll
    for (uint32_t h = 0; h < 2; ++h) {
      const uint32_t col = col0 + 4u * h;
      const uint32_t have = col < c.job.cols ? min(4u, c.job.cols - col) : 0u;
      const float* from = have != 0 ? src + 4u * h : c.job.x;  // any valid address when empty
      asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;" ::"r"(dst + 16u * h),
                   "l"(from), "r"(4u * have)
                   : "memory");
    }
  } else {
#pragma unroll
    for (uint32_t i = 0; i < 8; ++i) {
      slot[i] = col0 + i < c.job.cols ? __float_as_uint(src[i]) : 0u;
    }
  }
}

constexpr uint32_t kPlaneDepth = 4;       // units in flight per warp
constexpr uint32_t kPlaneWarps = 8;       // warps per CTA

// Each warp walks a contiguous range of units.  Its inputs arrive through a
// ring of kPlaneDepth units in shared memory filled by cp.async, so a warp
// keeps kPlaneDepth KB of loads in flight without holding them in registers.
__global__ void __launch_bounds__(kPlaneWarps * 32)
k_quantize_planes(const QuantJob* jobs, uint32_t njobs, const __grid_constant__ QuantJob inline_job,
                  uint32_t* error_flag) {
  __shared__ __align__(16) uint32_t ring[kPlaneWarps][kPlaneDepth][256];
  // lut[q & 0xFF]: the E2M1 codes of q's digits d0, d1, d2 in bytes 0, 1, 2,
  // with q = 64 d2 + 8 d1 + d0, d2 = RNE(q / 64), d1 = RNE((q - 64 d2) / 8).
  __shared__ uint32_t lut[256];
  {
    constexpr float kMagic = 12582912.0f;
    const float q = static_cast<float>(static_cast<int8_t>(threadIdx.x & 0xFFu));
    const float d2 = __fadd_rn(__fmaf_rn(q, 0.015625f, kMagic), -kMagic);
    const float r = __fmaf_rn(d2, -64.0f, q);
    const float d1 = __fadd_rn(__fmaf_rn(r, 0.125f, kMagic), -kMagic);
    const float d0 = __fmaf_rn(d1, -8.0f, r);
    const float d[8] = {d0, d1, d2, 0.0f, 0.0f, 0.0f, 0.0f, 0.0f};
    const uint32_t packed = pack_e2m1x8(d);  // nibble i = digit i's code
    if (threadIdx.x < 256u) {
      lut[threadIdx.x] = (packed & 0xFu) | ((packed >> 4) & 0xFu) << 8 | ((packed >> 8) & 0xFu) << 16;
    }
  }
  __syncthreads();
  // The table overlaps the kernel before; the activations it may have
  // written, and the operand blocks it may still read, come after.
  sm100::griddep_launch_dependents();
  sm100::griddep_wait();
  const uint32_t lane = threadIdx.x & 31u, wib = threadIdx.x >> 5;
  const uint32_t warp = blockIdx.x * kPlaneWarps + wib;
  const uint32_t nwarps = gridDim.x * kPlaneWarps;
  // The jobs may be a consecutive subset of a larger launch's: their units
  // are [first job's unit_begin, last job's end).
  const uint64_t base = jobs != nullptr ? jobs[0].unit_begin : 0;
  const uint64_t total = jobs != nullptr
                             ? jobs[njobs - 1].unit_begin + jobs[njobs - 1].units - base
                             : inline_job.units;
  const uint64_t per = (total + nwarps - 1) / nwarps;
  const uint64_t begin = base + static_cast<uint64_t>(warp) * per;
  const uint64_t end = begin + per < base + total ? begin + per : base + total;
  if (begin >= end) return;
  const uint32_t count = static_cast<uint32_t>(end - begin);
  PlaneCursor ld;
  ld.jx = 0;
  if (jobs != nullptr) {
    uint32_t lo = 0, hi = njobs - 1;
    while (lo < hi) {
      const uint32_t mid = (lo + hi + 1) >> 1;
      if (jobs[mid].unit_begin <= begin) lo = mid; else hi = mid - 1;
    }
    ld.jx = lo;
  }
  ld.job = plane_job(jobs != nullptr ? jobs[ld.jx] : inline_job);
  {
    const uint32_t u = static_cast<uint32_t>(begin - ld.job.unit_begin);
    ld.row = u / ld.job.k_steps;
    ld.step = u % ld.job.k_steps;
  }
  PlaneCursor pr = ld;
  PlaneOut out = plane_out(pr.job, pr.row, lane);
  uint32_t bad = 0;
  uint32_t* mine = &ring[wib][0][lane * 8u];
  // One commit group per unit (empty past the range) keeps the group count
  // uniform, so wait_group(kPlaneDepth - 1) always means "the oldest landed".
#pragma unroll
  for (uint32_t d = 0; d < kPlaneDepth; ++d) {
    if (d < count) {
      stage8(ld, lane, mine + d * 256u);
      plane_cursor_next(ld, jobs, njobs);
    }
    asm volatile("cp.async.commit_group;" ::: "memory");
  }
  for (uint32_t i = 0; i < count; ++i) {
    asm volatile("cp.async.wait_group %0;" ::"n"(kPlaneDepth - 1) : "memory");
    uint32_t* slot = mine + (i % kPlaneDepth) * 256u;
    uint32_t v[8];
    const uint4 lo = *reinterpret_cast<const uint4*>(slot);
    const uint4 hi = *reinterpret_cast<const uint4*>(slot + 4);
    v[0] = lo.x; v[1] = lo.y; v[2] = lo.z; v[3] = lo.w;
    v[4] = hi.x; v[5] = hi.y; v[6] = hi.z; v[7] = hi.w;
    if (pr.job.vec_rule) {
      encode_planes<true>(pr.job, out, pr.step, v, lane, bad, lut);
    } else {
      encode_planes<false>(pr.job, out, pr.step, v, lane, bad, lut);
    }
    if (plane_cursor_next(pr, jobs, njobs) && i + 1 < count) out = plane_out(pr.job, pr.row, lane);
    if (i + kPlaneDepth < count) {
      stage8(ld, lane, slot);
      plane_cursor_next(ld, jobs, njobs);
    }
    asm volatile("cp.async.commit_group;" ::: "memory");
  }
  if (__any_sync(0xFFFFFFFFu, bad != 0) && lane == 0) atomicOr(error_flag, 1u);
}


// ---------------------------------------------------------------------------
// The plane encoder's common case, specialised: E2M1 planes (kind::mxf4) of
// 16-byte-aligned FP32 rows, every job of the launch with NT-row tiles and
// one rounding rule.  Same outputs as k_quantize_planes; the work is laid
// out for fewer instructions per element:
//   * a warp takes one item at a time, one row's group of four 256-element
//     K steps (1024 values, 32 blocks), and lane l owns block l whole: the
//     block's largest magnitude is a max over the lane's own 32 values (no
//     shuffles), its scale is worked out once, and its three plane chunks
//     (a block is one 16-byte chunk of a plane row) leave as 16-byte stores;
//   * the item's 4 KB arrive by coalesced cp.async copies (lane l copies
//     16-byte chunks l + 32 j) into a ring slot, chunk c at position
//     c ^ ((c >> 3) & 7), so that each lane's eight chunks 8 l .. 8 l + 7 are
//     read without bank conflicts;
//   * q comes out of one fused multiply-add: t = x 2^(6 - e) + 1.5 2^23 is
//     rounded once to an integer (x 2^(6 - e) is exact), so the low byte of
//     t's bits is q in two's complement and (bits & 0xFF) * 4 is the byte
//     offset of q's digit codes in a table of words; a second table holds
//     the codes in the high nibbles, so an element pair merges with one OR;
//   * the job that holds a warp's first item is found with ballots over 32
//     jobs at a time instead of a serial search.
// Blocks whose scale 2^(6 - e) leaves the FP32 range (largest magnitude below
// 2^-120, or Inf/NaN) take the integer rules, as in k_quantize_planes.
constexpr uint32_t kE2m1Warps = 8;
constexpr uint32_t kE2m1Depth = 1;     // items in flight per warp (measured: 1 is 6 % faster
                                       // than 2 on C2; fewer registers, 4 CTAs an SM, slower)
constexpr uint32_t kE2m1Slot = 4096;   // bytes of one item
constexpr uint32_t kE2m1Smem = 2048 + kE2m1Warps * kE2m1Depth * kE2m1Slot;  // tables, ring

__device__ __forceinline__ uint32_t e2m1_pos(uint32_t c) { return c ^ ((c >> 3) & 7u); }

// A warp's walk over items (job jx, row, group of four K steps).
struct E2m1Walk {
  const float* x;
  uint8_t* tiles;
  uint32_t ldx, cols, rows, k_steps, groups;
  uint32_t jx, row, grp;
};

__device__ __forceinline__ void e2m1_job(E2m1Walk& w, const QuantJob& j) {
  w.x = j.x;
  w.tiles = j.tiles;
  w.ldx = j.ldx;
  w.cols = j.cols;
  w.rows = j.rows;
  w.k_steps = j.k_steps;
  w.groups = (j.k_steps + 3u) / 4u;
}

__device__ __forceinline__ void e2m1_next(E2m1Walk& w, const QuantJob* jobs, uint32_t njobs) {
  if (++w.grp < w.groups) return;
  w.grp = 0;
  if (++w.row == w.rows && jobs != nullptr && w.jx + 1u < njobs) {
    e2m1_job(w, jobs[++w.jx]);
    w.row = 0;
  }
}

// The item's 1024 values into a ring slot, zero past the row's end.
__device__ __forceinline__ void e2m1_stage(const E2m1Walk& w, uint32_t slot, uint32_t lane) {
  const uint32_t col0 = w.grp * 1024u;
  const float* src = w.x + static_cast<size_t>(w.row) * w.ldx + col0;
  if (col0 + 1024u <= w.cols) {
#pragma unroll
    for (uint32_t j = 0; j < 8; ++j) {
      const uint32_t c = lane + 32u * j;
      asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"(slot + 16u * e2m1_pos(c)),
                   "l"(src + 4u * c)
                   : "memory");
    }
  } else {
#pragma unroll
    for (uint32_t j = 0; j < 8; ++j) {
      const uint32_t c = lane + 32u * j;
      const uint32_t col = col0 + 4u * c;
      const uint32_t have = col < w.cols ? min(4u, w.cols - col) : 0u;
      const float* from = have != 0 ? src + 4u * c : w.x;  // any valid address when empty
      asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;" ::"r"(slot + 16u * e2m1_pos(c)),
                   "l"(from), "r"(4u * have)
                   : "memory");
    }
  }
}

// The integer rules for one element of a block whose scale 2^(6 - e) leaves
// the FP32 range: (q & 0xFF) * 4.  Out of line: it is rare, and inlined for
// each element it would crowd the instruction cache.  The planes' scales
// 2^(e - 6 + 3p) start below E8M0's 2^-127 when scale < 6: such a block is
// encoded as zero.
template <bool kVec>
__device__ __noinline__ uint32_t e2m1_slow_code(uint32_t x, uint32_t key, uint32_t scale) {
  const int32_t q = scale < 6u ? 0
                    : kVec     ? quantize_vec_rule(x, key)
                               : quantize_host_rule(x, static_cast<int32_t>(scale) - 127);
  return (static_cast<uint32_t>(q) & 0xFFu) << 2;
}

// Lane `lane`'s block of the item: its 32 values v into the three digit
// planes and their scale bytes.
template <uint32_t NT, bool kVec>
__device__ __forceinline__ void e2m1_block(const E2m1Walk& w, uint32_t (&v)[32], uint32_t lane,
                                           uint32_t& bad, const uint8_t* lut) {
  constexpr float kMagic = 12582912.0f;  // 1.5 * 2^23
  constexpr uint32_t kPlane = NT * 128u;
  float m[16];
#pragma unroll
  for (uint32_t i = 0; i < 16; ++i) m[i] = max_nan_abs(v[2 * i], v[2 * i + 1]);
#pragma unroll
  for (uint32_t s = 8; s >= 1; s /= 2) {
#pragma unroll
    for (uint32_t i = 0; i < s; ++i) m[i] = max_nan_abs(__float_as_uint(m[i]), __float_as_uint(m[i + s]));
  }
  const uint32_t mb = __float_as_uint(m[0]) & 0x7FFFFFFFu;
  // Host rule: the key is the largest magnitude (an Inf or NaN shows as a
  // key >= 0x7F800000); VEC rule: its exponent field, subnormals reading as
  // zero.
  const uint32_t key = kVec ? (mb >> 23) : mb;
  if (!kVec) bad = max(bad, key);
  const uint32_t step = w.grp * 4u + (lane >> 3);
  if (step >= w.k_steps) return;  // past the row's last K step: no operand block
  const uint32_t scale = key == 0 ? 127u : (kVec ? key : (key >> 23));  // e = scale - 127
  if (kVec) {
#pragma unroll
    for (uint32_t i = 0; i < 32; ++i) {
      if ((v[i] & 0x7F800000u) == 0) v[i] = 0;
    }
  }
  const uint32_t r = w.row % NT, b = lane & 7u;
  uint8_t* blk = w.tiles + (static_cast<size_t>(w.row / NT) * w.k_steps + step) * mx_act_block_bytes(NT);
  const bool fast = scale - 7u < 248u;  // 7 <= scale <= 254: 2^(6 - e) is a normal FP32
  // v[i] becomes (q & 0xFF) * 4.
  if (fast) {
    const float sc = __uint_as_float((260u - scale) << 23);
#pragma unroll
    for (uint32_t i = 0; i < 32; ++i) {
      // q >= -128 always; 128 clamps to 127.
      v[i] = (__float_as_uint(fminf(__fmaf_rn(__uint_as_float(v[i]), sc, kMagic),
                                    kMagic + 127.0f)) & 0xFFu) << 2;
    }
  } else {
#pragma unroll
    for (uint32_t i = 0; i < 32; ++i) v[i] = e2m1_slow_code<kVec>(v[i], key, scale);
  }
  uint32_t p0[4], p1[4], p2[4];
#pragma unroll
  for (uint32_t k = 0; k < 4; ++k) {
    uint32_t pair[4];
#pragma unroll
    for (uint32_t j = 0; j < 4; ++j) {
      pair[j] = *reinterpret_cast<const uint32_t*>(lut + v[8 * k + 2 * j]) |
                *reinterpret_cast<const uint32_t*>(lut + 1024u + v[8 * k + 2 * j + 1]);
    }
    const uint32_t a01 = __byte_perm(pair[0], pair[1], 0x5140u);  // p0: 0,4  p1: 1,5
    const uint32_t a23 = __byte_perm(pair[2], pair[3], 0x5140u);
    const uint32_t b01 = __byte_perm(pair[0], pair[1], 0x0062u);  // p2: 2,6
    const uint32_t b23 = __byte_perm(pair[2], pair[3], 0x0062u);
    p0[k] = __byte_perm(a01, a23, 0x5410u);
    p1[k] = __byte_perm(a01, a23, 0x7632u);
    p2[k] = __byte_perm(b01, b23, 0x5410u);
  }
  uint8_t* out = blk + r * 128u + ((b ^ (r & 7u)) << 4);
  *reinterpret_cast<uint4*>(out) = make_uint4(p0[0], p0[1], p0[2], p0[3]);
  *reinterpret_cast<uint4*>(out + kPlane) = make_uint4(p1[0], p1[1], p1[2], p1[3]);
  *reinterpret_cast<uint4*>(out + 2u * kPlane) = make_uint4(p2[0], p2[1], p2[2], p2[3]);
#pragma unroll
  for (uint32_t p = 0; p < 3; ++p) {
    int32_t se = static_cast<int32_t>(scale) - 6 + 3 * static_cast<int32_t>(p);
    if (!fast) se = se < 0 ? 0 : (se > 254 ? 254 : se);  // fast: always in [1, 254]
    blk[mx_act_sf_offset(NT, p * NT + r, b)] = static_cast<uint8_t>(se);
  }
}

template <uint32_t NT, bool kVec>
__global__ void __launch_bounds__(kE2m1Warps * 32, 3)
k_quantize_planes_e2m1(const QuantJob* jobs, uint32_t njobs,
                       const __grid_constant__ QuantJob inline_job, uint32_t* error_flag) {
  extern __shared__ __align__(16) uint8_t e2m1_smem[];
  // Byte offset 4 (q & 0xFF): the E2M1 codes of q's digits d0, d1, d2 (q =
  // 64 d2 + 8 d1 + d0, d2 = RNE(q / 64), d1 = RNE((q - 64 d2) / 8)) in the
  // low nibbles of bytes 0, 1, 2; from byte 1024 on, the same in the high
  // nibbles.  Then the ring: per warp kE2m1Depth slots of one item.
  uint32_t* lut = reinterpret_cast<uint32_t*>(e2m1_smem);
  {
    constexpr float kMagic = 12582912.0f;
    const float q = static_cast<float>(static_cast<int8_t>(threadIdx.x & 0xFFu));
    const float d2 = __fadd_rn(__fmaf_rn(q, 0.015625f, kMagic), -kMagic);
    const float r = __fmaf_rn(d2, -64.0f, q);
    const float d1 = __fadd_rn(__fmaf_rn(r, 0.125f, kMagic), -kMagic);
    const float d0 = __fmaf_rn(d1, -8.0f, r);
    const float d[8] = {d0, d1, d2, 0.0f, 0.0f, 0.0f, 0.0f, 0.0f};
    const uint32_t packed = pack_e2m1x8(d);  // nibble i = digit i's code
    const uint32_t codes =
        (packed & 0xFu) | ((packed >> 4) & 0xFu) << 8 | ((packed >> 8) & 0xFu) << 16;
    if (threadIdx.x < 256u) {
      lut[threadIdx.x] = codes;
      lut[256u + threadIdx.x] = codes << 4;
    }
  }
  __syncthreads();
  // The tables overlap the kernel before; the activations it may have
  // written, and the operand blocks it may still read, come after.
  sm100::griddep_launch_dependents();
  sm100::griddep_wait();
  const uint32_t lane = threadIdx.x & 31u, wib = threadIdx.x >> 5;
  const uint32_t warp = blockIdx.x * kE2m1Warps + wib;
  const uint32_t nwarps = gridDim.x * kE2m1Warps;
  const uint64_t base = jobs != nullptr ? jobs[0].group_begin : 0;
  uint64_t total;
  if (jobs != nullptr) {
    const QuantJob& last = jobs[njobs - 1];
    total = last.group_begin + static_cast<uint64_t>(last.rows) * ((last.k_steps + 3u) / 4u) - base;
  } else {
    total = static_cast<uint64_t>(inline_job.rows) * ((inline_job.k_steps + 3u) / 4u);
  }
  const uint64_t per = (total + nwarps - 1) / nwarps;
  const uint64_t begin = base + static_cast<uint64_t>(warp) * per;
  const uint64_t end = begin + per < base + total ? begin + per : base + total;
  if (begin >= end) return;
  const uint32_t count = static_cast<uint32_t>(end - begin);
  // The job of the first item: the last job starting at or before it,
  // narrowed 32 jobs a ballot.
  uint32_t jx = 0;
  if (jobs != nullptr) {
    uint32_t lo = 0, span = njobs;
    while (span > 1) {
      const uint32_t stride = (span + 31u) / 32u;
      const bool in = lane * stride < span;
      const bool le = in && jobs[lo + lane * stride].group_begin <= begin;
      const uint32_t k = 31u - __clz(__ballot_sync(0xFFFFFFFFu, le));  // lane 0 always holds
      lo += k * stride;
      span = min(stride, span - k * stride);
    }
    jx = lo;
  }
  E2m1Walk w;
  const QuantJob& j0 = jobs != nullptr ? jobs[jx] : inline_job;
  e2m1_job(w, j0);
  w.jx = jx;
  {
    const uint32_t u = static_cast<uint32_t>(begin - j0.group_begin);
    w.row = u / w.groups;
    w.grp = u % w.groups;
  }
  E2m1Walk ld = w;
  const uint8_t* lutb = e2m1_smem;
  uint8_t* ring = e2m1_smem + 2048 + wib * kE2m1Depth * kE2m1Slot;
  const uint32_t mine = static_cast<uint32_t>(__cvta_generic_to_shared(ring));
  uint32_t bad = 0;
  // One commit group per slot use, empty past the range, so that
  // wait_group(kE2m1Depth - 1) always means "the oldest has landed".
#pragma unroll
  for (uint32_t d = 0; d < kE2m1Depth; ++d) {
    if (d < count) {
      e2m1_stage(ld, mine + d * kE2m1Slot, lane);
      e2m1_next(ld, jobs, njobs);
    }
    asm volatile("cp.async.commit_group;" ::: "memory");
  }
#pragma unroll 1
  for (uint32_t i = 0; i < count; ++i) {
    const uint32_t d = i % kE2m1Depth;
    asm volatile("cp.async.wait_group %0;" ::"n"(kE2m1Depth - 1) : "memory");
    __syncwarp();  // the slot was filled by every lane's copies
    const uint8_t* slot = ring + d * kE2m1Slot;
    uint32_t v[32];
#pragma unroll
    for (uint32_t j = 0; j < 8; ++j) {
      const uint4 t = *reinterpret_cast<const uint4*>(slot + 16u * (8u * lane + (j ^ (lane & 7u))));
      v[4 * j] = t.x;
      v[4 * j + 1] = t.y;
      v[4 * j + 2] = t.z;
      v[4 * j + 3] = t.w;
    }
    __syncwarp();  // every lane has read the slot before it is refilled
    if (i + kE2m1Depth < count) {
      e2m1_stage(ld, mine + d * kE2m1Slot, lane);
      e2m1_next(ld, jobs, njobs);
    }
    asm volatile("cp.async.commit_group;" ::: "memory");
    e2m1_block<NT, kVec>(w, v, lane, bad, lutb);
    e2m1_next(w, jobs, njobs);
  }
  if (!kVec && __any_sync(0xFFFFFFFFu, bad >= 0x7F800000u) && lane == 0) atomicOr(error_flag, 1u);
}

}  // namespace

void launch_quantize(const QuantJob* jobs_dev, uint32_t njobs, const QuantJob* inline_job,
                     uint64_t total_units, uint32_t* error_flag, int sm_count,
                     cudaStream_t stream) {
  // Enough warps to keep every SM full (8 CTAs of 256 threads per SM); each
  // walks a contiguous range of units.
  uint64_t blocks = (total_units + 7) / 8;
  const uint64_t cap = static_cast<uint64_t>(sm_count) * 8;
  if (blocks > cap) blocks = cap;
  if (blocks == 0) blocks = 1;
  QuantJob one{};
  if (inline_job != nullptr) one = *inline_job;
  k_quantize<<<static_cast<unsigned>(blocks), 256, 0, stream>>>(jobs_dev, njobs, one, error_flag);
}

namespace {

// Which plane encoder serves a launch: 0 the general k_quantize_planes; else
// the specialised E2M1 kernel, 1 + 2 (tiles of 128 rows) + 1 (VEC rule), when
// every job holds E2M1 planes of 16-byte-aligned rows with one tile height
// and one rule.
uint32_t planes_variant(const QuantJob* jobs, uint32_t n) {
  if (jobs == nullptr || n == 0) return 0;
  const QuantJob& f = jobs[0];
  if (f.tile_rows != 64u && f.tile_rows != 128u) return 0;
  for (uint32_t i = 0; i < n; ++i) {
    const QuantJob& j = jobs[i];
    if (j.tiles_kind != 2u || !j.vec4 || j.tile_rows != f.tile_rows || j.vec_rule != f.vec_rule) {
      return 0;
    }
  }
  return 1u + (f.tile_rows == 128u ? 2u : 0u) + (f.vec_rule ? 1u : 0u);
}

template <typename K>
int occupancy_of(K kernel, uint32_t threads, uint32_t smem) {
  int n = 0;
  if (cudaOccupancyMaxActiveBlocksPerMultiprocessor(&n, kernel, threads, smem) != cudaSuccess ||
      n < 1) {
    n = 1;
  }
  return n;
}

}  // namespace

void launch_quantize_planes(const QuantJob* jobs_dev, uint32_t njobs, const QuantJob* inline_job,
                            uint64_t total_units, uint32_t* error_flag, int sm_count,
                            cudaStream_t stream, const QuantJob* jobs_host) {
  const QuantJob* host = inline_job != nullptr ? inline_job : jobs_host;
  const uint32_t n = inline_job != nullptr ? 1u : njobs;
  const uint32_t variant = planes_variant(host, n);
  using Fn = void (*)(const QuantJob*, uint32_t, const QuantJob, uint32_t*);
  static const Fn kFns[5] = {k_quantize_planes, k_quantize_planes_e2m1<64, false>,
                             k_quantize_planes_e2m1<64, true>, k_quantize_planes_e2m1<128, false>,
                             k_quantize_planes_e2m1<128, true>};
  const uint32_t warps = variant == 0 ? kPlaneWarps : kE2m1Warps;
  const uint32_t smem = variant == 0 ? 0u : kE2m1Smem;
  if (smem != 0 && !set_smem_limit_once(reinterpret_cast<const void*>(kFns[variant]), smem)) {
    return;  // the launch error surfaces through cudaGetLastError
  }
  // Work units: (row, 256-element step) for the general kernel, (row, group
  // of four steps) for the specialised one.
  uint64_t units = total_units;
  if (variant != 0) {
    units = 0;
    for (uint32_t i = 0; i < n; ++i) units += uint64_t{host[i].rows} * ((host[i].k_steps + 3u) / 4u);
  }
  // As many CTAs as fit at once (no second wave); each warp takes a
  // contiguous range of at least a few units.
  static int per_sm[5] = {0, 0, 0, 0, 0};
  if (per_sm[variant] == 0) per_sm[variant] = occupancy_of(kFns[variant], warps * 32u, smem);
  // Several units a warp when that fills the GPU; a smaller job (a few
  // hundred rows) spreads down to one unit a warp, so a warp waits for one
  // load, not several in a row.
  const uint64_t each = variant == 0 ? 4u : 2u;
  uint64_t blocks = (units + each * warps - 1) / (each * warps);
  const uint64_t cap = static_cast<uint64_t>(sm_count) * per_sm[variant];
  if (blocks < cap) blocks = std::min<uint64_t>(cap, (units + warps - 1) / warps);
  if (blocks > cap) blocks = cap;
  if (blocks == 0) blocks = 1;
  QuantJob one{};
  if (inline_job != nullptr) one = *inline_job;
  // Programmatic stream serialisation: the kernel waits (griddep_wait)
  // before it touches memory.
  cudaLaunchConfig_t cfg{};
  cfg.gridDim = dim3(static_cast<unsigned>(blocks));
  cfg.blockDim = dim3(warps * 32u);
  cfg.dynamicSmemBytes = smem;
  cfg.stream = stream;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  cudaLaunchKernelEx(&cfg, kFns[variant], jobs_dev, njobs, one, error_flag);
}

// ---------------------------------------------------------------------------
// MXINT8 activations (row format or dense) to the tensor-core operands.

namespace {

// The unit of token m, plane p: its window offset, or ~0 for a null entry;
// sets `outside` when the unit leaves the window.
__device__ __forceinline__ uint64_t rows_unit(const RowsSrc& s, uint32_t m, uint32_t p,
                                              bool& outside) {
  uint64_t off;
  if (s.index != nullptr) {
    const uint32_t e = s.index[m];
    if (e == 0xFFFFFFFFu) return ~uint64_t{0};
    const uint64_t addr = uint64_t{e} * 16u;
    if (addr < s.ddr_base) {
      outside = true;
      return ~uint64_t{0};
    }
    off = addr - s.ddr_base;
  } else {
    off = s.first + uint64_t{m / s.row_tokens} * s.row_stride +
          uint64_t{m % s.row_tokens} * s.unit_bytes;
  }
  off += uint64_t{p} * s.plane_stride;
  if (off + s.unit_bytes > s.window_bytes) {
    outside = true;
    return ~uint64_t{0};
  }
  return off;
}

// Eight codes (bytes 8 c .. 8 c + 7 of block b) of token m and the block's
// scale byte; a null entry or a block past kb reads as zero codes with
// scale 127 (the null unit of LoadRows, dma_engine.cpp:250-255).
__device__ __forceinline__ void rows_load8(const RowsSrc& s, uint32_t m, uint32_t b, uint32_t c,
                                           uint2& codes, uint32_t& scale, bool& outside) {
  codes = make_uint2(0u, 0u);
  scale = 127u;
  if (b >= s.kb) return;
  if (s.window == nullptr) {
    codes = *reinterpret_cast<const uint2*>(s.aq + size_t{m} * s.kp + b * 32u + c * 8u);
    scale = s.ascale[size_t{m} * s.kb + b];
    return;
  }
  const uint32_t p = b / s.tok, t = b % s.tok;
  const uint64_t off = rows_unit(s, m, p, outside);
  if (off == ~uint64_t{0}) return;
  const uint8_t* unit = s.window + off;
  codes = *reinterpret_cast<const uint2*>(unit + t * 32u + c * 8u);
  scale = unit[s.tok * 32u + t];
}

__global__ void __launch_bounds__(256)
k_rows_planes(const __grid_constant__ RowsSrc src, const __grid_constant__ QuantJob qj,
              uint32_t* error_flag) {
  __shared__ uint32_t lut[256];  // q -> its three E2M1 digit codes, as k_quantize_planes's
  {
    constexpr float kMagic = 12582912.0f;
    const float q = static_cast<float>(static_cast<int8_t>(threadIdx.x & 0xFFu));
    const float d2 = __fadd_rn(__fmaf_rn(q, 0.015625f, kMagic), -kMagic);
    const float r = __fmaf_rn(d2, -64.0f, q);
    const float d1 = __fadd_rn(__fmaf_rn(r, 0.125f, kMagic), -kMagic);
    const float d0 = __fmaf_rn(d1, -8.0f, r);
    const float d[8] = {d0, d1, d2, 0.0f, 0.0f, 0.0f, 0.0f, 0.0f};
    const uint32_t packed = pack_e2m1x8(d);
    lut[threadIdx.x] = (packed & 0xFu) | ((packed >> 4) & 0xFu) << 8 | ((packed >> 8) & 0xFu) << 16;
  }
  __syncthreads();
  sm100::griddep_launch_dependents();
  sm100::griddep_wait();
  constexpr float kMagic = 12582912.0f;
  const PlaneJob j = plane_job(qj);
  const uint32_t lane = threadIdx.x & 31u;
  const uint64_t warp = (uint64_t{blockIdx.x} * blockDim.x + threadIdx.x) >> 5;
  const uint64_t nwarps = (uint64_t{gridDim.x} * blockDim.x) >> 5;
  uint32_t bad = 0;
  bool outside = false;
  const bool e2m1 = !j.f8 && !j.bf16;
  for (uint64_t u = warp; u < j.units; u += nwarps) {
    // Unit (row m, 256-element group g): lane l holds elements 8 l .. 8 l + 7,
    // block 8 g + l / 4.
    const uint32_t m = static_cast<uint32_t>(u / j.k_steps);
    const uint32_t g = static_cast<uint32_t>(u % j.k_steps);
    uint2 codes;
    uint32_t scale;
    rows_load8(src, m, g * 8u + lane / 4u, lane & 3u, codes, scale, outside);
    float t[8];
#pragma unroll
    for (uint32_t i = 0; i < 8; ++i) {
      const uint32_t word = i < 4 ? codes.x : codes.y;
      t[i] = kMagic + static_cast<float>(static_cast<int8_t>((word >> (8u * (i & 3u))) & 0xFFu));
    }
    // As the FP32 encoders: E2M1 and E4M3 planes of a block with scale < 6
    // start below E8M0's range and the block is zero; E2M1's top plane
    // needs scale + 0 <= 254.
    if (!j.bf16 && scale < 6u) {
#pragma unroll
      for (uint32_t i = 0; i < 8; ++i) t[i] = kMagic;
    }
    if (e2m1 && scale == 255u) bad |= kErrScaleRange;
    write_planes(j, plane_out(j, m, lane), g, t, scale, lane, lut);
  }
  if (outside) bad |= kErrRowOutside;
  bad = __reduce_or_sync(0xFFFFFFFFu, bad);
  if (bad != 0 && lane == 0) atomicOr(error_flag, bad);
}

// Dense codes and scales: one warp per (token, group of 8 blocks); lane l
// copies 8 bytes of block 8 g + l / 4, lanes l % 4 == 0 the scale byte.
__global__ void __launch_bounds__(256)
k_rows_dense(const __grid_constant__ RowsSrc src, uint32_t M, int8_t* aq, uint8_t* ascale,
             uint32_t* error_flag) {
  sm100::griddep_launch_dependents();
  sm100::griddep_wait();
  const uint32_t lane = threadIdx.x & 31u;
  const uint64_t warp = (uint64_t{blockIdx.x} * blockDim.x + threadIdx.x) >> 5;
  const uint64_t nwarps = (uint64_t{gridDim.x} * blockDim.x) >> 5;
  const uint32_t groups = (src.kb + 7u) / 8u;
  bool outside = false;
  for (uint64_t u = warp; u < uint64_t{M} * groups; u += nwarps) {
    const uint32_t m = static_cast<uint32_t>(u / groups);
    const uint32_t b = static_cast<uint32_t>(u % groups) * 8u + lane / 4u;
    if (b >= src.kb) continue;
    uint2 codes;
    uint32_t scale;
    rows_load8(src, m, b, lane & 3u, codes, scale, outside);
    *reinterpret_cast<uint2*>(aq + size_t{m} * src.kb * 32u + b * 32u + (lane & 3u) * 8u) = codes;
    if ((lane & 3u) == 0) ascale[size_t{m} * src.kb + b] = static_cast<uint8_t>(scale);
  }
  if (__any_sync(0xFFFFFFFFu, outside) && lane == 0) atomicOr(error_flag, kErrRowOutside);
}

void launch_pdl(const void* fn, uint64_t work_warps, int sm_count, cudaStream_t stream,
                void** args) {
  uint64_t blocks = (work_warps + 7u) / 8u;
  const uint64_t cap = static_cast<uint64_t>(sm_count) * 8u;
  blocks = blocks > cap ? cap : (blocks == 0 ? 1 : blocks);
  cudaLaunchConfig_t cfg{};
  cfg.gridDim = dim3(static_cast<unsigned>(blocks));
  cfg.blockDim = dim3(256);
  cfg.stream = stream;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  cudaLaunchKernelExC(&cfg, fn, args);
}

}  // namespace

void launch_rows_planes(const RowsSrc& src, const QuantJob& job, uint32_t* error_flag,
                        int sm_count, cudaStream_t stream) {
  RowsSrc s = src;
  QuantJob j = job;
  uint32_t* e = error_flag;
  void* args[] = {&s, &j, &e};
  launch_pdl(reinterpret_cast<const void*>(k_rows_planes), job.units, sm_count, stream, args);
}

void launch_rows_dense(const RowsSrc& src, uint32_t M, int8_t* aq, uint8_t* ascale,
                       uint32_t* error_flag, int sm_count, cudaStream_t stream) {
  RowsSrc s = src;
  uint32_t m = M;
  int8_t* q = aq;
  uint8_t* sc = ascale;
  uint32_t* e = error_flag;
  void* args[] = {&s, &m, &q, &sc, &e};
  launch_pdl(reinterpret_cast<const void*>(k_rows_dense),
             uint64_t{M} * ((src.kb + 7u) / 8u), sm_count, stream, args);
}

}  // namespace hrb
