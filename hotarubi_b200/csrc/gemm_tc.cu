// The tensor-core GEMM (tcgen05, BF16 operands, FP32 accumulation in TMEM).
//
// Why BF16: hotarubi's activations are MXINT8 (q * 2^(e-6), |q| <= 128),
// which no FP8/FP6/FP4 element type holds exactly; an 8-bit significand does
// fit BF16, and so do every E2M1, E4M3 and int8 weight value times its E8M0
// scale.  So both operands are the exact dequantized values in BF16, the
// products are exact in FP32, and the only difference from the reference's
// chain is the order and grouping of the FP32 additions (HRB_MODE_FAST).
// One BF16 MMA costs the same tensor time as the two FP8 MMAs an exact
// 8-bit activation would need in a block-scaled FP8 kind.
//
// Operands travel as tiles prepared for one bulk copy each:
//   * activations: the encoder writes BF16 tiles of NT rows (tokens) x 64 K
//     (128 bytes per row), rows already in the 128-byte swizzle the MMA's
//     shared-memory descriptor expects, so a linear copy lands ready to use;
//   * weights: translated once per plan into chunks of 128 columns x 64 K of
//     raw codes (4-bit: 32 bytes per column, 8-bit: 64) followed by their
//     128 x 2 E8M0 scales.  Decoder warps expand a chunk to swizzled BF16.
//
// One CTA computes C[tokens m0..m0+NT) x [columns n0..n0+128) with the weight
// tile as the MMA's A operand (M = 128 columns) and the activation tile as B
// (N = NT tokens): D[column][token] in TMEM, 128 lanes x NT columns.
// Warp roles: 0 = weight-chunk producer, 1 = TMEM owner and MMA issuer,
// 2 = activation-tile producer, 3..6 = weight decoders, then the epilogue
// (TMEM -> registers -> C); warps 3..6 cover the four TMEM subpartitions.
#include <cuda_bf16.h>

#include <algorithm>
#include <cstdint>
#include <mutex>
#include <tuple>
#include <vector>

#include "hrb_device.cuh"
#include "hrb_kernels.cuh"
#include "hrb_tc.cuh"
#include "sm100.cuh"

namespace hrb {
namespace {

using namespace sm100;

constexpr uint32_t kTileW = 128;      // weight columns per CTA (MMA M)
constexpr uint32_t kStepK = 64;       // K elements per pipeline step
constexpr uint32_t kRowBytes = 128;   // one BF16 row of a step

__host__ __device__ constexpr uint32_t raw_row_bytes(uint32_t wfmt) {
  return wfmt == 0 ? 32u : 64u;
}
__host__ __device__ constexpr uint32_t chunk_bytes(uint32_t wfmt) {
  return kTileW * raw_row_bytes(wfmt) + kTileW * 2u;
}

template <uint32_t NT, uint32_t WF>
struct TcCfg {
  // Rings: activation tiles (bulk-copied), decoded BF16 weight tiles
  // (written by the decoder warps), raw weight chunks (bulk-copied).  Sized
  // so that NT = 64 fits two CTAs per SM.
  static constexpr uint32_t kAStages = NT == 256 ? 3u : 4u;
  static constexpr uint32_t kWStages = 2;
  static constexpr uint32_t kRaw = WF == 0 ? 8u : 5u;
  static constexpr uint32_t kABytes = NT * kRowBytes;
  static constexpr uint32_t kWBytes = kTileW * kRowBytes;
  static constexpr uint32_t kChunk = chunk_bytes(WF);
  static constexpr uint32_t kRawStride = (kChunk + 127) / 128 * 128;
  static constexpr uint32_t kTmemCols = NT < 32 ? 32 : NT;
  // Layout: [A stages][W stages][raw chunks][barriers][tmem slot]
  static constexpr uint32_t kOffW = kAStages * kABytes;
  static constexpr uint32_t kOffRaw = kOffW + kWStages * kWBytes;
  static constexpr uint32_t kOffBar = kOffRaw + kRaw * kRawStride;
  static constexpr uint32_t kSmem = kOffBar + 256 + 1024;  // + alignment slack
  static constexpr uint32_t kThreads = 224;
};

struct TcParams {
  const TcJob* jobs;   // device-resident jobs, or null: use inline_job
  uint32_t njobs;
  uint32_t* err;
  TcJob inline_job;
};

__device__ __forceinline__ uint32_t find_tc_job(const TcJob* jobs, uint32_t njobs, uint32_t tile) {
  uint32_t lo = 0, hi = njobs - 1;
  while (lo < hi) {
    const uint32_t mid = (lo + hi + 1) >> 1;
    if (jobs[mid].tile_begin <= tile) lo = mid; else hi = mid - 1;
  }
  return lo;
}

// bf16x2 of two FP32 (exact when they have at most 8 significant bits).
__device__ __forceinline__ uint32_t pack_bf16x2(float lo, float hi) {
  uint32_t r;
  asm("cvt.rn.bf16x2.f32 %0, %1, %2;" : "=r"(r) : "f"(hi), "f"(lo));
  return r;
}

__device__ __forceinline__ uint32_t bf16x2_mul(uint32_t a, uint32_t b) {
  __nv_bfloat162 x = *reinterpret_cast<__nv_bfloat162*>(&a);
  __nv_bfloat162 y = *reinterpret_cast<__nv_bfloat162*>(&b);
  __nv_bfloat162 z = __hmul2(x, y);
  return *reinterpret_cast<uint32_t*>(&z);
}

// 2^(e - 127) as a bf16x2 pair (e in 1..254).
__device__ __forceinline__ uint32_t pow2_bf16x2(uint32_t e) {
  const uint32_t h = (e & 0xFFu) << 7;
  return h | (h << 16);
}

// Eight E2M1 codes (one word, element 0 lowest) -> eight BF16 values of the
// E2M1 numbers {0, .5, 1, 1.5, 2, 3, 4, 6} with sign, as four bf16x2 words.
// The high and low byte of each BF16 come from 8-entry byte tables (prmt).
__device__ __forceinline__ void e2m1x8_to_bf16(uint32_t x, uint32_t out[4]) {
  // magnitudes 0, .5, 1, 1.5, 2, 3, 4, 6 -> BF16 0000 3F00 3F80 3FC0 4000 4040 4080 40C0
  constexpr uint32_t kHi0 = 0x3F3F3F00u, kHi1 = 0x40404040u;   // high bytes, index 0..7
  constexpr uint32_t kNh0 = 0xBFBFBF00u, kNh1 = 0xC0C0C0C0u;   // with the sign bit
  constexpr uint32_t kLo0 = 0xC0800000u, kLo1 = 0xC0804000u;   // low bytes
#pragma unroll
  for (int half = 0; half < 2; ++half) {
    const uint32_t v = x >> (16 * half);
    const uint32_t sel = v & 0x7777u;
    const uint32_t hp = __byte_perm(kHi0, kHi1, sel);
    const uint32_t hn = __byte_perm(kNh0, kNh1, sel);
    const uint32_t h = __byte_perm(hp, hn, 0x3210u | ((v >> 1) & 0x4444u));
    const uint32_t l = __byte_perm(kLo0, kLo1, sel);
    out[2 * half] = __byte_perm(l, h, 0x5140u);       // elements 0,1 of the group
    out[2 * half + 1] = __byte_perm(l, h, 0x7362u);   // elements 2,3
  }
}

// The decoded 128-byte row r of a step: 16-byte chunk c goes to c ^ (r % 8).
__device__ __forceinline__ uint32_t swz(uint32_t r, uint32_t c) {
  return r * kRowBytes + ((c ^ (r & 7u)) << 4);
}

// Decodes one raw weight row (64 K elements) into BF16, swizzled.
template <uint32_t WF>
__device__ __forceinline__ void decode_row(const uint8_t* raw, uint32_t r, uint8_t* dst) {
  const uint8_t* sc = raw + kTileW * raw_row_bytes(WF) + r * 2u;
  const uint32_t s0 = sc[0], s1 = sc[1];
  if constexpr (WF == 0) {
    const uint4* src = reinterpret_cast<const uint4*>(raw + r * 32u);
#pragma unroll
    for (int blk = 0; blk < 2; ++blk) {
      const uint4 w = src[blk];
      const uint32_t words[4] = {w.x, w.y, w.z, w.w};
      const uint32_t f = pow2_bf16x2(blk == 0 ? s0 : s1);
#pragma unroll
      for (int q = 0; q < 4; ++q) {       // 8 elements = one 16-byte chunk
        uint32_t o[4];
        e2m1x8_to_bf16(words[q], o);
        uint4 v;
        v.x = bf16x2_mul(o[0], f);
        v.y = bf16x2_mul(o[1], f);
        v.z = bf16x2_mul(o[2], f);
        v.w = bf16x2_mul(o[3], f);
        *reinterpret_cast<uint4*>(dst + swz(r, blk * 4 + q)) = v;
      }
    }
  } else {
    const uint4* src = reinterpret_cast<const uint4*>(raw + r * 64u);
#pragma unroll
    for (int q = 0; q < 4; ++q) {         // 16 bytes = 16 elements = two chunks
      const uint4 w = src[q];
      const uint32_t words[4] = {w.x, w.y, w.z, w.w};
      const uint32_t e = q < 2 ? s0 : s1;
      // W8: q * 2^(e - 133); MXFP8: E4M3 * 2^(e - 127).  Power-of-two FP32
      // scale (exact), then pack pairs to BF16 (exact: <= 8 significant bits).
      const float f = __uint_as_float(((WF == 1 ? e - 6u : e) & 0xFFu) << 23);
      uint32_t outw[8];
#pragma unroll
      for (int i = 0; i < 4; ++i) {
        float v[4];
#pragma unroll
        for (int j = 0; j < 4; ++j) {
          const uint32_t byte = (words[i] >> (8 * j)) & 0xFFu;
          if (WF == 1) {
            v[j] = (__int_as_float(0x4B400000 + static_cast<int32_t>(static_cast<int8_t>(byte))) -
                    12582912.0f) * f;
          } else {
            v[j] = static_cast<float>(e4m3_units(byte)) * 0.001953125f * f;
          }
        }
        outw[2 * i] = pack_bf16x2(v[0], v[1]);
        outw[2 * i + 1] = pack_bf16x2(v[2], v[3]);
      }
      *reinterpret_cast<uint4*>(dst + swz(r, 2 * q)) = make_uint4(outw[0], outw[1], outw[2], outw[3]);
      *reinterpret_cast<uint4*>(dst + swz(r, 2 * q + 1)) =
          make_uint4(outw[4], outw[5], outw[6], outw[7]);
    }
  }
}

template <uint32_t NT, uint32_t WF>
__global__ void __launch_bounds__(224, 1) k_gemm_tc(const __grid_constant__ TcParams p) {
  using Cfg = TcCfg<NT, WF>;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) &
                                             ~uintptr_t(1023));
  uint8_t* sA = smem;
  uint8_t* sW = smem + Cfg::kOffW;
  uint8_t* sRaw = smem + Cfg::kOffRaw;
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + Cfg::kOffBar);
  uint64_t* a_full = bars;                            // [kAStages] tile landed
  uint64_t* a_free = a_full + Cfg::kAStages;          // [kAStages] MMA done with it
  uint64_t* w_full = a_free + Cfg::kAStages;          // [kWStages] decoded (128 arrivals)
  uint64_t* w_free = w_full + Cfg::kWStages;          // [kWStages] MMA done with it
  uint64_t* raw_full = w_free + Cfg::kWStages;        // [kRaw] chunk landed
  uint64_t* raw_free = raw_full + Cfg::kRaw;          // [kRaw] chunk decoded (128 arrivals)
  uint64_t* acc_full = raw_free + Cfg::kRaw;          // accumulator complete
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(acc_full + 1);

  const TcJob& job = p.jobs != nullptr ? p.jobs[find_tc_job(p.jobs, p.njobs, blockIdx.x)]
                                       : p.inline_job;
  const uint32_t local = blockIdx.x - job.tile_begin;
  const uint32_t mt = local / job.n_tiles, nt = local % job.n_tiles;
  const uint32_t steps = job.k_steps;
  const uint32_t warp = threadIdx.x >> 5, lane = threadIdx.x & 31u;

  if (threadIdx.x == 0) {
    for (uint32_t s = 0; s < Cfg::kAStages; ++s) {
      mbar_init(&a_full[s], 1);
      mbar_init(&a_free[s], 1);
    }
    for (uint32_t s = 0; s < Cfg::kWStages; ++s) {
      mbar_init(&w_full[s], 128);
      mbar_init(&w_free[s], 1);
    }
    for (uint32_t s = 0; s < Cfg::kRaw; ++s) {
      mbar_init(&raw_full[s], 1);
      mbar_init(&raw_free[s], 128);
    }
    mbar_init(acc_full, 1);
    fence_barrier_init();
  }
  if (warp == 1) {
    tmem_alloc(tmem_slot, Cfg::kTmemCols);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;
  bool ok = true;

  if (warp == 0) {
    // Raw weight chunks, as far ahead as the raw ring allows.
    if (lane == 0) {
      const uint8_t* w_base = job.w_tiles + static_cast<size_t>(nt) * steps * Cfg::kChunk;
      for (uint32_t i = 0; i < steps && ok; ++i) {
        const uint32_t r = i % Cfg::kRaw;
        if (i >= Cfg::kRaw) ok = mbar_wait(&raw_free[r], ((i / Cfg::kRaw) - 1) & 1u, p.err);
        if (!ok) break;
        mbar_arrive_expect_tx(&raw_full[r], Cfg::kChunk);
        bulk_g2s(sRaw + r * Cfg::kRawStride, w_base + static_cast<size_t>(i) * Cfg::kChunk,
                 Cfg::kChunk, &raw_full[r]);
      }
      // Leave only after every copy issued here has landed.
      for (uint32_t i = (steps > Cfg::kRaw ? steps - Cfg::kRaw : 0); i < steps && ok; ++i) {
        ok = mbar_wait(&raw_full[i % Cfg::kRaw], (i / Cfg::kRaw) & 1u, p.err);
      }
    }
  } else if (warp == 2) {
    // Activation tiles, as far ahead as the A ring allows.
    if (lane == 0) {
      const uint8_t* a_base = job.a_tiles + static_cast<size_t>(mt) * steps * Cfg::kABytes;
      for (uint32_t i = 0; i < steps && ok; ++i) {
        const uint32_t s = i % Cfg::kAStages;
        if (i >= Cfg::kAStages) ok = mbar_wait(&a_free[s], ((i / Cfg::kAStages) - 1) & 1u, p.err);
        if (!ok) break;
        mbar_arrive_expect_tx(&a_full[s], Cfg::kABytes);
        bulk_g2s(sA + s * Cfg::kABytes, a_base + static_cast<size_t>(i) * Cfg::kABytes,
                 Cfg::kABytes, &a_full[s]);
      }
      for (uint32_t i = (steps > Cfg::kAStages ? steps - Cfg::kAStages : 0); i < steps && ok; ++i) {
        ok = mbar_wait(&a_full[i % Cfg::kAStages], (i / Cfg::kAStages) & 1u, p.err);
      }
    }
  } else if (warp == 1) {
    // MMA issuer.
    if (lane == 0) {
      const uint32_t idesc = idesc_bf16(kTileW, NT);
      for (uint32_t i = 0; i < steps && ok; ++i) {
        const uint32_t sa = i % Cfg::kAStages, sw = i % Cfg::kWStages;
        ok = mbar_wait(&a_full[sa], (i / Cfg::kAStages) & 1u, p.err) &&
             mbar_wait(&w_full[sw], (i / Cfg::kWStages) & 1u, p.err);
        if (!ok) break;
        tc_fence_after();
        const uint32_t a_addr = smem_addr(sW + sw * Cfg::kWBytes);
        const uint32_t b_addr = smem_addr(sA + sa * Cfg::kABytes);
#pragma unroll
        for (uint32_t k = 0; k < kStepK / 16; ++k) {
          mma_bf16(tmem, desc_sw128(a_addr + k * 32u), desc_sw128(b_addr + k * 32u), idesc,
                   (i > 0 || k > 0) ? 1u : 0u);
        }
        mma_commit(&a_free[sa]);
        mma_commit(&w_free[sw]);
      }
      mma_commit(acc_full);
    }
  } else {
    // Decoders: thread d expands weight row d of every step.
    const uint32_t d = threadIdx.x - 96u;
    for (uint32_t i = 0; i < steps && ok; ++i) {
      const uint32_t sw = i % Cfg::kWStages, r = i % Cfg::kRaw;
      if (i >= Cfg::kWStages) ok = mbar_wait(&w_free[sw], ((i / Cfg::kWStages) - 1) & 1u, p.err);
      ok = ok && mbar_wait(&raw_full[r], (i / Cfg::kRaw) & 1u, p.err);
      if (!ok) break;
      decode_row<WF>(sRaw + r * Cfg::kRawStride, d, sW + sw * Cfg::kWBytes);
      fence_proxy_async_smem();
      mbar_arrive(&raw_free[r]);
      mbar_arrive(&w_full[sw]);
    }
    // Epilogue: D[column][token] -> C[token][column].
    if (ok) ok = mbar_wait(acc_full, 0, p.err);
    ok = __all_sync(0xFFFFFFFFu, ok);   // tcgen05.ld needs the whole warp
    tc_fence_after();
    if (ok) {
      // Job fields in registers: stores to C could alias the job in global
      // memory and would force reloads after every store.
      const uint32_t M = job.M, N = job.N, ldc = job.ldc, acc_in = job.accumulate;
      const float* bias_p = job.bias;
      const uint32_t sp = warp & 3u;                      // TMEM subpartition of this warp
      const uint32_t col = nt * kTileW + sp * 32u + lane; // output column of this thread
      const bool col_ok = col < N;
      const float bias = (bias_p != nullptr && col_ok) ? bias_p[col] : 0.0f;
      const uint32_t row0 = mt * NT;
      float* cbase = job.c + static_cast<size_t>(row0) * ldc + col;
#pragma unroll 1
      for (uint32_t j0 = 0; j0 < NT; j0 += 16) {
        uint32_t v[16];
        tmem_ld16(tmem + ((sp * 32u) << 16) + j0, v);
        tmem_wait_ld();
#pragma unroll
        for (uint32_t j = 0; j < 16; ++j) {
          if (col_ok && row0 + j0 + j < M) {
            float* dst = cbase + static_cast<size_t>(j0 + j) * ldc;
            float x = __uint_as_float(v[j]);
            if (acc_in) x += *dst;
            *dst = x + bias;
          }
        }
      }
    }
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem, Cfg::kTmemCols);
  }
}

// ---------------------------------------------------------------------------
// Operand preparation

// Dense weights -> chunks of 128 columns x 64 K (raw codes) + scales.
__global__ void k_tile_weights(const uint8_t* __restrict__ w, const uint8_t* __restrict__ ws,
                               uint32_t N, uint32_t kb, uint32_t wfmt, uint8_t* __restrict__ out) {
  const uint32_t rb = raw_row_bytes(wfmt);
  const uint32_t steps = (kb + 1) / 2;
  const uint32_t n_tiles = (N + kTileW - 1) / kTileW;
  const uint32_t cb = chunk_bytes(wfmt);
  const size_t row_bytes = wfmt == 0 ? size_t{kb} * 16u : size_t{kb} * 32u;
  const uint64_t total = static_cast<uint64_t>(n_tiles) * steps * cb;
  for (uint64_t i = blockIdx.x * static_cast<uint64_t>(blockDim.x) + threadIdx.x; i < total;
       i += static_cast<uint64_t>(gridDim.x) * blockDim.x) {
    const uint64_t chunk = i / cb;
    const uint32_t byte = static_cast<uint32_t>(i % cb);
    const uint32_t tile = static_cast<uint32_t>(chunk / steps), step = static_cast<uint32_t>(chunk % steps);
    uint8_t v = 0;
    if (byte < kTileW * rb) {
      const uint32_t r = byte / rb, off = byte % rb;
      const uint32_t n = tile * kTileW + r;
      const size_t src = static_cast<size_t>(step) * rb + off;
      if (n < N && src < row_bytes) v = w[static_cast<size_t>(n) * row_bytes + src];
    } else {
      const uint32_t e = byte - kTileW * rb;
      const uint32_t r = e / 2, blk = step * 2 + (e & 1u);
      const uint32_t n = tile * kTileW + r;
      v = (n < N && blk < kb) ? ws[static_cast<size_t>(n) * kb + blk] : 127;
    }
    out[i] = v;
  }
}

template <uint32_t NT, uint32_t WF>
int launch_one(const TcJob* jobs_dev, uint32_t njobs, const TcJob* inline_job, uint32_t tiles,
               uint32_t* err, cudaStream_t s) {
  using Cfg = TcCfg<NT, WF>;
  if (!set_smem_limit_once(reinterpret_cast<const void*>(k_gemm_tc<NT, WF>), Cfg::kSmem)) {
    return -1;
  }
  TcParams p{};
  p.jobs = jobs_dev;
  p.njobs = njobs;
  p.err = err;
  if (inline_job != nullptr) p.inline_job = *inline_job;
  k_gemm_tc<NT, WF><<<tiles, Cfg::kThreads, Cfg::kSmem, s>>>(p);
  return cudaPeekAtLastError() == cudaSuccess ? 1 : -1;
}

}  // namespace

bool set_smem_limit_once(const void* kernel, uint32_t bytes) {
  // The limit is a per-(kernel, device) attribute; the host call is not free
  // (it would sit between back-to-back launches), so it is made once.
  static std::mutex mu;
  static std::vector<std::tuple<const void*, int, uint32_t>> done;
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess) return false;
  std::lock_guard<std::mutex> lock(mu);
  for (const auto& d : done) {
    if (std::get<0>(d) == kernel && std::get<1>(d) == dev && std::get<2>(d) >= bytes) return true;
  }
  if (cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                           static_cast<int>(bytes)) != cudaSuccess) {
    return false;
  }
  done.emplace_back(kernel, dev, bytes);
  return true;
}

uint32_t tc_tokens_per_tile(uint32_t M) { return M <= 64 ? 64u : (M <= 128 ? 128u : 256u); }

uint32_t tc_k_steps(uint32_t kb) { return (kb + 1) / 2; }

size_t tc_weight_tile_bytes(uint32_t wfmt, uint32_t N, uint32_t kb) {
  return static_cast<size_t>((N + kTileW - 1) / kTileW) * tc_k_steps(kb) * chunk_bytes(wfmt);
}

size_t tc_act_tile_bytes(uint32_t M, uint32_t kb) {
  const uint32_t nt = tc_tokens_per_tile(M);
  return static_cast<size_t>((M + nt - 1) / nt) * tc_k_steps(kb) * nt * kRowBytes;
}

void launch_tile_weights(const uint8_t* w, const uint8_t* ws, uint32_t N, uint32_t kb,
                         uint32_t wfmt, uint8_t* out, cudaStream_t s) {
  const uint64_t total = tc_weight_tile_bytes(wfmt, N, kb);
  uint64_t grid = (total + 255) / 256;
  if (grid > 148u * 32u) grid = 148u * 32u;
  k_tile_weights<<<static_cast<unsigned>(grid ? grid : 1), 256, 0, s>>>(w, ws, N, kb, wfmt, out);
}

void tc_fill_job(TcJob& t, uint32_t wfmt, uint32_t M, uint32_t N, uint32_t kb) {
  t.wfmt = wfmt;
  t.M = M;
  t.N = N;
  t.kb = kb;
  t.k_steps = tc_k_steps(kb);
  t.n_tiles = (N + kTileW - 1) / kTileW;
  t.m_tiles = (M + tc_tokens_per_tile(M) - 1) / tc_tokens_per_tile(M);
}

int launch_tc_jobs(const TcJob* jobs_dev, uint32_t njobs, const TcJob* inline_job, uint32_t nt,
                   uint32_t wfmt, uint32_t tiles, uint32_t* err, cudaStream_t s) {
  if (tiles == 0) return 0;
  switch (nt * 4 + wfmt) {
    case 64 * 4 + 0: return launch_one<64, 0>(jobs_dev, njobs, inline_job, tiles, err, s);
    case 64 * 4 + 1: return launch_one<64, 1>(jobs_dev, njobs, inline_job, tiles, err, s);
    case 64 * 4 + 2: return launch_one<64, 2>(jobs_dev, njobs, inline_job, tiles, err, s);
    case 128 * 4 + 0: return launch_one<128, 0>(jobs_dev, njobs, inline_job, tiles, err, s);
    case 128 * 4 + 1: return launch_one<128, 1>(jobs_dev, njobs, inline_job, tiles, err, s);
    case 128 * 4 + 2: return launch_one<128, 2>(jobs_dev, njobs, inline_job, tiles, err, s);
    case 256 * 4 + 0: return launch_one<256, 0>(jobs_dev, njobs, inline_job, tiles, err, s);
    case 256 * 4 + 1: return launch_one<256, 1>(jobs_dev, njobs, inline_job, tiles, err, s);
    case 256 * 4 + 2: return launch_one<256, 2>(jobs_dev, njobs, inline_job, tiles, err, s);
  }
  return -1;
}

}  // namespace hrb
