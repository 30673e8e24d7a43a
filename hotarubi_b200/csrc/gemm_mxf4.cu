// Tensor-core GEMM for MXFP4 weights with hardware block scales:
// tcgen05.mma kind::mxf4.block_scale.scale_vec::2X (E2M1 x E2M1, one E8M0
// scale per 32 elements of K on each side, FP32 accumulation in TMEM).
//
// Exact operands without any CUDA-core decode:
//   * weights are the reference's own E2M1 codes and E8M0 scales
//     (tools/compiler/weights.cpp:39-70, tools/compiler/tensors.cpp:66-90);
//   * an MXINT8 activation q * 2^(e-6), |q| <= 128, is split into three
//     E2M1 digit planes, q = 64 d2 + 8 d1 + d0 with every digit an integer in
//     [-4, 4] (E2M1 holds 0..4 exactly); plane p carries the scale
//     2^(e - 6 + 3p).  The planes are stacked as 3 NT operand rows, so one
//     M = 128, N = 192 MMA per 64 elements of K multiplies a weight tile by
//     all three planes of 64 tokens (each plane row with its own scales) and
//     the epilogue adds the three FP32 partial sums.  The products are exact;
//     only the FP32 summation order differs from the reference's chain
//     (HRB_MODE_FAST).
//
// Data layout (all prepared once per plan or written by the encoder):
//   K runs in steps of 256 elements = one 128-byte row of packed E2M1 (element
//   2j in the low nibble of byte j), stored in the 128-byte swizzle (16-byte
//   chunk c of row r at c ^ (r % 8)) so a linear bulk copy lands in the shared
//   memory layout the MMA descriptors describe.
//   Weights: per (128-column tile, step) one 17 KB chunk: 128 rows x 128 B,
//   then two 512-byte scale chunks (blocks 0-3 and 4-7 of the step).
//   Activations: per (NT-row tile, step) the block of mx_act_block_bytes
//   (hrb_tc.cuh): 3 NT stacked plane rows, then their scale chunks.
//   A scale chunk covers 128 rows x 4 blocks in the order tcgen05.cp
//   .32x128b.warpx4 copies to TMEM: row i of 32, bytes 4j + s = scale of
//   row i + 32 j, block s.  In TMEM the chunk occupies 4 columns (column j
//   holds rows 32 j .. 32 j + 31), replicated in all four lane quarters; MMA
//   k (64 elements = blocks 2k, 2k+1) reads the chunks of group k / 2 at
//   byte 2 (k % 2) (the sf_id).
//
// One persistent CTA per SM walks output tiles (128 weight columns x NT
// tokens): warp 0 streams operand stages with bulk copies, warp 1 owns TMEM
// and issues scale copies and MMAs, warps 3..6 drain finished accumulators
// (for NT = 64 two TMEM accumulator buffers, so one tile's epilogue overlaps
// the next tile's MMAs).  Every wait is bounded.
#include <algorithm>
#include <cstdint>

#include "hrb_kernels.cuh"
#include "hrb_tc.cuh"
#include "sm100.cuh"

namespace hrb {
namespace {

using namespace sm100;

constexpr uint32_t kTileW = 128;       // weight columns per tile (MMA M)
constexpr uint32_t kStep = 256;        // K elements per step
constexpr uint32_t kRowB = 128;        // bytes per operand row per step
constexpr uint32_t kSfChunk = 512;     // 128 rows x 4 blocks
constexpr uint32_t kWChunk = kTileW * kRowB + 2 * kSfChunk;  // 17408

template <uint32_t NT>
struct MxCfg {
  static constexpr uint32_t kPlane = NT * kRowB;
  static constexpr uint32_t kParts = mx_parts(NT);               // 192-row MMAs per K slice
  static constexpr uint32_t kABlock = mx_act_block_bytes(NT);
  static constexpr uint32_t kStageBytes = kWChunk + kABlock;    // multiple of 1024
  static constexpr uint32_t kStages = NT == 64 ? 5u : 3u;
  // Accumulator buffers of 3 NT columns (one per stacked plane row); two for
  // NT = 64 so one tile's epilogue overlaps the next tile's MMAs.
  static constexpr uint32_t kDBufs = NT == 64 ? 2u : 1u;
  static constexpr uint32_t kDCols = 3 * NT;
  // TMEM columns: accumulators, weight scales (2 groups x 4), activation
  // scales (per part, 2 groups x 8).
  static constexpr uint32_t kColSfa = kDBufs * kDCols;
  static constexpr uint32_t kColSfb = kColSfa + 8;
  static constexpr uint32_t kTmemCols = 512;
  static_assert(kColSfb + 16 * kParts <= kTmemCols, "TMEM columns");
  static constexpr uint32_t kOffBar = kStages * kStageBytes;
  static constexpr uint32_t kSmem = kOffBar + 256 + 1024;
  static_assert(kStageBytes % 1024 == 0, "stage alignment");
  static_assert(kSmem <= 232448, "shared memory");
  static constexpr uint32_t kThreads = 224;
};

struct MxParams {
  const MxTile* tiles;  // device tiles, or null: the tiles of inline_job
  uint32_t total_tiles;
  uint32_t* err;
  TcJob inline_job;
};

__host__ __device__ inline MxTile make_tile(const TcJob& job, uint32_t nt, uint32_t local) {
  const uint32_t mt = local / job.n_tiles, n_tile = local % job.n_tiles;
  const uint32_t row0 = mt * nt, col0 = n_tile * kTileW;
  MxTile t;
  t.w = job.w_tiles + static_cast<size_t>(n_tile) * job.k_steps * kWChunk;
  t.a = job.a_tiles + static_cast<size_t>(mt) * job.k_steps * mx_act_block_bytes(nt);
  t.c = job.c + static_cast<size_t>(row0) * job.ldc + col0;
  t.bias = job.bias != nullptr ? job.bias + col0 : nullptr;
  t.rows = job.M - row0 < nt ? job.M - row0 : nt;
  t.cols = job.N - col0 < kTileW ? job.N - col0 : kTileW;
  t.ldc = job.ldc;
  t.steps_acc = job.k_steps | (job.accumulate ? 0x80000000u : 0u);
  return t;
}

template <uint32_t NT>
__device__ __forceinline__ MxTile tile_info(const MxParams& p, uint32_t tile) {
  if (p.tiles == nullptr) return make_tile(p.inline_job, NT, tile);
  // Three independent 16-byte loads; nothing consumes them until the tile
  // is reached.
  const uint4* src = reinterpret_cast<const uint4*>(p.tiles + tile);
  const uint4 x = __ldg(src), y = __ldg(src + 1), z = __ldg(src + 2);
  MxTile t;
  t.w = reinterpret_cast<const uint8_t*>((static_cast<uint64_t>(x.y) << 32) | x.x);
  t.a = reinterpret_cast<const uint8_t*>((static_cast<uint64_t>(x.w) << 32) | x.z);
  t.c = reinterpret_cast<float*>((static_cast<uint64_t>(y.y) << 32) | y.x);
  t.bias = reinterpret_cast<const float*>((static_cast<uint64_t>(y.w) << 32) | y.z);
  t.rows = z.x;
  t.cols = z.y;
  t.ldc = z.z;
  t.steps_acc = z.w;
  return t;
}

// Instruction descriptor of kind::mxf4 block-scaled (E2M1 x E2M1, E8M0
// scales): A/B format 1 at [7,10)/[10,13), B scale id [4,6), N >> 3 at
// [17,23), scale format E8M0 at bit 23, M >> 4 at [24,29), A scale id [29,31).
__device__ __forceinline__ uint32_t idesc_mxf4(uint32_t m, uint32_t n, uint32_t sf_id) {
  return (sf_id << 4) | (1u << 7) | (1u << 10) | ((n >> 3) << 17) | (1u << 23) |
         ((m >> 4) << 24) | (sf_id << 29);
}

__device__ __forceinline__ void mma_mxf4(uint32_t d_tmem, uint64_t a_desc, uint64_t b_desc,
                                         uint32_t idesc, uint32_t sfa, uint32_t sfb,
                                         uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %6, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::mxf4.block_scale.scale_vec::2X [%0], %1, %2, %3, [%4], [%5], p;\n\t}"
      ::"r"(d_tmem), "l"(a_desc), "l"(b_desc), "r"(idesc), "r"(sfa), "r"(sfb), "r"(accumulate)
      : "memory");
}

// Shared-memory descriptor of one 512-byte scale chunk for tcgen05.cp
// .32x128b: 32 rows of 16 bytes, no swizzle, 8-row core matrices 128 bytes
// apart.
__device__ __forceinline__ uint64_t desc_sf_chunk(uint32_t smem_byte_addr) {
  uint64_t d = 0;
  d |= static_cast<uint64_t>((smem_byte_addr >> 4) & 0x3FFFu);
  d |= static_cast<uint64_t>(1u) << 16;
  d |= static_cast<uint64_t>(128u >> 4) << 32;
  d |= static_cast<uint64_t>(1u) << 46;
  return d;
}

__device__ __forceinline__ void sf_copy(uint32_t taddr, uint64_t desc) {
  asm volatile("tcgen05.cp.cta_group::1.32x128b.warpx4 [%0], %1;" ::"r"(taddr), "l"(desc)
               : "memory");
}

template <uint32_t NT>
__global__ void __launch_bounds__(224, 1) k_gemm_mxf4(const __grid_constant__ MxParams p) {
  using Cfg = MxCfg<NT>;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) &
                                             ~uintptr_t(1023));
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + Cfg::kOffBar);
  uint64_t* full = bars;                           // [kStages] stage landed
  uint64_t* empty = full + Cfg::kStages;           // [kStages] MMAs done with the stage
  uint64_t* acc_full = empty + Cfg::kStages;       // [kDBufs] accumulator ready
  uint64_t* acc_empty = acc_full + Cfg::kDBufs;    // [kDBufs] drained (128 arrivals)
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(acc_empty + Cfg::kDBufs);
  const uint32_t warp = threadIdx.x >> 5, lane = threadIdx.x & 31u;

  if (threadIdx.x == 0) {
    for (uint32_t s = 0; s < Cfg::kStages; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 1);
    }
    for (uint32_t b = 0; b < Cfg::kDBufs; ++b) {
      mbar_init(&acc_full[b], 1);
      mbar_init(&acc_empty[b], 128);
    }
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
    if (lane == 0) {
      uint32_t g = 0;  // global step counter across this CTA's tiles
      // Each tile's job fields are loaded one tile ahead, so their global
      // memory latency overlaps the previous tile's copies.
      MxTile next = tile_info<NT>(p, blockIdx.x);
      for (uint32_t tile = blockIdx.x; tile < p.total_tiles && ok; tile += gridDim.x) {
        const MxTile ti = next;
        if (tile + gridDim.x < p.total_tiles) next = tile_info<NT>(p, tile + gridDim.x);
        const uint8_t* wsrc = ti.w;
        const uint8_t* asrc = ti.a;
        const uint32_t k_steps = ti.steps_acc & 0x7FFFFFFFu;
        for (uint32_t i = 0; i < k_steps && ok; ++i, ++g) {
          const uint32_t s = g % Cfg::kStages;
          if (g >= Cfg::kStages) ok = mbar_wait(&empty[s], ((g / Cfg::kStages) - 1) & 1u, p.err);
          if (!ok) break;
          uint8_t* st = smem + s * Cfg::kStageBytes;
          mbar_arrive_expect_tx(&full[s], Cfg::kStageBytes);
          bulk_g2s(st, wsrc + static_cast<size_t>(i) * kWChunk, kWChunk, &full[s]);
          bulk_g2s(st + kWChunk, asrc + static_cast<size_t>(i) * Cfg::kABlock, Cfg::kABlock,
                   &full[s]);
        }
      }
      // Drain: every issued copy has landed before this thread leaves.
      for (uint32_t k = (g > Cfg::kStages ? g - Cfg::kStages : 0); k < g && ok; ++k) {
        ok = mbar_wait(&full[k % Cfg::kStages], (k / Cfg::kStages) & 1u, p.err);
      }
    }
  } else if (warp == 1) {
    if (lane == 0) {
      uint32_t g = 0, t = 0;
      const uint32_t sfa = tmem + Cfg::kColSfa;
      uint32_t next_steps = tile_info<NT>(p, blockIdx.x).steps_acc & 0x7FFFFFFFu;
      for (uint32_t tile = blockIdx.x; tile < p.total_tiles && ok; tile += gridDim.x, ++t) {
        const uint32_t k_steps = next_steps;
        if (tile + gridDim.x < p.total_tiles) {
          next_steps = tile_info<NT>(p, tile + gridDim.x).steps_acc & 0x7FFFFFFFu;
        }
        const uint32_t b = t % Cfg::kDBufs;
        if (t >= Cfg::kDBufs) ok = mbar_wait(&acc_empty[b], ((t / Cfg::kDBufs) - 1) & 1u, p.err);
        if (!ok) break;
        tc_fence_after();
        const uint32_t d = tmem + b * Cfg::kDCols;
        for (uint32_t i = 0; i < k_steps && ok; ++i, ++g) {
          const uint32_t s = g % Cfg::kStages;
          ok = mbar_wait(&full[s], (g / Cfg::kStages) & 1u, p.err);
          if (!ok) break;
          tc_fence_after();
          const uint32_t st = smem_addr(smem + s * Cfg::kStageBytes);
          const uint32_t w_tile = st, w_sf = st + kTileW * kRowB;
          const uint32_t a_planes = st + kWChunk, a_sf = a_planes + 3 * Cfg::kPlane;
          // Scales of this step into TMEM (ordered before the MMAs below).
          sf_copy(sfa, desc_sf_chunk(w_sf));
          sf_copy(sfa + 4, desc_sf_chunk(w_sf + kSfChunk));
#pragma unroll
          for (uint32_t c = 0; c < 4 * Cfg::kParts; ++c) {
            // chunk c = (part * 2 + group) * 2 + half -> columns 8 (part * 2 + group) + 4 half
            sf_copy(tmem + Cfg::kColSfb + 4 * c, desc_sf_chunk(a_sf + c * kSfChunk));
          }
#pragma unroll
          for (uint32_t k = 0; k < 4; ++k) {
            const uint32_t grp = k / 2, sf_id = (k % 2) * 2;
            const uint32_t idesc = idesc_mxf4(kTileW, 192, sf_id);
            const uint32_t sfa_k = (sfa + 4 * grp) | (sf_id << 30);
#pragma unroll
            for (uint32_t part = 0; part < Cfg::kParts; ++part) {
              const uint32_t sfb_k = (tmem + Cfg::kColSfb + 8 * (part * 2 + grp)) | (sf_id << 30);
              mma_mxf4(d + 192 * part, desc_sw128(w_tile + 32 * k),
                       desc_sw128(a_planes + part * 192 * kRowB + 32 * k), idesc, sfa_k, sfb_k,
                       (i > 0 || k > 0) ? 1u : 0u);
            }
          }
          mma_commit(&empty[s]);
        }
        mma_commit(&acc_full[b]);
      }
    }
  } else if (warp >= 3) {
    const uint32_t sp = warp & 3u;
    uint32_t t = 0;
    MxTile next = tile_info<NT>(p, blockIdx.x);
    for (uint32_t tile = blockIdx.x; tile < p.total_tiles; tile += gridDim.x, ++t) {
      const MxTile ti = next;
      if (tile + gridDim.x < p.total_tiles) next = tile_info<NT>(p, tile + gridDim.x);
      const uint32_t b = t % Cfg::kDBufs;
      if (ok) ok = mbar_wait(&acc_full[b], (t / Cfg::kDBufs) & 1u, p.err);
      ok = __all_sync(0xFFFFFFFFu, ok);
      if (!ok) break;
      tc_fence_after();
      const uint32_t col = sp * 32u + lane;
      const bool col_ok = col < ti.cols;
      const bool acc = (ti.steps_acc >> 31) != 0;
      const float bias = (ti.bias != nullptr && col_ok) ? ti.bias[col] : 0.0f;
      float* cbase = ti.c + col;
#pragma unroll 1
      for (uint32_t j0 = 0; j0 < NT; j0 += 16) {
        // The three digit-plane partial sums of tokens j0..j0+15, added
        // smallest scale first.
        uint32_t v0[16], v1[16], v2[16];
        const uint32_t taddr = tmem + ((sp * 32u) << 16) + b * Cfg::kDCols + j0;
        tmem_ld16(taddr, v0);
        tmem_ld16(taddr + NT, v1);
        tmem_ld16(taddr + 2 * NT, v2);
        tmem_wait_ld();
#pragma unroll
        for (uint32_t j = 0; j < 16; ++j) {
          if (col_ok && j0 + j < ti.rows) {
            float* dst = cbase + static_cast<size_t>(j0 + j) * ti.ldc;
            float x = (__uint_as_float(v0[j]) + __uint_as_float(v1[j])) + __uint_as_float(v2[j]);
            if (acc) x += *dst;
            *dst = x + bias;
          }
        }
      }
      tc_fence_before();
      mbar_arrive(&acc_empty[b]);
    }
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem, Cfg::kTmemCols);
  }
}

// Dense MXFP4 weights [N][kp/2] + scales [N][kb] -> the per-(tile, step)
// chunks above.  One thread per 16-byte output piece.
__global__ void k_tile_weights_mxf4(const uint8_t* __restrict__ w, const uint8_t* __restrict__ ws,
                                    uint32_t N, uint32_t kb, uint32_t steps,
                                    uint8_t* __restrict__ out) {
  const uint32_t n_tiles = (N + kTileW - 1) / kTileW;
  const uint64_t pieces = static_cast<uint64_t>(n_tiles) * steps * (kWChunk / 16u);
  const size_t row_bytes = static_cast<size_t>(kb) * 16u;
  for (uint64_t i = blockIdx.x * static_cast<uint64_t>(blockDim.x) + threadIdx.x; i < pieces;
       i += static_cast<uint64_t>(gridDim.x) * blockDim.x) {
    const uint64_t chunk = i / (kWChunk / 16u);
    const uint32_t piece = static_cast<uint32_t>(i % (kWChunk / 16u));
    const uint32_t tile = static_cast<uint32_t>(chunk / steps), step = static_cast<uint32_t>(chunk % steps);
    uint8_t v[16];
    if (piece < kTileW * kRowB / 16u) {
      // Row r, stored 16-byte chunk p holds logical chunk c = p ^ (r % 8):
      // bytes 16c .. 16c+15 of the step's 128-byte row = elements 32c .. 32c+31.
      const uint32_t r = piece / 8u, pc = piece % 8u, c = pc ^ (r & 7u);
      const uint32_t n = tile * kTileW + r;
      const size_t src = static_cast<size_t>(step) * kRowB + c * 16u;
#pragma unroll
      for (int k = 0; k < 16; ++k) {
        v[k] = (n < N && src + k < row_bytes) ? w[static_cast<size_t>(n) * row_bytes + src + k] : 0;
      }
    } else {
      // Scale chunk grp, bytes 16i .. 16i+15: bytes 4j + s = scale of row
      // i + 32 j, block 8 step + 4 grp + s.
      const uint32_t sp = piece - kTileW * kRowB / 16u;
      const uint32_t grp = sp / 32u, i32 = sp % 32u;
#pragma unroll
      for (int k = 0; k < 16; ++k) {
        const uint32_t j = k / 4, s = k % 4;
        const uint32_t n = tile * kTileW + i32 + 32u * j;
        const uint32_t blk = step * 8u + grp * 4u + s;
        v[k] = (n < N && blk < kb) ? ws[static_cast<size_t>(n) * kb + blk] : 127;
      }
    }
    uint4 o;
    o.x = v[0] | (v[1] << 8) | (v[2] << 16) | (static_cast<uint32_t>(v[3]) << 24);
    o.y = v[4] | (v[5] << 8) | (v[6] << 16) | (static_cast<uint32_t>(v[7]) << 24);
    o.z = v[8] | (v[9] << 8) | (v[10] << 16) | (static_cast<uint32_t>(v[11]) << 24);
    o.w = v[12] | (v[13] << 8) | (v[14] << 16) | (static_cast<uint32_t>(v[15]) << 24);
    reinterpret_cast<uint4*>(out)[i] = o;
  }
}

template <uint32_t NT>
int launch_mx(const MxTile* tiles_dev, const TcJob* inline_job, uint32_t tiles, int sm_count,
              uint32_t* err, cudaStream_t s) {
  using Cfg = MxCfg<NT>;
  if (!set_smem_limit_once(reinterpret_cast<const void*>(k_gemm_mxf4<NT>), Cfg::kSmem)) {
    return -1;
  }
  MxParams p{};
  p.tiles = tiles_dev;
  p.total_tiles = tiles;
  p.err = err;
  if (inline_job != nullptr) p.inline_job = *inline_job;
  const uint32_t grid = std::min<uint32_t>(tiles, static_cast<uint32_t>(sm_count));
  k_gemm_mxf4<NT><<<grid, Cfg::kThreads, Cfg::kSmem, s>>>(p);
  return cudaPeekAtLastError() == cudaSuccess ? 1 : -1;
}

}  // namespace

uint32_t mx_tokens_per_tile(uint32_t M) { return M <= 64 ? 64u : 128u; }

uint32_t mx_k_steps(uint32_t kb) { return (kb + 7) / 8; }

size_t mx_weight_bytes(uint32_t N, uint32_t kb) {
  return static_cast<size_t>((N + kTileW - 1) / kTileW) * mx_k_steps(kb) * kWChunk;
}

size_t mx_act_bytes(uint32_t M, uint32_t kb) {
  const uint32_t nt = mx_tokens_per_tile(M);
  return static_cast<size_t>((M + nt - 1) / nt) * mx_k_steps(kb) * mx_act_block_bytes(nt);
}

void launch_tile_weights_mxf4(const uint8_t* w, const uint8_t* ws, uint32_t N, uint32_t kb,
                              uint8_t* out, cudaStream_t s) {
  const uint64_t pieces = mx_weight_bytes(N, kb) / 16u;
  uint64_t grid = (pieces + 255) / 256;
  if (grid > 148u * 16u) grid = 148u * 16u;
  k_tile_weights_mxf4<<<static_cast<unsigned>(grid ? grid : 1), 256, 0, s>>>(w, ws, N, kb,
                                                                           mx_k_steps(kb), out);
}

void mx_fill_tiles(const TcJob& job, uint32_t nt, MxTile* out) {
  for (uint32_t i = 0; i < job.m_tiles * job.n_tiles; ++i) out[i] = make_tile(job, nt, i);
}

int launch_mxf4(const MxTile* tiles_dev, const TcJob* inline_job, uint32_t nt, uint32_t tiles,
                int sm_count, uint32_t* err, cudaStream_t s) {
  if (tiles == 0) return 0;
  if (tiles_dev == nullptr && inline_job == nullptr) return -1;
  if (nt == 64) return launch_mx<64>(tiles_dev, inline_job, tiles, sm_count, err, s);
  if (nt == 128) return launch_mx<128>(tiles_dev, inline_job, tiles, sm_count, err, s);
  return -1;
}

}  // namespace hrb
