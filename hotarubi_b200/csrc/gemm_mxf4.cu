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
#include <cstdlib>
#include <cstdint>
#include <mutex>
#include <tuple>
#include <vector>

#include "hrb_kernels.cuh"
#include "hrb_quant.cuh"
#include "hrb_tc.cuh"
#include "sm100.cuh"

namespace hrb {
namespace {

using namespace sm100;

constexpr uint32_t kTileW = 128;       // weight columns per tile (MMA M)
constexpr uint32_t kRowB = 128;        // bytes per operand row per step
constexpr uint32_t kSfChunk = 512;     // 128 rows x 4 blocks
constexpr uint32_t kWChunk = kTileW * kRowB + 2 * kSfChunk;  // 17408
constexpr uint32_t kSmemLimit = 232448;

// NT tokens per tile; WP weight planes per step (1: MXFP4 or MXFP8 codes;
// 3: the E2M1 digit planes of W8 weights); KB the operand bits (4:
// kind::mxf4 with three E2M1 activation planes and 256-element steps; 8:
// kind::mxf8f6f4 with two E4M3 activation planes and 128-element steps).
//   WP = 1: one ring of stages, each a weight chunk and the activation block
//   of one K step, filled by one producer thread.
//   WP = 3: weights and activations stream through two rings of their own,
//   filled by two producer threads, so the weight stream (from HBM, three
//   chunks a step) runs several steps ahead of the activation blocks (L2).
template <uint32_t NT, uint32_t WP, uint32_t KB>
struct MxCfg {
  static constexpr bool kF8 = KB == 8;
  static constexpr bool kSplit = WP > 1;
  static constexpr uint32_t kPlane = NT * kRowB;
  static constexpr uint32_t kAPlanes = kF8 ? 2u : 3u;            // activation digit planes
  static constexpr uint32_t kPartRows = kF8 ? 2u * NT : 192u;    // stacked rows per MMA (N)
  static constexpr uint32_t kParts = kF8 ? 1u : mx_parts(NT);     // MMAs per K slice
  static constexpr uint32_t kABlock = kF8 ? mx8_act_block_bytes(NT) : mx_act_block_bytes(NT);
  static constexpr uint32_t kWSf = kF8 ? 1u : 2u;                 // weight scale chunks a step
  static constexpr uint32_t kASf = kF8 ? 2u * NT / 128u : 4u * kParts;  // activation chunks
  static constexpr uint32_t kASlots = kSplit ? (NT == 64 ? 3u : 2u) : 0u;
  static constexpr uint32_t kOffW = kASlots * kABlock;            // W ring after the A ring
  // A slot of the W ring: one weight chunk, plus the step's activation block
  // when the rings are combined.
  static constexpr uint32_t kWSlot = kWChunk + (kSplit ? 0u : kABlock);
  // After the barriers, 512 bytes per epilogue warp to regroup outputs for
  // 16-byte stores, where that costs no ring slot (not for W8 at NT = 128,
  // whose weight ring would lose one).
  static constexpr uint32_t kStage = (NT == 128 && kSplit) ? 0u : 512u * (NT == 64 ? 8u : 16u);
  static constexpr uint32_t kWSlots = (kSmemLimit - 1024 - 512 - kStage - kOffW) / kWSlot;
  static_assert(kWSlots >= WP + 1, "weight ring");
  // Accumulator buffers of kAPlanes NT columns (one per stacked plane row);
  // two for NT = 64 so one tile's epilogue overlaps the next tile's MMAs.
  static constexpr uint32_t kDBufs = NT == 64 ? 2u : 1u;
  static constexpr uint32_t kDCols = kAPlanes * NT;
  // TMEM columns: accumulators, weight scales (4 per chunk per plane),
  // activation scales (4 per chunk).
  static constexpr uint32_t kColSfa = kDBufs * kDCols;
  static constexpr uint32_t kColSfb = kColSfa + 4 * kWSf * WP;
  static constexpr uint32_t kTmemCols = 512;
  static_assert(kColSfb + 4 * kASf <= kTmemCols, "TMEM columns");
  static constexpr uint32_t kOffBar = kOffW + kWSlots * kWSlot;
  static constexpr uint32_t kOffStage = kOffBar + 512;
  static constexpr uint32_t kSmem = kOffStage + kStage + 1024;
  static_assert(kABlock % 1024 == 0 && kWSlot % 1024 == 0, "ring alignment");
  static_assert(kSmem <= kSmemLimit, "shared memory");
  // Warps: 0 weight producer, 1 TMEM owner and MMA issuer, 2 activation
  // producer (split rings), then kEpiWarps epilogue warps: warp w drains TMEM
  // lane quarter w % 4, token rows of its share of the tile.  NT = 128 has a
  // single accumulator buffer, whose drain holds up the next tile's MMAs:
  // more warps drain it.
  static constexpr uint32_t kEpiWarps = NT == 64 ? 8u : 16u;
  static_assert(kStage == 0 || kStage == 512u * kEpiWarps, "a staging buffer per epilogue warp");
};

struct MxParams {
  const MxTile* tiles;  // device tiles, or null: the tiles of inline_job
  uint32_t total_tiles;
  uint32_t* err;
  MxPeers peers;        // outputs also stored at these byte offsets (peer GPUs)
  TcJob inline_job;
  MxGather gather;      // the gathering variant's source (convolutions)
  // The weight chunks were written and synchronised before this launch's
  // stream work began (plans translate them at creation): the weight stream
  // may start before griddep_wait, overlapping the kernel before.
  uint32_t weights_ready;
};

__host__ __device__ inline uint32_t mx_planes_of(uint32_t wfmt) {
  return wfmt == HRB_WFMT_W8 ? 3u : 1u;
}

// Weight bytes of one (tile, K step) and activation block bytes of a path
// format.
__host__ __device__ inline uint32_t w_step_bytes(uint32_t wfmt) {
  return wfmt == kTcW8Bf16 ? kMxRawChunk : mx_planes_of(wfmt) * kWChunk;
}

__host__ __device__ inline uint32_t act_block_bytes(uint32_t wfmt, uint32_t nt) {
  return wfmt == HRB_WFMT_MXFP8 ? mx8_act_block_bytes(nt)
         : wfmt == kTcW8Bf16    ? mxbf_act_block_bytes(nt)
                                : mx_act_block_bytes(nt);
}

__host__ __device__ inline MxTile make_tile(const TcJob& job, uint32_t nt, uint32_t local) {
  const uint32_t mt = local / job.n_tiles, n_tile = local % job.n_tiles;
  const uint32_t row0 = mt * nt, col0 = n_tile * kTileW;
  MxTile t;
  t.w = job.w_tiles + static_cast<size_t>(n_tile) * job.k_steps * w_step_bytes(job.wfmt);
  t.a = job.a_tiles + static_cast<size_t>(mt) * job.k_steps * act_block_bytes(job.wfmt, nt);
  t.c = job.c != nullptr ? job.c + static_cast<size_t>(row0) * job.ldc + col0 : nullptr;
  t.bias = job.epv != nullptr ? job.epv + 2u * col0 : (job.bias != nullptr ? job.bias + col0 : nullptr);
  // Blocks per row of the MXINT8 copy.
  const uint32_t kbq = job.ldcq != 0 ? job.ldcq / 32u : (job.N + 31u) / 32u;
  t.cq = job.cq != nullptr ? job.cq + static_cast<size_t>(row0) * kbq * 32u + col0 : nullptr;
  t.cscale = job.cq != nullptr ? job.cscale + static_cast<size_t>(row0) * kbq + col0 / 32u
                               : nullptr;
  t.rows = job.M - row0 < nt ? job.M - row0 : nt;
  t.cols_kbq = (job.N - col0 < kTileW ? job.N - col0 : kTileW) | (kbq << 8);
  t.ldc = job.ldc;
  t.flags = job.k_steps | (job.epv != nullptr ? 0x10000000u : 0u) | (job.relu ? 0x20000000u : 0u) |
            (job.cquant == HRB_QUANT_VEC ? 0x40000000u : 0u) | (job.accumulate ? 0x80000000u : 0u);
  return t;
}

template <uint32_t NT>
__device__ __forceinline__ MxTile tile_info(const MxParams& p, uint32_t tile) {
  if (p.tiles == nullptr) return make_tile(p.inline_job, NT, tile);
  // Four independent 16-byte loads; nothing consumes them until the tile
  // is reached.
  const uint4* src = reinterpret_cast<const uint4*>(p.tiles + tile);
  const uint4 x = __ldg(src), y = __ldg(src + 1), z = __ldg(src + 2), u = __ldg(src + 3);
  MxTile t;
  t.w = reinterpret_cast<const uint8_t*>((static_cast<uint64_t>(x.y) << 32) | x.x);
  t.a = reinterpret_cast<const uint8_t*>((static_cast<uint64_t>(x.w) << 32) | x.z);
  t.c = reinterpret_cast<float*>((static_cast<uint64_t>(y.y) << 32) | y.x);
  t.bias = reinterpret_cast<const float*>((static_cast<uint64_t>(y.w) << 32) | y.z);
  t.cq = reinterpret_cast<int8_t*>((static_cast<uint64_t>(z.y) << 32) | z.x);
  t.cscale = reinterpret_cast<uint8_t*>((static_cast<uint64_t>(z.w) << 32) | z.z);
  t.rows = u.x;
  t.cols_kbq = u.y;
  t.ldc = u.z;
  t.flags = u.w;
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

// Instruction descriptor of kind::mxf8f6f4 block-scaled with E4M3 A and B
// (format 0 at [7,10) and [10,13)) and E8M0 scales (bit 23), K = 32: B scale
// id [4,6), N >> 3 at [17,23), M >> 4 at [24,29), A scale id [29,31).
__device__ __forceinline__ uint32_t idesc_mxf8(uint32_t m, uint32_t n, uint32_t sf_id) {
  return (sf_id << 4) | ((n >> 3) << 17) | (1u << 23) | ((m >> 4) << 24) | (sf_id << 29);
}

__device__ __forceinline__ void mma_mxf8(uint32_t d_tmem, uint64_t a_desc, uint64_t b_desc,
                                         uint32_t idesc, uint32_t sfa, uint32_t sfb,
                                         uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %6, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::mxf8f6f4.block_scale.scale_vec::1X [%0], %1, %2, %3, [%4], [%5], p;\n\t}"
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

// The same for a CTA pair, issued by rank 0: each CTA's chunk at the
// descriptor's offset of its own shared memory into its own TMEM.
__device__ __forceinline__ void sf_copy_pair(uint32_t taddr, uint64_t desc) {
  asm volatile("tcgen05.cp.cta_group::2.32x128b.warpx4 [%0], %1;" ::"r"(taddr), "l"(desc)
               : "memory");
}

// kind::mxf4 MMA of a CTA pair (M = 256: rank 0's 128 rows of A, then rank
// 1's; B's rows half from each CTA), issued by rank 0.
__device__ __forceinline__ void mma_mxf4_pair(uint32_t d_tmem, uint64_t a_desc, uint64_t b_desc,
                                              uint32_t idesc, uint32_t sfa, uint32_t sfb,
                                              uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %6, 0;\n\t"
      "tcgen05.mma.cta_group::2.kind::mxf4.block_scale.scale_vec::2X [%0], %1, %2, %3, [%4], [%5], p;\n\t}"
      ::"r"(d_tmem), "l"(a_desc), "l"(b_desc), "r"(idesc), "r"(sfa), "r"(sfb), "r"(accumulate)
      : "memory");
}

// Global -> shared copies of 16 and 4 bytes that complete asynchronously;
// `bytes` of the source are read and the rest zero-filled (0: all zeros,
// the source is not read).
__device__ __forceinline__ void cp_async16(uint32_t dst, const void* src, uint32_t bytes) {
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;" ::"r"(dst), "l"(src), "r"(bytes)
               : "memory");
}
__device__ __forceinline__ void cp_async4(uint32_t dst, const void* src, uint32_t bytes) {
  asm volatile("cp.async.ca.shared.global [%0], [%1], 4, %2;" ::"r"(dst), "l"(src), "r"(bytes)
               : "memory");
}
// Arrives on the mbarrier once this thread's earlier cp.async copies have
// landed (the barrier's expected count includes this arrival).
__device__ __forceinline__ void cp_async_arrive(uint64_t* bar) {
  asm volatile("cp.async.mbarrier.arrive.noinc.shared::cta.b64 [%0];" ::"r"(smem_addr(bar))
               : "memory");
}
__device__ __forceinline__ void cp_async_wait_all() {
  asm volatile("cp.async.wait_all;" ::: "memory");
}

// The gathering variant's activation block of one K step (MXFP4, 256-channel
// planes, so a step is one (channel plane, tap) of the convolution): lane l
// copies, for tile rows l, l + 32 kWarps, ..., the step's three digit-plane rows
// (8 chunks of 16 bytes each, re-swizzled from the map's row to the tile's
// row) and their scale words from the encoded input map; rows outside the
// map or past M are zero-filled.
template <uint32_t NT, uint32_t kWarps>
__device__ __forceinline__ void gather_block(const MxGather& g, uint8_t* blk, uint32_t row0,
                                             uint32_t step, uint32_t lane) {
  const ConvGeom& geom = g.geom;
  const uint32_t taps = geom.kh * geom.kh;
  const uint32_t tap = step % taps, plane_in = step / taps;  // bp = 8: one map step
  const uint32_t map_nt = 1u << g.map_shift;
  const uint32_t dst0 = smem_addr(blk);
#pragma unroll 1
  for (uint32_t dr = lane; dr < NT; dr += 32u * kWarps) {
    const uint32_t row = row0 + dr;
    const int64_t src = row < g.rows ? conv_source_row(geom, row, tap) : -1;
    const uint32_t pos = src >= 0 ? static_cast<uint32_t>(src) : 0u;
    const uint32_t sr = pos & (map_nt - 1u);
    const uint8_t* sblk =
        g.map_tiles + (static_cast<size_t>(pos >> g.map_shift) * g.map_steps + plane_in) *
                          g.map_block_bytes;
    const uint32_t n16 = src >= 0 ? 16u : 0u, n4 = src >= 0 ? 4u : 0u;
#pragma unroll
    for (uint32_t p = 0; p < 3; ++p) {
      const uint8_t* srow = sblk + (p * map_nt + sr) * kRowB;
      const uint32_t drow = dst0 + (p * NT + dr) * kRowB;
#pragma unroll
      for (uint32_t c = 0; c < 8; ++c) {
        cp_async16(drow + ((c ^ (dr & 7u)) << 4), srow + ((c ^ (sr & 7u)) << 4), n16);
      }
#pragma unroll
      for (uint32_t h = 0; h < 2; ++h) {
        cp_async4(dst0 + mx_act_sf_offset(NT, p * NT + dr, 4u * h),
                  sblk + mx_act_sf_offset(map_nt, p * map_nt + sr, 4u * h), n4);
      }
    }
  }
}

// The MXINT8 copy of rows j0 .. j0 + 15 of this warp's output block (32
// columns, one per lane; columns past N count as zero): the block's key is a
// warp max, each lane encodes its element (QuantizeBlock / EncodeMxint8 rules,
// hrb_quant.cuh).  Non-finite values under the host rule set error bit 1.
// With peers, each byte also goes to every peer's copy (the fused
// all-gather of a sharded layer's MXINT8 output).
__device__ __forceinline__ void requant_rows(const MxTile& ti, const float (&x)[16], uint32_t j0,
                                             uint32_t sp, uint32_t lane, bool col_ok,
                                             uint32_t kbq, uint32_t* err, const MxPeers& peers) {
  const bool vec = ((ti.flags >> 30) & 1u) != 0;
  bool bad = false;
#pragma unroll
  for (uint32_t j = 0; j < 16; ++j) {
    if (j0 + j >= ti.rows) break;  // the same for the whole warp
    const uint32_t bits = col_ok ? __float_as_uint(x[j]) : 0u;
    const uint32_t mag = bits & 0x7FFFFFFFu;
    const uint32_t key = __reduce_max_sync(0xFFFFFFFFu, vec ? (mag >> 23) : mag);
    bad |= !vec && key >= 0x7F800000u;
    uint32_t scale;
    const int32_t q = mxint8_code(bits, key, vec, scale);
    const size_t row = j0 + j;
    int8_t* qd = ti.cq + row * kbq * 32u + sp * 32u + lane;
    uint8_t* sd = ti.cscale + row * kbq + sp;
    *qd = static_cast<int8_t>(q);
    if (lane == 0) *sd = static_cast<uint8_t>(scale);
    for (uint32_t r = 0; r < peers.count; ++r) {
      reinterpret_cast<int8_t*>(reinterpret_cast<char*>(qd) + peers.delta[r])[0] =
          static_cast<int8_t>(q);
      if (lane == 0) {
        reinterpret_cast<uint8_t*>(reinterpret_cast<char*>(sd) + peers.delta[r])[0] =
            static_cast<uint8_t>(scale);
      }
    }
  }
  if (bad && lane == 0) atomicOr(err, 1u);
}

// One epilogue warp's view of a finished tile: its 32 weight columns (TMEM
// lane quarter sp) with the tile's epilogue fields.  The accumulator holds
// kSums partial sums per output (the digit-plane products, at TMEM columns
// taddr, taddr + NT, taddr + 2 NT), added smallest scale first (load); then
// C (with accumulate), the column scale, the bias and RELU, and the stores:
// C, the peers' copies of C and the MXINT8 copy (finish).
//
// With `stage` (512 bytes of shared memory for this warp), a full chunk of
// 16 rows x 32 columns of an output without accumulate, C and the peers'
// copies 16-byte aligned, is regrouped through shared memory, four rows at a
// time, into 16-byte stores (local, then each peer): lane l writes row l / 8,
// columns 4 (l % 8) .. + 3.
template <uint32_t NT, uint32_t kSums>
struct TileDrain {
  const MxParams& p;
  const MxTile& ti;
  uint32_t taddr, sp, lane;
  float* stage;
  uint32_t col, cols, kbq, npeers;
  bool col_ok, acc, relu, scaled, requant, staged;
  float bias, scale;
  float* cbase;

  __device__ __forceinline__ TileDrain(const MxParams& p_, const MxTile& ti_, uint32_t taddr_,
                                       uint32_t sp_, uint32_t lane_, float* stage_)
      : p(p_), ti(ti_), taddr(taddr_), sp(sp_), lane(lane_), stage(stage_) {
    col = sp * 32u + lane;
    cols = ti.cols_kbq & 0xFFu;
    kbq = ti.cols_kbq >> 8;
    col_ok = col < cols;
    acc = (ti.flags >> 31) != 0;
    relu = ((ti.flags >> 29) & 1u) != 0;
    scaled = ((ti.flags >> 28) & 1u) != 0;
    bias = 0.0f;
    scale = 1.0f;
    if (ti.bias != nullptr && col_ok) {
      if (scaled) {
        const float2 sb = reinterpret_cast<const float2*>(ti.bias)[col];
        scale = sb.x;
        bias = sb.y;
      } else {
        bias = ti.bias[col];
      }
    }
    cbase = ti.c + col;
    npeers = p.peers.count;
    // The MXINT8 copy: this warp's 32 columns are one block of the next
    // layer's K (tiles start on 128-column boundaries); the block exists
    // when it starts before column N.
    requant = ti.cq != nullptr && sp * 32u < cols;
    // Peers' copies (the fused all-gather) take the same 16-byte stores when
    // every peer buffer sits at a 16-byte multiple from the local one.
    bool peers16 = true;
    for (uint32_t q = 0; q < npeers; ++q) peers16 &= (p.peers.delta[q] & 15) == 0;
    staged = stage != nullptr && !acc && peers16 && ti.c != nullptr && cols == kTileW &&
             (ti.ldc & 3u) == 0 && (reinterpret_cast<uintptr_t>(ti.c) & 15u) == 0;
  }

  // The plane sums of rows j0 .. j0 + 15 out of TMEM.
  __device__ __forceinline__ void load(uint32_t j0, float (&x)[16]) const {
    uint32_t v0[16], v1[16], v2[16];
    tmem_ld16(taddr + j0, v0);
    if constexpr (kSums > 1) tmem_ld16(taddr + NT + j0, v1);
    if constexpr (kSums > 2) tmem_ld16(taddr + 2 * NT + j0, v2);
    tmem_wait_ld();
#pragma unroll
    for (uint32_t j = 0; j < 16; ++j) {
      x[j] = __uint_as_float(v0[j]);
      if constexpr (kSums > 1) x[j] = x[j] + __uint_as_float(v1[j]);
      if constexpr (kSums > 2) x[j] += __uint_as_float(v2[j]);
    }
  }

  // Accumulate, scale, bias, RELU and the stores of rows j0 .. j0 + 15.
  __device__ __forceinline__ void finish(uint32_t j0, float (&x)[16]) const {
    if (staged && j0 + 16u <= ti.rows) {
#pragma unroll
      for (uint32_t j = 0; j < 16; ++j) {
        if (scaled) x[j] = __fmul_rn(x[j], scale);
        x[j] = __fadd_rn(x[j], bias);
        if (relu) x[j] = x[j] > 0.0f ? x[j] : 0.0f;
      }
#pragma unroll
      for (uint32_t q = 0; q < 4; ++q) {
#pragma unroll
        for (uint32_t j = 0; j < 4; ++j) stage[j * 32u + lane] = x[4u * q + j];
        __syncwarp();
        const float4 v = reinterpret_cast<const float4*>(stage)[lane];
        __syncwarp();
        const size_t row = j0 + 4u * q + (lane >> 3);
        float* dst = ti.c + row * ti.ldc + sp * 32u + 4u * (lane & 7u);
        *reinterpret_cast<float4*>(dst) = v;
        for (uint32_t r = 0; r < npeers; ++r) {
          *reinterpret_cast<float4*>(reinterpret_cast<char*>(dst) + p.peers.delta[r]) = v;
        }
      }
      if (requant) requant_rows(ti, x, j0, sp, lane, col_ok, kbq, p.err, p.peers);
      return;
    }
    if (col_ok) {
#pragma unroll
      for (uint32_t j = 0; j < 16; ++j) {
        if (j0 + j < ti.rows) {
          if (acc) x[j] += cbase[static_cast<size_t>(j0 + j) * ti.ldc];
          if (scaled) x[j] = __fmul_rn(x[j], scale);
          x[j] = __fadd_rn(x[j], bias);
          if (relu) x[j] = x[j] > 0.0f ? x[j] : 0.0f;
          if (ti.c != nullptr) cbase[static_cast<size_t>(j0 + j) * ti.ldc] = x[j];
        }
      }
      if (npeers != 0 && ti.c != nullptr) {
        // The same outputs into each peer's C (NVLink stores); none when
        // the FP32 output is not kept (the MXINT8 copy alone is gathered).
        for (uint32_t q = 0; q < npeers; ++q) {
          char* peer = reinterpret_cast<char*>(cbase) + p.peers.delta[q];
#pragma unroll
          for (uint32_t j = 0; j < 16; ++j) {
            if (j0 + j < ti.rows) {
              *reinterpret_cast<float*>(peer + static_cast<size_t>(j0 + j) * ti.ldc * 4u) = x[j];
            }
          }
        }
      }
    }
    if (requant) requant_rows(ti, x, j0, sp, lane, col_ok, kbq, p.err, p.peers);
  }
};

// One epilogue warp's share of a finished tile: token rows [r0, r1) of the
// warp's 32 weight columns (TileDrain).  With `release` and 32 rows for this
// warp, both chunks are read out of TMEM first and the accumulator is
// released (an arrival on `release`) before the stores, so the next tile's
// MMAs overlap them; returns whether it was.
template <uint32_t NT, uint32_t kSums, bool kEarly = false>
__device__ __forceinline__ bool drain_tile(const MxParams& p, const MxTile& ti, uint32_t taddr,
                                           uint32_t r0, uint32_t r1, uint32_t sp, uint32_t lane,
                                           float* stage = nullptr, uint64_t* release = nullptr) {
  const TileDrain<NT, kSums> d(p, ti, taddr, sp, lane, stage);
  if constexpr (kEarly) {
    if (release != nullptr && r1 - r0 == 32u) {
      float xa[16], xb[16];
      d.load(r0, xa);
      d.load(r0 + 16u, xb);
      tc_fence_before();
      mbar_arrive(release);
      d.finish(r0, xa);
      d.finish(r0 + 16u, xb);
      return true;
    }
  }
#pragma unroll 1
  for (uint32_t j0 = r0; j0 < r1; j0 += 16) {
    float x[16];
    d.load(j0, x);
    d.finish(j0, x);
  }
  return false;
}

// A ring of `slots` buffers with full/empty mbarriers, walked by a running
// counter: slot = n % slots, phase parity = (n / slots) & 1.
struct Ring {
  uint64_t* full;
  uint64_t* empty;
  uint32_t slots;
};

// Producer side: waits until slot n is free (the consumer released the use
// of it `slots` ago), then arms its full barrier for `bytes`.
__device__ __forceinline__ bool ring_acquire(const Ring& r, uint32_t n, uint32_t bytes,
                                             uint32_t* err) {
  const uint32_t s = n % r.slots;
  if (n >= r.slots && !mbar_wait(&r.empty[s], ((n / r.slots) - 1) & 1u, err)) return false;
  mbar_arrive_expect_tx(&r.full[s], bytes);
  return true;
}

// Producer side, at the end: every copy it issued has landed.
__device__ __forceinline__ bool ring_drain(const Ring& r, uint32_t n, uint32_t* err) {
  bool ok = true;
  for (uint32_t k = (n > r.slots ? n - r.slots : 0); k < n && ok; ++k) {
    ok = mbar_wait(&r.full[k % r.slots], (k / r.slots) & 1u, err);
  }
  return ok;
}

// Warps of a launch: the role warps (0 producer, 1 MMA, 2 split-ring
// producer or, gathering, the first gathering warp), the extra gathering
// warps, then the epilogue warps.
constexpr uint32_t kGatherWarps = 2;
template <uint32_t NT, uint32_t WP, uint32_t KB, bool kGather>
struct MxWarps {
  static constexpr uint32_t kFirstEpi = kGather ? 2u + kGatherWarps : 3u;
  static constexpr uint32_t kThreads = 32u * (kFirstEpi + MxCfg<NT, WP, KB>::kEpiWarps);
};

// kEarly (NT = 128 launches with several tiles a CTA): the epilogue releases
// the single accumulator before its stores (drain_tile).
template <uint32_t NT, uint32_t WP, uint32_t KB, bool kGather, bool kEarly = false>
__global__ void __launch_bounds__(MxWarps<NT, WP, KB, kGather>::kThreads, 1)
    k_gemm_mxf4(const __grid_constant__ MxParams p) {
  static_assert(!kGather || (WP == 1 && KB == 4), "the gathering variant is MXFP4 only");
  constexpr uint32_t kFirstEpi = MxWarps<NT, WP, KB, kGather>::kFirstEpi;
  using Cfg = MxCfg<NT, WP, KB>;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) &
                                             ~uintptr_t(1023));
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + Cfg::kOffBar);
  const Ring aring{bars, bars + Cfg::kASlots, Cfg::kASlots};
  const Ring wring{bars + 2 * Cfg::kASlots, bars + 2 * Cfg::kASlots + Cfg::kWSlots, Cfg::kWSlots};
  uint64_t* acc_full = bars + 2 * (Cfg::kASlots + Cfg::kWSlots);  // [kDBufs] accumulator ready
  uint64_t* acc_empty = acc_full + Cfg::kDBufs;                    // [kDBufs] drained (128)
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(acc_empty + Cfg::kDBufs);
  uint8_t* abase = smem;
  uint8_t* wbase = smem + Cfg::kOffW;
  const uint32_t warp = threadIdx.x >> 5, lane = threadIdx.x & 31u;

  if (threadIdx.x == 0) {
    if constexpr (Cfg::kSplit) {
      for (uint32_t s = 0; s < Cfg::kASlots; ++s) {
        mbar_init(&aring.full[s], 1);
        mbar_init(&aring.empty[s], 1);
      }
    }
    for (uint32_t s = 0; s < Cfg::kWSlots; ++s) {
      // Gathering: the weight producer's arrival and one per gathering lane.
      mbar_init(&wring.full[s], kGather ? 1u + 32u * kGatherWarps : 1u);
      mbar_init(&wring.empty[s], 1);
    }
    for (uint32_t b = 0; b < Cfg::kDBufs; ++b) {
      mbar_init(&acc_full[b], 1);
      mbar_init(&acc_empty[b], 32 * Cfg::kEpiWarps);
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
  // Launch setup, barriers and TMEM overlap the kernel before; its outputs
  // (this kernel's activations) and its reads of C come before any access.
  // With ready weights the weight producer waits later (combined rings:
  // after issuing the weight halves of its first stages) or not at all
  // (split rings: it reads nothing else).
  griddep_launch_dependents();
  const bool early_weights = !kGather && p.weights_ready != 0 && warp == 0;
  if (!early_weights) griddep_wait();

  if (kGather && warp >= 2 && warp < 2 + kGatherWarps) {
    // Gathering lanes: the activation half of every ring slot, in the weight
    // producer's order, once the slot is free; gathering warp g takes every
    // kGatherWarps-th group of 32 tile rows.
    const TcJob& job = p.inline_job;
    uint32_t n = 0;
    for (uint32_t tile = blockIdx.x; tile < p.total_tiles && ok; tile += gridDim.x) {
      const uint32_t row0 = (tile / job.n_tiles) * NT;
      for (uint32_t i = 0; i < job.k_steps && ok; ++i, ++n) {
        const uint32_t sl = n % wring.slots;
        if (n >= wring.slots) ok = mbar_wait(&wring.empty[sl], ((n / wring.slots) - 1) & 1u, p.err);
        ok = __all_sync(0xFFFFFFFFu, ok);
        if (!ok) break;
        gather_block<NT, kGatherWarps>(p.gather, wbase + sl * Cfg::kWSlot + kWChunk, row0, i,
                                       lane + 32u * (warp - 2u));
        cp_async_arrive(&wring.full[sl]);
      }
    }
    cp_async_wait_all();
  } else if (warp == 0 || (Cfg::kSplit && warp == 2)) {
    // Warp 0 lane 0 streams weight chunks (and, with combined rings, the
    // activation blocks too); warp 2 lane 0 the activation blocks of split
    // rings.  Each tile's fields are loaded one tile ahead.
    if (lane == 0) {
      const bool weights = warp == 0;
      const Ring& ring = weights ? wring : aring;
      uint32_t n = 0;  // uses of the ring so far
      MxTile next = tile_info<NT>(p, blockIdx.x);
      for (uint32_t tile = blockIdx.x; tile < p.total_tiles && ok; tile += gridDim.x) {
        const MxTile ti = next;
        if (tile + gridDim.x < p.total_tiles) next = tile_info<NT>(p, tile + gridDim.x);
        const uint32_t k_steps = (ti.flags & 0x0FFFFFFFu);
        if (weights) {
          // Stages of the first tile whose weight half went out before the
          // dependency wait (combined rings with ready weights).
          uint32_t pre = 0;
          if (early_weights && !Cfg::kSplit && n == 0) {
            pre = k_steps * WP < ring.slots ? k_steps * WP : ring.slots;
            for (uint32_t c = 0; c < pre; ++c) {
              mbar_arrive_expect_tx(&ring.full[c], Cfg::kWSlot);
              bulk_g2s(wbase + c * Cfg::kWSlot, ti.w + static_cast<size_t>(c) * kWChunk, kWChunk,
                       &ring.full[c]);
            }
            griddep_wait();
          }
          for (uint32_t c = 0; c < k_steps * WP && ok; ++c, ++n) {
            const uint32_t sl = n % ring.slots;
            if (c >= pre) {
              ok = ring_acquire(ring, n, kGather ? kWChunk : Cfg::kWSlot, p.err);
              if (!ok) break;
              bulk_g2s(wbase + sl * Cfg::kWSlot, ti.w + static_cast<size_t>(c) * kWChunk, kWChunk,
                       &ring.full[sl]);
            }
            if (!Cfg::kSplit && !kGather) {
              bulk_g2s(wbase + sl * Cfg::kWSlot + kWChunk,
                       ti.a + static_cast<size_t>(c) * Cfg::kABlock, Cfg::kABlock,
                       &ring.full[sl]);
            }
          }
        } else {
          for (uint32_t i = 0; i < k_steps && ok; ++i, ++n) {
            ok = ring_acquire(ring, n, Cfg::kABlock, p.err);
            if (ok) {
              bulk_g2s(abase + (n % ring.slots) * Cfg::kABlock,
                       ti.a + static_cast<size_t>(i) * Cfg::kABlock, Cfg::kABlock,
                       &ring.full[n % ring.slots]);
            }
          }
        }
      }
      if (ok) ring_drain(ring, n, p.err);
    }
  } else if (warp == 1) {
    if (lane == 0) {
      uint32_t na = 0, nw = 0, t = 0;
      const uint32_t sfa = tmem + Cfg::kColSfa;
      uint32_t next_steps = tile_info<NT>(p, blockIdx.x).flags & 0x0FFFFFFFu;
      for (uint32_t tile = blockIdx.x; tile < p.total_tiles && ok; tile += gridDim.x, ++t) {
        const uint32_t k_steps = next_steps;
        if (tile + gridDim.x < p.total_tiles) {
          next_steps = tile_info<NT>(p, tile + gridDim.x).flags & 0x0FFFFFFFu;
        }
        const uint32_t b = t % Cfg::kDBufs;
        if (t >= Cfg::kDBufs) ok = mbar_wait(&acc_empty[b], ((t / Cfg::kDBufs) - 1) & 1u, p.err);
        if (!ok) break;
        tc_fence_after();
        const uint32_t d = tmem + b * Cfg::kDCols;
        for (uint32_t i = 0; i < k_steps && ok; ++i, ++na, nw += WP) {
          uint32_t as = 0;
          if constexpr (Cfg::kSplit) {
            as = na % Cfg::kASlots;
            ok = mbar_wait(&aring.full[as], (na / Cfg::kASlots) & 1u, p.err);
          }
#pragma unroll
          for (uint32_t pl = 0; pl < WP && ok; ++pl) {
            const uint32_t n = nw + pl;
            ok = mbar_wait(&wring.full[n % Cfg::kWSlots], (n / Cfg::kWSlots) & 1u, p.err);
          }
          if (!ok) break;
          tc_fence_after();
          // Gathered blocks were written through the generic proxy.
          if constexpr (kGather) fence_proxy_async_smem();
          const uint32_t a_planes =
              Cfg::kSplit ? smem_addr(abase + as * Cfg::kABlock)
                          : smem_addr(wbase + (nw % Cfg::kWSlots) * Cfg::kWSlot + kWChunk);
          const uint32_t a_sf = a_planes + Cfg::kAPlanes * Cfg::kPlane;
          uint32_t w_tile[WP];
          // Scales of this step into TMEM (ordered before the MMAs below).
#pragma unroll
          for (uint32_t pl = 0; pl < WP; ++pl) {
            w_tile[pl] = smem_addr(wbase + ((nw + pl) % Cfg::kWSlots) * Cfg::kWSlot);
            const uint32_t w_sf = w_tile[pl] + kTileW * kRowB;
#pragma unroll
            for (uint32_t c = 0; c < Cfg::kWSf; ++c) {
              sf_copy(sfa + 4 * Cfg::kWSf * pl + 4 * c, desc_sf_chunk(w_sf + c * kSfChunk));
            }
          }
#pragma unroll
          for (uint32_t c = 0; c < Cfg::kASf; ++c) {
            // E2M1: chunk c = (part * 2 + group) * 2 + half -> columns
            // 8 (part * 2 + group) + 4 half.  E4M3: chunk c (stacked rows
            // 128 c ..) -> columns 4 c.
            sf_copy(tmem + Cfg::kColSfb + 4 * c, desc_sf_chunk(a_sf + c * kSfChunk));
          }
#pragma unroll
          for (uint32_t k = 0; k < 4; ++k) {
            // E2M1: MMA k covers blocks 2k, 2k+1 (group k / 2, bytes 2 (k % 2)
            // of its columns); E4M3: block k (byte k).
            const uint32_t grp = Cfg::kF8 ? 0u : k / 2, sf_id = Cfg::kF8 ? k : (k % 2) * 2;
            const uint32_t idesc = Cfg::kF8 ? idesc_mxf8(kTileW, Cfg::kPartRows, sf_id)
                                            : idesc_mxf4(kTileW, Cfg::kPartRows, sf_id);
#pragma unroll
            for (uint32_t pl = 0; pl < WP; ++pl) {
              const uint32_t sfa_k = (sfa + 4 * Cfg::kWSf * pl + 4 * grp) | (sf_id << 30);
#pragma unroll
              for (uint32_t part = 0; part < Cfg::kParts; ++part) {
                const uint32_t sfb_k =
                    (tmem + Cfg::kColSfb + 8 * (part * 2 + grp)) | (sf_id << 30);
                const uint64_t wd = desc_sw128(w_tile[pl] + 32 * k);
                const uint64_t ad = desc_sw128(a_planes + part * Cfg::kPartRows * kRowB + 32 * k);
                const uint32_t acc = (i > 0 || k > 0 || pl > 0) ? 1u : 0u;
                if constexpr (Cfg::kF8) {
                  mma_mxf8(d + Cfg::kPartRows * part, wd, ad, idesc, sfa_k, sfb_k, acc);
                } else {
                  mma_mxf4(d + Cfg::kPartRows * part, wd, ad, idesc, sfa_k, sfb_k, acc);
                }
              }
            }
          }
          // Release the step's slots once these MMAs have read them.
#pragma unroll
          for (uint32_t pl = 0; pl < WP; ++pl) mma_commit(&wring.empty[(nw + pl) % Cfg::kWSlots]);
          if (Cfg::kSplit) mma_commit(&aring.empty[as]);
        }
        mma_commit(&acc_full[b]);
      }
    }
  } else if (warp >= kFirstEpi) {
    const uint32_t sp = warp & 3u;
    // Token rows [r0, r1) of each tile: the epilogue warps of a lane quarter
    // split the tile's rows.
    constexpr uint32_t kRowsPer = NT / (Cfg::kEpiWarps / 4);
    const uint32_t r0 = ((warp - kFirstEpi) / 4u) * kRowsPer, r1 = r0 + kRowsPer;
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
      // A single accumulator (NT = 128) is released as soon as it is read
      // when another tile follows.
      const bool more = tile + gridDim.x < p.total_tiles;
      const bool released = drain_tile<NT, Cfg::kAPlanes, kEarly>(
          p, ti, tmem + ((sp * 32u) << 16) + b * Cfg::kDCols, r0, r1, sp, lane,
          Cfg::kStage != 0 ? reinterpret_cast<float*>(smem + Cfg::kOffStage) + (warp - kFirstEpi) * 128u
                           : nullptr,
          Cfg::kDBufs == 1 && more ? &acc_empty[b] : nullptr);
      if (!released) {
        tc_fence_before();
        mbar_arrive(&acc_empty[b]);
      }
    }
    // Peer stores performed before the kernel is seen to finish.
    if (p.peers.count != 0) __threadfence_system();
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem, Cfg::kTmemCols);
  }
}

// ---------------------------------------------------------------------------
// MXFP4 on CTA pairs (tcgen05 .cta_group::2).
//
// The kernel above reads each activation block once per 128-column weight
// tile, so for the GEMMs of this path the operand traffic from L2 is
// dominated by activation re-reads (about 1.5 times the weight bytes at
// 64 tokens, 3 times at 4096), and that L2-to-SM stream, not HBM or the
// tensor pipe, sets the pace.  Here the two CTAs of a cluster take two
// adjacent column tiles of the same token tile and run them as one MMA of
// M = 256: each streams its own weight chunk but only half of the
// activation block's stacked plane rows (rows [96 r, 96 r + 96) of each
// 192-row part for rank r; the MMA takes B's rows half from each CTA), plus
// all the scale chunks (each CTA's TMEM needs the scales of every B row).
// Activation bytes from L2 halve; the epilogue is the same per CTA (its
// 128 weight columns x NT tokens in its own TMEM).
//
// Roles: warp 0 lane 0 of each CTA streams its stages into its own ring;
// warp 1 owns the pair's TMEM (allocated by both CTAs together); on rank 0
// lane 0 of warp 1 issues the scale copies and MMAs for both CTAs once both
// halves of a stage have landed (rank 1's warp 1 relays its stage
// completions to rank 0), and its commits free the stage in both CTAs and
// publish finished accumulators to both epilogues, which hand the
// accumulator back to rank 0.  Tiles go in pairs: p.tiles in pair order
// (tile 2u + rank of pair u; a dummy tile with no columns fills an odd
// column count), or the inline job's. Every wait is bounded; both CTAs meet
// at a cluster barrier before TMEM is freed.
template <uint32_t NT>
struct PairCfg {
  using Base = MxCfg<NT, 1, 4>;
  static constexpr uint32_t kParts = Base::kParts;              // 192-row MMA parts
  static constexpr uint32_t kHalf = Base::kPartRows / 2u;       // stacked rows a CTA a part
  static constexpr uint32_t kHalfBytes = kHalf * kRowB;         // 12 KB
  static constexpr uint32_t kSfBytes = kParts * 2048u;          // the block's scale chunks
  static constexpr uint32_t kABlock = mx_act_block_bytes(NT);   // the block in global memory
  static constexpr uint32_t kOffA = kWChunk;                    // in a slot: weights, halves, scales
  static constexpr uint32_t kOffSf = kOffA + kParts * kHalfBytes;
  static constexpr uint32_t kSlot = kOffSf + kSfBytes;
  static constexpr uint32_t kSlots = NT == 64 ? 7u : 4u;
  static constexpr uint32_t kOffBar = kSlots * kSlot;
  static constexpr uint32_t kStage = Base::kStage;
  static constexpr uint32_t kOffStage = kOffBar + 512;
  static constexpr uint32_t kSmem = kOffStage + kStage + 1024;
  static constexpr uint32_t kEpiWarps = Base::kEpiWarps;
  static constexpr uint32_t kFirstEpi = 3;
  static constexpr uint32_t kThreads = 32u * (kFirstEpi + kEpiWarps);
  static_assert(kSlot % 1024 == 0 && kOffA % 1024 == 0 && kHalfBytes % 1024 == 0, "alignment");
  static_assert(kSmem <= kSmemLimit, "shared memory");
};

__host__ __device__ inline MxTile dummy_tile(MxTile t) {
  t.c = nullptr;
  t.cq = nullptr;
  t.cscale = nullptr;
  t.cols_kbq &= ~0xFFu;
  t.flags &= ~0x80000000u;
  return t;
}

template <uint32_t NT>
__device__ __forceinline__ MxTile pair_tile(const MxParams& p, uint32_t u, uint32_t rank) {
  if (p.tiles != nullptr) return tile_info<NT>(p, 2u * u + rank);
  const TcJob& job = p.inline_job;
  const uint32_t np = (job.n_tiles + 1u) / 2u;
  const uint32_t mt = u / np, n = 2u * (u % np) + rank;
  return n < job.n_tiles ? make_tile(job, NT, mt * job.n_tiles + n)
                         : dummy_tile(make_tile(job, NT, mt * job.n_tiles + n - 1u));
}

template <uint32_t NT, bool kEarly>
__global__ void __launch_bounds__(PairCfg<NT>::kThreads, 1)
    k_gemm_mxf4_pair(const __grid_constant__ MxParams p) {
  using Cfg = PairCfg<NT>;
  using Base = typename Cfg::Base;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) &
                                             ~uintptr_t(1023));
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + Cfg::kOffBar);
  const Ring ring{bars, bars + Cfg::kSlots, Cfg::kSlots};
  uint64_t* peer_full = bars + 2 * Cfg::kSlots;        // rank 0: rank 1's stage landed
  uint64_t* acc_full = bars + 3 * Cfg::kSlots;         // [kDBufs]
  uint64_t* acc_empty = acc_full + Base::kDBufs;       // [kDBufs] rank 0: both epilogues done
  uint64_t* drained = acc_empty + Base::kDBufs;        // rank 0: every MMA complete
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(drained + 1);
  const uint32_t warp = threadIdx.x >> 5, lane = threadIdx.x & 31u;
  const uint32_t rank = cluster_rank();
  const uint32_t first = blockIdx.x >> 1, stride = gridDim.x >> 1;
  const uint32_t pairs = p.total_tiles >> 1;

  if (threadIdx.x == 0) {
    for (uint32_t s = 0; s < Cfg::kSlots; ++s) {
      mbar_init(&ring.full[s], 1);
      mbar_init(&ring.empty[s], 1);
      mbar_init(&peer_full[s], 1);
    }
    for (uint32_t b = 0; b < Base::kDBufs; ++b) {
      mbar_init(&acc_full[b], 1);
      mbar_init(&acc_empty[b], 2u * Cfg::kEpiWarps);
    }
    mbar_init(drained, 1);
    fence_barrier_init();
  }
  if (warp == 1) {
    tmem_alloc_pair(tmem_slot, Base::kTmemCols);
    tmem_relinquish_pair();
  }
  tc_fence_before();
  cluster_sync();  // barriers of both CTAs initialised, the pair's TMEM allocated
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;
  bool ok = true;
  griddep_launch_dependents();
  const bool early_weights = p.weights_ready != 0 && warp == 0;
  if (!early_weights) griddep_wait();

  if (warp == 0) {
    if (lane == 0) {
      uint32_t n = 0;
      MxTile next = pair_tile<NT>(p, first, rank);
      for (uint32_t u = first; u < pairs && ok; u += stride) {
        const MxTile ti = next;
        if (u + stride < pairs) next = pair_tile<NT>(p, u + stride, rank);
        const uint32_t k_steps = ti.flags & 0x0FFFFFFFu;
        uint32_t pre = 0;
        if (early_weights && n == 0) {
          pre = k_steps < Cfg::kSlots ? k_steps : Cfg::kSlots;
          for (uint32_t c = 0; c < pre; ++c) {
            mbar_arrive_expect_tx(&ring.full[c], Cfg::kSlot);
            bulk_g2s(smem + c * Cfg::kSlot, ti.w + static_cast<size_t>(c) * kWChunk, kWChunk,
                     &ring.full[c]);
          }
          griddep_wait();
        }
        for (uint32_t c = 0; c < k_steps && ok; ++c, ++n) {
          const uint32_t sl = n % Cfg::kSlots;
          uint8_t* slot = smem + sl * Cfg::kSlot;
          if (c >= pre) {
            ok = ring_acquire(ring, n, Cfg::kSlot, p.err);
            if (!ok) break;
            bulk_g2s(slot, ti.w + static_cast<size_t>(c) * kWChunk, kWChunk, &ring.full[sl]);
          }
          const uint8_t* blk = ti.a + static_cast<size_t>(c) * Cfg::kABlock;
#pragma unroll
          for (uint32_t part = 0; part < Cfg::kParts; ++part) {
            bulk_g2s(slot + Cfg::kOffA + part * Cfg::kHalfBytes,
                     blk + (part * Base::kPartRows + rank * Cfg::kHalf) * kRowB, Cfg::kHalfBytes,
                     &ring.full[sl]);
          }
          bulk_g2s(slot + Cfg::kOffSf, blk + 3u * NT * kRowB, Cfg::kSfBytes, &ring.full[sl]);
        }
      }
      if (ok) ring_drain(ring, n, p.err);
    }
  } else if (warp == 1 && rank == 1) {
    // Relay: each landed stage of this CTA, announced to rank 0.
    if (lane == 0) {
      uint32_t n = 0;
      for (uint32_t u = first; u < pairs && ok; u += stride) {
        const uint32_t k_steps = pair_tile<NT>(p, u, rank).flags & 0x0FFFFFFFu;
        for (uint32_t c = 0; c < k_steps && ok; ++c, ++n) {
          const uint32_t sl = n % Cfg::kSlots;
          ok = mbar_spin(&ring.full[sl], (n / Cfg::kSlots) & 1u, p.err);
          if (ok) mbar_arrive_cluster(&peer_full[sl], 0);
        }
      }
    }
  } else if (warp == 1) {
    if (lane == 0) {
      uint32_t n = 0, t = 0;
      const uint32_t sfa = tmem + Base::kColSfa;
      for (uint32_t u = first; u < pairs && ok; u += stride, ++t) {
        const uint32_t k_steps = pair_tile<NT>(p, u, 0).flags & 0x0FFFFFFFu;
        const uint32_t b = t % Base::kDBufs;
        if (t >= Base::kDBufs) {
          ok = mbar_wait_cluster(&acc_empty[b], ((t / Base::kDBufs) - 1) & 1u, p.err);
        }
        if (!ok) break;
        tc_fence_after();
        const uint32_t d = tmem + b * Base::kDCols;
        for (uint32_t i = 0; i < k_steps && ok; ++i, ++n) {
          const uint32_t sl = n % Cfg::kSlots, par = (n / Cfg::kSlots) & 1u;
          ok = mbar_wait(&ring.full[sl], par, p.err) && mbar_wait_cluster(&peer_full[sl], par, p.err);
          if (!ok) break;
          tc_fence_after();
          const uint32_t w_tile = smem_addr(smem + sl * Cfg::kSlot);
          const uint32_t a_half = w_tile + Cfg::kOffA;
          const uint32_t a_sf = w_tile + Cfg::kOffSf;
#pragma unroll
          for (uint32_t c = 0; c < 2; ++c) {
            sf_copy_pair(sfa + 4 * c, desc_sf_chunk(w_tile + kTileW * kRowB + c * kSfChunk));
          }
#pragma unroll
          for (uint32_t c = 0; c < Base::kASf; ++c) {
            sf_copy_pair(tmem + Base::kColSfb + 4 * c, desc_sf_chunk(a_sf + c * kSfChunk));
          }
#pragma unroll
          for (uint32_t k = 0; k < 4; ++k) {
            const uint32_t grp = k / 2, sf_id = (k % 2) * 2;
            const uint32_t idesc = idesc_mxf4(2u * kTileW, Base::kPartRows, sf_id);
#pragma unroll
            for (uint32_t part = 0; part < Cfg::kParts; ++part) {
              const uint32_t sfb_k = (tmem + Base::kColSfb + 8 * (part * 2 + grp)) | (sf_id << 30);
              mma_mxf4_pair(d + Base::kPartRows * part, desc_sw128(w_tile + 32 * k),
                            desc_sw128(a_half + part * Cfg::kHalfBytes + 32 * k), idesc,
                            (sfa + 4 * grp) | (sf_id << 30), sfb_k, (i > 0 || k > 0) ? 1u : 0u);
            }
          }
          mma_commit_pair(&ring.empty[sl]);  // the stage is free in both CTAs
        }
        if (ok) mma_commit_pair(&acc_full[b]);
      }
      // Every MMA issued has completed before the pair's TMEM is freed.
      asm volatile("tcgen05.commit.cta_group::2.mbarrier::arrive::one.shared::cluster.b64 [%0];"
                   ::"r"(smem_addr(drained))
                   : "memory");
      mbar_wait(drained, 0, p.err);
    }
  } else if (warp >= Cfg::kFirstEpi) {
    const uint32_t sp = warp & 3u;
    constexpr uint32_t kRowsPer = NT / (Cfg::kEpiWarps / 4);
    const uint32_t r0 = ((warp - Cfg::kFirstEpi) / 4u) * kRowsPer, r1 = r0 + kRowsPer;
    float* stage = Cfg::kStage != 0
                       ? reinterpret_cast<float*>(smem + Cfg::kOffStage) + (warp - Cfg::kFirstEpi) * 128u
                       : nullptr;
    uint32_t t = 0;
    for (uint32_t u = first; u < pairs; u += stride, ++t) {
      const MxTile ti = pair_tile<NT>(p, u, rank);
      const uint32_t b = t % Base::kDBufs;
      if (ok) ok = mbar_wait(&acc_full[b], (t / Base::kDBufs) & 1u, p.err);
      ok = __all_sync(0xFFFFFFFFu, ok);
      if (!ok) break;
      tc_fence_after();
      const TileDrain<NT, 3> dr(p, ti, tmem + ((sp * 32u) << 16) + b * Base::kDCols, sp, lane,
                                stage);
      const bool early = kEarly && Base::kDBufs == 1 && r1 - r0 == 32u;
      if (early) {
        // Both row chunks in registers, then the accumulator goes back.
        float xa[16], xb[16];
        dr.load(r0, xa);
        dr.load(r0 + 16u, xb);
        tc_fence_before();
        __syncwarp();
        if (lane == 0) mbar_arrive_cluster(&acc_empty[b], 0);
        dr.finish(r0, xa);
        dr.finish(r0 + 16u, xb);
      } else {
#pragma unroll 1
        for (uint32_t j0 = r0; j0 < r1; j0 += 16) {
          float x[16];
          dr.load(j0, x);
          dr.finish(j0, x);
        }
        tc_fence_before();
        __syncwarp();
        if (lane == 0) mbar_arrive_cluster(&acc_empty[b], 0);
      }
    }
    if (p.peers.count != 0) __threadfence_system();
  }
  __syncwarp();
  tc_fence_before();
  cluster_sync();  // both CTAs done: no more arrivals on rank 0's barriers, no MMA reads
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc_pair(tmem, Base::kTmemCols);
  }
}

// ---------------------------------------------------------------------------
// W8 with at most 64 tokens (path format kTcW8Bf16): kind::f16 on BF16.
//
// These GEMMs are bound by the weight stream, so the weights travel as the
// int8 codes themselves (one byte a weight, against 1.5 for the three E2M1
// digit planes) and converter warps turn each K step of a tile into BF16
// rows of the MMA's A operand, written straight into tensor memory (no
// shared-memory round trip for the converted weights); one M = 128, N = 64,
// K = 16 MMA per 16 elements of K then multiplies them by the BF16
// activations from shared memory, one product per weight instead of nine
// digit-plane products.
//
// Warps: 0 streams raw weight chunks and 2 activation blocks (bulk copies
// into two rings, so neither waits on the other's consumers), 1 owns TMEM
// and issues the MMAs, 3 .. 10 convert, 11 .. 18 drain the two
// accumulators.  TMEM columns: accumulators 0-63 and 64-127, then 4 A
// buffers of 64 columns (128 rows x 128 BF16 values).  Converter warp w owns
// lane quarter w % 4 (TMEM's access rule) and half (w - 3) / 4 of each
// step's K: 32 columns, 64 values of one weight row per thread.
constexpr uint32_t kCvtWarps = 8;
constexpr uint32_t kBfNt = 64;
constexpr uint32_t kBfRawSlot = 17408;  // kMxRawChunk rounded up to 1 KB
constexpr uint32_t kBfRawSlots = 6;
constexpr uint32_t kBfAOp = mxbf_act_block_bytes(kBfNt);
constexpr uint32_t kBfActSlots = 6;
constexpr uint32_t kBfSlots = 4;        // A buffers in TMEM
constexpr uint32_t kBfOffAct = kBfRawSlots * kBfRawSlot;
constexpr uint32_t kBfOffBar = kBfOffAct + kBfActSlots * kBfAOp;
constexpr uint32_t kBfSmem = kBfOffBar + 512 + 1024;
constexpr uint32_t kBfFirstCvt = 3;
constexpr uint32_t kBfEpiWarps = 8;
constexpr uint32_t kBfFirstEpi = kBfFirstCvt + kCvtWarps;
constexpr uint32_t kBfThreads = 32u * (kBfFirstEpi + kBfEpiWarps);
constexpr uint32_t kBfColA = 2u * kBfNt;  // first A buffer column
constexpr uint32_t kBfTmemCols = 512;
static_assert(kBfColA + 64u * kBfSlots <= kBfTmemCols, "TMEM columns");
static_assert(kMxRawChunk <= kBfRawSlot && kBfSmem <= kSmemLimit, "shared memory");
static_assert(kBfAOp % 1024 == 0, "activation slots hold 1 KB-aligned swizzle atoms");

// 16 int8 codes w (x, first code in the low byte) of one scale block -> 16
// BF16 values w * s, s = 2^(e - 133), two to a word, low half first.  With
// u = w + 128 (the sign bit flipped), the FP32 value 2^23 + u is assembled
// from bytes, and (2^23 + u) s - (2^23 + 128) s = w s is one fused
// multiply-add, exact: w s has at most 8 significant bits and s is a power
// of two, so it is representable (as a subnormal too) and its low 16 bits
// are zero, which makes its high half the exact BF16 value.  kWide (e > 237,
// where (2^23 + 128) s overflows): the subtraction first, then the product.
template <bool kWide>
__device__ __forceinline__ void w8_piece_to_bf16(const uint4 x, float s, uint32_t* o) {
  const float c = -8388736.0f * s;
  const uint32_t in[4] = {x.x, x.y, x.z, x.w};
#pragma unroll
  for (uint32_t q = 0; q < 4; ++q) {
    const uint32_t u = in[q] ^ 0x80808080u;
    float f[4];
#pragma unroll
    for (uint32_t j = 0; j < 4; ++j) {
      const float m = __uint_as_float(__byte_perm(u, 0x4B000000u, 0x7540u + j));
      f[j] = kWide ? __fmul_rn(__fadd_rn(m, -8388736.0f), s) : __fmaf_rn(m, s, c);
    }
    o[2 * q] = __byte_perm(__float_as_uint(f[0]), __float_as_uint(f[1]), 0x7632u);
    o[2 * q + 1] = __byte_perm(__float_as_uint(f[2]), __float_as_uint(f[3]), 0x7632u);
  }
}

// 2^(e - 133) as FP32 (a subnormal for e < 7).
__device__ __forceinline__ float w8_scale(uint32_t e) {
  return __uint_as_float(e >= 7u ? (e - 6u) << 23 : 1u << (e + 16u));
}

__global__ void __launch_bounds__(kBfThreads, 1) k_gemm_w8bf(const __grid_constant__ MxParams p) {
  constexpr uint32_t NT = kBfNt;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) &
                                             ~uintptr_t(1023));
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + kBfOffBar);
  const Ring raw{bars, bars + kBfRawSlots, kBfRawSlots};
  const Ring actr{bars + 2 * kBfRawSlots, bars + 2 * kBfRawSlots + kBfActSlots, kBfActSlots};
  uint64_t* a_full = bars + 2 * (kBfRawSlots + kBfActSlots);  // [kBfSlots] converted A
  uint64_t* a_empty = a_full + kBfSlots;       // [kBfSlots] the step's MMAs done
  uint64_t* acc_full = a_empty + kBfSlots;     // [2]
  uint64_t* acc_empty = acc_full + 2;          // [2]
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(acc_empty + 2);
  uint8_t* rbase = smem;
  uint8_t* abase = smem + kBfOffAct;
  const uint32_t warp = threadIdx.x >> 5, lane = threadIdx.x & 31u;

  if (threadIdx.x == 0) {
    for (uint32_t s = 0; s < kBfRawSlots; ++s) {
      mbar_init(&raw.full[s], 1);
      mbar_init(&raw.empty[s], kCvtWarps);
    }
    for (uint32_t s = 0; s < kBfActSlots; ++s) {
      mbar_init(&actr.full[s], 1);
      mbar_init(&actr.empty[s], 1);
    }
    for (uint32_t s = 0; s < kBfSlots; ++s) {
      mbar_init(&a_full[s], kCvtWarps);
      mbar_init(&a_empty[s], 1);
    }
    for (uint32_t b = 0; b < 2; ++b) {
      mbar_init(&acc_full[b], 1);
      mbar_init(&acc_empty[b], 32 * kBfEpiWarps);
    }
    fence_barrier_init();
  }
  if (warp == 1) {
    tmem_alloc(tmem_slot, kBfTmemCols);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;
  bool ok = true;
  griddep_launch_dependents();
  griddep_wait();

  if (warp == 0 || warp == 2) {
    // Lane 0 of warp 0: the raw weight chunks; of warp 2: the activation
    // blocks.  Each tile's fields are loaded one tile ahead.
    if (lane == 0) {
      const bool weights = warp == 0;
      const Ring& ring = weights ? raw : actr;
      uint32_t n = 0;
      MxTile next = tile_info<NT>(p, blockIdx.x);
      for (uint32_t tile = blockIdx.x; tile < p.total_tiles && ok; tile += gridDim.x) {
        const MxTile ti = next;
        if (tile + gridDim.x < p.total_tiles) next = tile_info<NT>(p, tile + gridDim.x);
        const uint32_t k_steps = ti.flags & 0x0FFFFFFFu;
        for (uint32_t i = 0; i < k_steps && ok; ++i, ++n) {
          const uint32_t sl = n % ring.slots;
          ok = ring_acquire(ring, n, weights ? kMxRawChunk : kBfAOp, p.err);
          if (!ok) break;
          if (weights) {
            bulk_g2s(rbase + sl * kBfRawSlot, ti.w + static_cast<size_t>(i) * kMxRawChunk,
                     kMxRawChunk, &ring.full[sl]);
          } else {
            bulk_g2s(abase + sl * kBfAOp, ti.a + static_cast<size_t>(i) * kBfAOp, kBfAOp,
                     &ring.full[sl]);
          }
        }
      }
      if (ok) ring_drain(ring, n, p.err);
    }
  } else if (warp == 1) {
    if (lane == 0) {
      uint32_t n = 0, t = 0;
      uint32_t next_steps = tile_info<NT>(p, blockIdx.x).flags & 0x0FFFFFFFu;
      for (uint32_t tile = blockIdx.x; tile < p.total_tiles && ok; tile += gridDim.x, ++t) {
        const uint32_t k_steps = next_steps;
        if (tile + gridDim.x < p.total_tiles) {
          next_steps = tile_info<NT>(p, tile + gridDim.x).flags & 0x0FFFFFFFu;
        }
        const uint32_t b = t & 1u;
        if (t >= 2) ok = mbar_wait(&acc_empty[b], ((t >> 1) - 1) & 1u, p.err);
        if (!ok) break;
        tc_fence_after();
        const uint32_t d = tmem + b * NT;
        for (uint32_t i = 0; i < k_steps && ok; ++i, ++n) {
          const uint32_t sl = n % kBfSlots, as = n % kBfActSlots;
          ok = mbar_wait(&actr.full[as], (n / kBfActSlots) & 1u, p.err) &&
               mbar_wait(&a_full[sl], (n / kBfSlots) & 1u, p.err);
          if (!ok) break;
          tc_fence_after();
          const uint32_t a_tm = tmem + kBfColA + 64u * sl;
          const uint32_t act = smem_addr(abase + as * kBfAOp);
#pragma unroll
          for (uint32_t k = 0; k < 8; ++k) {
            // K = 16 slice k: A columns 8k .. 8k + 7; activation atom k / 4,
            // 32 bytes in.
            mma_bf16_ts(d, a_tm + 8u * k, desc_sw128(act + (k >> 2) * (NT * kRowB) + 32u * (k & 3u)),
                        idesc_bf16(kTileW, NT), (i > 0 || k > 0) ? 1u : 0u);
          }
          mma_commit(&a_empty[sl]);
          mma_commit(&actr.empty[as]);
        }
        mma_commit(&acc_full[b]);
      }
    }
  } else if (warp >= kBfFirstCvt && warp < kBfFirstEpi) {
    // Converters, all in step: per K step, once the A buffer is free and the
    // raw chunk has landed, each thread loads its row's 64 codes and 2 scale
    // bytes (16-byte chunk c of row r sits at c ^ (r % 8), so 8 consecutive
    // rows read conflict-free), releases the raw slot, converts and stores
    // 32 TMEM columns.  A step's store is waited for, and its buffer
    // signalled, after the next step's conversion, which so overlaps it.
    const uint32_t quarter = warp & 3u, half = (warp - kBfFirstCvt) >> 2;
    const uint32_t r = quarter * 32u + lane;
    constexpr uint32_t kNone = 0xFFFFFFFFu;
    uint32_t pending = kNone;  // the A buffer whose store is in flight
    const auto publish = [&]() {
      if (pending == kNone) return;
      tmem_wait_st();
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&a_full[pending]);
      pending = kNone;
    };
    uint32_t n = 0;
    uint32_t next_steps = tile_info<NT>(p, blockIdx.x).flags & 0x0FFFFFFFu;
    for (uint32_t tile = blockIdx.x; tile < p.total_tiles && ok; tile += gridDim.x) {
      const uint32_t k_steps = next_steps;
      if (tile + gridDim.x < p.total_tiles) {
        next_steps = tile_info<NT>(p, tile + gridDim.x).flags & 0x0FFFFFFFu;
      }
      for (uint32_t i = 0; i < k_steps && ok; ++i, ++n) {
        const uint32_t sl = n % kBfSlots, rs = n % kBfRawSlots;
        if (n >= kBfSlots) ok = mbar_wait(&a_empty[sl], ((n / kBfSlots) - 1) & 1u, p.err);
        if (ok) ok = mbar_wait(&raw.full[rs], (n / kBfRawSlots) & 1u, p.err);
        ok = __all_sync(0xFFFFFFFFu, ok);
        if (!ok) break;
        const uint8_t* row = rbase + rs * kBfRawSlot + r * kRowB;
        uint4 x[4];
#pragma unroll
        for (uint32_t j = 0; j < 4; ++j) {
          x[j] = *reinterpret_cast<const uint4*>(row + (((4u * half + j) ^ (r & 7u)) << 4));
        }
        const uint32_t sc = *reinterpret_cast<const uint16_t*>(rbase + rs * kBfRawSlot +
                                                                kTileW * kRowB + r * 4u + 2u * half);
        __syncwarp();
        if (lane == 0) mbar_arrive(&raw.empty[rs]);
        uint32_t o[32];
#pragma unroll
        for (uint32_t j = 0; j < 4; ++j) {
          const uint32_t e = (sc >> (8u * (j >> 1))) & 0xFFu;  // block 2 half + j / 2
          if (e <= 237u) {
            w8_piece_to_bf16<false>(x[j], w8_scale(e), o + 8u * j);
          } else {
            w8_piece_to_bf16<true>(x[j], w8_scale(e), o + 8u * j);
          }
        }
        publish();
        tc_fence_after();  // after the wait for the A buffer's last readers
        tmem_st32(tmem + ((quarter * 32u) << 16) + kBfColA + 64u * sl + 32u * half, o);
        pending = sl;
      }
    }
    publish();
  } else {
    const uint32_t sp = warp & 3u;
    constexpr uint32_t kRowsPer = NT / (kBfEpiWarps / 4);
    const uint32_t r0 = ((warp - kBfFirstEpi) / 4u) * kRowsPer, r1 = r0 + kRowsPer;
    uint32_t t = 0;
    MxTile next = tile_info<NT>(p, blockIdx.x);
    for (uint32_t tile = blockIdx.x; tile < p.total_tiles; tile += gridDim.x, ++t) {
      const MxTile ti = next;
      if (tile + gridDim.x < p.total_tiles) next = tile_info<NT>(p, tile + gridDim.x);
      const uint32_t b = t & 1u;
      if (ok) ok = mbar_wait_sleep(&acc_full[b], (t >> 1) & 1u, p.err);
      ok = __all_sync(0xFFFFFFFFu, ok);
      if (!ok) break;
      tc_fence_after();
      drain_tile<NT, 1>(p, ti, tmem + ((sp * 32u) << 16) + b * NT, r0, r1, sp, lane);
      tc_fence_before();
      mbar_arrive(&acc_empty[b]);
    }
    if (p.peers.count != 0) __threadfence_system();
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem, kBfTmemCols);
  }
}

// Dense W8 weights [N][kp] + scales [N][kb] -> the raw chunks of the
// kind::f16 kernel, per (128-column tile, 128-element step): 128 rows of 128
// codes (zero past K or N), 16-byte chunk c of row r stored at c ^ (r % 8),
// then the rows' four scale bytes (127 past K or N).  One thread per
// 16-byte output piece.
__global__ void k_tile_weights_w8raw(const uint8_t* __restrict__ w, const uint8_t* __restrict__ ws,
                                     uint32_t N, uint32_t kb, uint32_t steps,
                                     uint8_t* __restrict__ out) {
  constexpr uint32_t kPieces = kMxRawChunk / 16u;
  const uint32_t n_tiles = (N + kTileW - 1) / kTileW;
  const uint64_t pieces = static_cast<uint64_t>(n_tiles) * steps * kPieces;
  const size_t kp = static_cast<size_t>(kb) * 32u;
  for (uint64_t i = blockIdx.x * static_cast<uint64_t>(blockDim.x) + threadIdx.x; i < pieces;
       i += static_cast<uint64_t>(gridDim.x) * blockDim.x) {
    const uint64_t chunk = i / kPieces;
    const uint32_t piece = static_cast<uint32_t>(i % kPieces);
    const uint32_t tile = static_cast<uint32_t>(chunk / steps), step = static_cast<uint32_t>(chunk % steps);
    uint8_t v[16];
    if (piece < kTileW * kRowB / 16u) {
      const uint32_t r = piece / 8u, n = tile * kTileW + r;
      const size_t e0 = static_cast<size_t>(step) * 128u + ((piece % 8u) ^ (r & 7u)) * 16u;
#pragma unroll
      for (int k = 0; k < 16; ++k) {
        v[k] = (n < N && e0 + k < kp) ? w[static_cast<size_t>(n) * kp + e0 + k] : 0;
      }
    } else {
      const uint32_t r0 = (piece - kTileW * kRowB / 16u) * 4u;
#pragma unroll
      for (int k = 0; k < 16; ++k) {
        const uint32_t n = tile * kTileW + r0 + k / 4, blk = step * 4u + k % 4;
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

// One launch with programmatic stream serialisation (the kernels call
// griddep_wait before touching memory): 1 on success, -1 on a launch error.
int launch_pdl(const void* fn, uint32_t grid, uint32_t threads, uint32_t smem, cudaStream_t s,
               const MxParams& p) {
  cudaLaunchConfig_t cfg{};
  cfg.gridDim = dim3(grid);
  cfg.blockDim = dim3(threads);
  cfg.dynamicSmemBytes = smem;
  cfg.stream = s;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  void* args[] = {const_cast<MxParams*>(&p)};
  return cudaLaunchKernelExC(&cfg, fn, args) == cudaSuccess ? 1 : -1;
}

int launch_w8bf(const MxTile* tiles_dev, const TcJob* inline_job, uint32_t tiles, int sm_count,
                uint32_t* err, cudaStream_t s, const MxPeers* peers) {
  MxParams p{};
  p.tiles = tiles_dev;
  p.total_tiles = tiles;
  p.err = err;
  if (peers != nullptr) p.peers = *peers;
  if (inline_job != nullptr) p.inline_job = *inline_job;
  const uint32_t grid = std::min<uint32_t>(tiles, static_cast<uint32_t>(sm_count));
  if (!set_smem_limit_once(reinterpret_cast<const void*>(k_gemm_w8bf), kBfSmem)) return -1;
  return launch_pdl(reinterpret_cast<const void*>(k_gemm_w8bf), grid, kBfThreads, kBfSmem, s, p);
}

// E2M1 code of a digit in [-4, 4]: 0, 1, 2, 3, 4 -> 0b000, 0b010, 0b100,
// 0b101, 0b110; the sign in bit 3.
__device__ __forceinline__ uint32_t e2m1_of_digit(int32_t d) {
  const uint32_t m = static_cast<uint32_t>(d < 0 ? -d : d);
  const uint32_t code = (0x65420u >> (4u * m)) & 0xFu;
  return d < 0 ? (code | 8u) : code;
}

// Digit p of a W8 weight q = 64 d2 + 8 d1 + d0 (d2 = floor((q + 32) / 64),
// d1 = floor((r + 4) / 8) of the rest r, all digits in [-4, 4]).
__device__ __forceinline__ int32_t w8_digit(int32_t q, uint32_t p) {
  const int32_t d2 = (q + 32) >> 6;
  const int32_t r = q - 64 * d2;
  const int32_t d1 = (r + 4) >> 3;
  return p == 2 ? d2 : (p == 1 ? d1 : r - 8 * d1);
}

// Dense weights + scales [N][kb] -> the per-(tile, step, plane) chunks of
// the kernel: MXFP4 [N][kp/2] codes as they are (one plane, 256-element
// steps), W8 [N][kp] int8 as three E2M1 digit planes with scales e - 6 + 3p,
// or MXFP8 [N][kp] E4M3 codes as they are (one plane, 128-element steps:
// one scale chunk, then 512 bytes of padding).  One thread per 16-byte
// output piece.
__global__ void k_tile_weights_mxf4(const uint8_t* __restrict__ w, const uint8_t* __restrict__ ws,
                                    uint32_t N, uint32_t kb, uint32_t steps, uint32_t wp,
                                    uint32_t f8, uint8_t* __restrict__ out) {
  const uint32_t n_tiles = (N + kTileW - 1) / kTileW;
  const uint64_t pieces = static_cast<uint64_t>(n_tiles) * steps * wp * (kWChunk / 16u);
  for (uint64_t i = blockIdx.x * static_cast<uint64_t>(blockDim.x) + threadIdx.x; i < pieces;
       i += static_cast<uint64_t>(gridDim.x) * blockDim.x) {
    const uint64_t chunk = i / (kWChunk / 16u);
    const uint32_t piece = static_cast<uint32_t>(i % (kWChunk / 16u));
    const uint32_t plane = static_cast<uint32_t>(chunk % wp);
    const uint64_t ts = chunk / wp;
    const uint32_t tile = static_cast<uint32_t>(ts / steps), step = static_cast<uint32_t>(ts % steps);
    uint8_t v[16];
    if (piece < kTileW * kRowB / 16u) {
      // Row r, stored 16-byte chunk p holds logical chunk c = p ^ (r % 8):
      // bytes 16c .. 16c+15 of the step's 128-byte row = elements 32c .. 32c+31.
      const uint32_t r = piece / 8u, pc = piece % 8u, c = pc ^ (r & 7u);
      const uint32_t n = tile * kTileW + r;
      const uint32_t e0 = step * 256u + c * 32u;  // first element of the piece
      if (f8) {
        const size_t kp = static_cast<size_t>(kb) * 32u;
        const size_t e8 = static_cast<size_t>(step) * 128u + c * 16u;
#pragma unroll
        for (int k = 0; k < 16; ++k) {
          v[k] = (n < N && e8 + k < kp) ? w[static_cast<size_t>(n) * kp + e8 + k] : 0;
        }
      } else if (wp == 1) {
        const size_t row_bytes = static_cast<size_t>(kb) * 16u;
#pragma unroll
        for (int k = 0; k < 16; ++k) {
          const size_t src = e0 / 2u + k;
          v[k] = (n < N && src < row_bytes) ? w[static_cast<size_t>(n) * row_bytes + src] : 0;
        }
      } else {
        const size_t kp = static_cast<size_t>(kb) * 32u;
#pragma unroll
        for (int k = 0; k < 16; ++k) {
          uint32_t nib[2] = {0u, 0u};
#pragma unroll
          for (int h = 0; h < 2; ++h) {
            const size_t e = e0 + 2u * k + h;
            if (n < N && e < kp) {
              const int32_t q = static_cast<int8_t>(w[static_cast<size_t>(n) * kp + e]);
              nib[h] = e2m1_of_digit(w8_digit(q, plane));
            }
          }
          v[k] = static_cast<uint8_t>(nib[0] | (nib[1] << 4));
        }
      }
    } else {
      // Scale chunk grp, bytes 16i .. 16i+15: bytes 4j + s = scale of row
      // i + 32 j, block 8 step + 4 grp + s (plane p of W8: e - 6 + 3p).
      const uint32_t sp = piece - kTileW * kRowB / 16u;
      const uint32_t grp = sp / 32u, i32 = sp % 32u;
#pragma unroll
      for (int k = 0; k < 16; ++k) {
        const uint32_t j = k / 4, s = k % 4;
        const uint32_t n = tile * kTileW + i32 + 32u * j;
        const uint32_t blk = f8 ? (grp == 0 ? step * 4u + s : kb) : step * 8u + grp * 4u + s;
        int32_t sc = (n < N && blk < kb) ? ws[static_cast<size_t>(n) * kb + blk] : 127;
        if (f8 && grp != 0) sc = 0;  // padding after the one scale chunk
        if (wp == 3) sc = sc - 6 + 3 * static_cast<int32_t>(plane);
        v[k] = static_cast<uint8_t>(sc < 0 ? 0 : (sc > 254 ? 254 : sc));
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

template <uint32_t NT, uint32_t WP, uint32_t KB>
int launch_mx(const MxTile* tiles_dev, const TcJob* inline_job, uint32_t tiles, int sm_count,
              uint32_t* err, cudaStream_t s, const MxPeers* peers,
              const MxGather* gather = nullptr, bool weights_ready = false) {
  using Cfg = MxCfg<NT, WP, KB>;
  MxParams p{};
  p.weights_ready = weights_ready ? 1u : 0u;
  p.tiles = tiles_dev;
  p.total_tiles = tiles;
  p.err = err;
  if (peers != nullptr) p.peers = *peers;
  if (inline_job != nullptr) p.inline_job = *inline_job;
  const uint32_t grid = std::min<uint32_t>(tiles, static_cast<uint32_t>(sm_count));
  if constexpr (WP == 1 && KB == 4) {
    if (gather != nullptr) {
      p.gather = *gather;
      const void* fn = reinterpret_cast<const void*>(k_gemm_mxf4<NT, WP, KB, true>);
      if (!set_smem_limit_once(fn, Cfg::kSmem)) return -1;
      return launch_pdl(fn, grid, MxWarps<NT, WP, KB, true>::kThreads, Cfg::kSmem, s, p);
    }
  }
  if (gather != nullptr) return -1;
  // Early accumulator release pays where CTAs run several tiles; launches
  // of one or two tiles a CTA take the plain (smaller) kernel.
  const void* fn = Cfg::kDBufs == 1 && tiles >= 3u * grid
                       ? reinterpret_cast<const void*>(k_gemm_mxf4<NT, WP, KB, false, true>)
                       : reinterpret_cast<const void*>(k_gemm_mxf4<NT, WP, KB, false, false>);
  if (!set_smem_limit_once(fn, Cfg::kSmem)) return -1;
  return launch_pdl(fn, grid, MxWarps<NT, WP, KB, false>::kThreads, Cfg::kSmem, s, p);
}

// The CTA-pair kernel: clusters of two, as many as fit at once.
template <uint32_t NT>
int launch_pair(const MxTile* tiles_dev, const TcJob* inline_job, uint32_t tiles, int sm_count,
                uint32_t* err, cudaStream_t s, const MxPeers* peers, bool weights_ready) {
  using Cfg = PairCfg<NT>;
  MxParams p{};
  p.weights_ready = weights_ready ? 1u : 0u;
  p.tiles = tiles_dev;
  p.total_tiles = tiles;
  p.err = err;
  if (peers != nullptr) p.peers = *peers;
  if (inline_job != nullptr) p.inline_job = *inline_job;
  const uint32_t pairs = tiles / 2u;
  if (pairs == 0) return 0;
  static int max_clusters[2] = {0, 0};
  int& mc = max_clusters[NT == 64 ? 0 : 1];
  cudaLaunchConfig_t cfg{};
  cudaLaunchAttribute attr[2];
  attr[0].id = cudaLaunchAttributeClusterDimension;
  attr[0].val.clusterDim.x = 2;
  attr[0].val.clusterDim.y = 1;
  attr[0].val.clusterDim.z = 1;
  attr[1].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[1].val.programmaticStreamSerializationAllowed = 1;
  cfg.blockDim = dim3(Cfg::kThreads);
  cfg.dynamicSmemBytes = Cfg::kSmem;
  cfg.stream = s;
  cfg.attrs = attr;
  cfg.numAttrs = 2;
  const void* plain = reinterpret_cast<const void*>(k_gemm_mxf4_pair<NT, false>);
  const void* early = reinterpret_cast<const void*>(k_gemm_mxf4_pair<NT, true>);
  if (!set_smem_limit_once(plain, Cfg::kSmem) || !set_smem_limit_once(early, Cfg::kSmem)) return -1;
  if (mc == 0) {
    cfg.gridDim = dim3(static_cast<unsigned>(sm_count & ~1));
    int n = 0;
    if (cudaOccupancyMaxActiveClusters(&n, plain, &cfg) != cudaSuccess || n < 1) {
      (void)cudaGetLastError();
      n = sm_count / 2;
    }
    mc = n;
  }
  const uint32_t clusters = std::min<uint32_t>(pairs, static_cast<uint32_t>(mc));
  cfg.gridDim = dim3(2u * clusters);
  const void* fn = MxCfg<NT, 1, 4>::kDBufs == 1 && pairs >= 3u * clusters ? early : plain;
  void* args[] = {&p};
  return cudaLaunchKernelExC(&cfg, fn, args) == cudaSuccess ? 1 : -1;
}

template <uint32_t NT, uint32_t WP, uint32_t KB>
struct Pick {
  static constexpr uint32_t kNt = NT, kWp = WP, kKb = KB;
};

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

uint32_t mx_tokens_per_tile(uint32_t M) { return M <= 64 ? 64u : 128u; }

uint32_t mx_k_steps(uint32_t kb) { return (kb + 7) / 8; }

uint32_t mx8_k_steps(uint32_t kb) { return (kb + 3) / 4; }

uint32_t mx_steps_of(uint32_t wfmt, uint32_t kb) {
  return wfmt == HRB_WFMT_MXFP8 || wfmt == kTcW8Bf16 ? mx8_k_steps(kb) : mx_k_steps(kb);
}

uint32_t mx_block_bytes_of(uint32_t wfmt, uint32_t nt) { return act_block_bytes(wfmt, nt); }

size_t mx_weight_bytes(uint32_t wfmt, uint32_t N, uint32_t kb) {
  return static_cast<size_t>((N + kTileW - 1) / kTileW) * mx_steps_of(wfmt, kb) *
         w_step_bytes(wfmt);
}

size_t mx_act_bytes(uint32_t wfmt, uint32_t M, uint32_t kb) {
  const uint32_t nt = wfmt == kTcW8Bf16 ? kBfNt : mx_tokens_per_tile(M);
  return static_cast<size_t>((M + nt - 1) / nt) * mx_steps_of(wfmt, kb) *
         act_block_bytes(wfmt, nt);
}

void launch_tile_weights_mxf4(uint32_t wfmt, const uint8_t* w, const uint8_t* ws, uint32_t N,
                              uint32_t kb, uint8_t* out, cudaStream_t s) {
  const uint64_t pieces = mx_weight_bytes(wfmt, N, kb) / 16u;
  uint64_t grid = (pieces + 255) / 256;
  if (grid > 148u * 16u) grid = 148u * 16u;
  if (wfmt == kTcW8Bf16) {
    k_tile_weights_w8raw<<<static_cast<unsigned>(grid ? grid : 1), 256, 0, s>>>(
        w, ws, N, kb, mx_steps_of(wfmt, kb), out);
    return;
  }
  k_tile_weights_mxf4<<<static_cast<unsigned>(grid ? grid : 1), 256, 0, s>>>(
      w, ws, N, kb, mx_steps_of(wfmt, kb), mx_planes_of(wfmt), wfmt == HRB_WFMT_MXFP8 ? 1u : 0u,
      out);
}

bool mx_pairs(uint32_t wfmt, uint32_t n_tiles) {
  // Opt-in (HRB_CTA_PAIRS=1): on the B200 the pair kernel measures slower
  // than one CTA a tile at every shape of the benchmark (it halves the
  // activation bytes from L2, but neither kernel is bound by them).
  static const bool enabled = [] {
    const char* e = std::getenv("HRB_CTA_PAIRS");
    return e != nullptr && e[0] == '1';
  }();
  return enabled && wfmt == HRB_WFMT_MXFP4 && n_tiles >= 2;
}

uint32_t mx_job_tiles(const TcJob& job, bool pairs) {
  return pairs ? job.m_tiles * 2u * ((job.n_tiles + 1u) / 2u) : job.m_tiles * job.n_tiles;
}

void mx_fill_tiles(const TcJob& job, uint32_t nt, MxTile* out, bool pairs) {
  if (!pairs) {
    for (uint32_t i = 0; i < job.m_tiles * job.n_tiles; ++i) out[i] = make_tile(job, nt, i);
    return;
  }
  // Pair order: tiles 2u, 2u + 1 are column tiles 2c, 2c + 1 of one token
  // tile; an odd last column tile is paired with a dummy (no columns).
  uint32_t k = 0;
  for (uint32_t mt = 0; mt < job.m_tiles; ++mt) {
    for (uint32_t n = 0; n < job.n_tiles; n += 2) {
      const MxTile a = make_tile(job, nt, mt * job.n_tiles + n);
      out[k++] = a;
      out[k++] = n + 1 < job.n_tiles ? make_tile(job, nt, mt * job.n_tiles + n + 1) : dummy_tile(a);
    }
  }
}

int launch_mxf4_gather(const TcJob& inline_job, uint32_t nt, uint32_t tiles, int sm_count,
                       uint32_t* err, cudaStream_t s, const MxGather& gather,
                       const MxPeers* peers) {
  if (tiles == 0) return 0;
  if (inline_job.wfmt != HRB_WFMT_MXFP4 || gather.geom.bp != 8u) return -1;
  if (peers != nullptr && peers->count > kMaxPeers) return -1;
  if (nt == 64) return launch_mx<64, 1, 4>(nullptr, &inline_job, tiles, sm_count, err, s, peers, &gather);
  if (nt == 128) return launch_mx<128, 1, 4>(nullptr, &inline_job, tiles, sm_count, err, s, peers, &gather);
  return -1;
}

int launch_mxf4(const MxTile* tiles_dev, const TcJob* inline_job, uint32_t nt, uint32_t wfmt,
                uint32_t tiles, int sm_count, uint32_t* err, cudaStream_t s,
                const MxPeers* peers, bool weights_ready, int pairs) {
  if (tiles == 0) return 0;
  if (tiles_dev == nullptr && inline_job == nullptr) return -1;
  if (peers != nullptr && peers->count > kMaxPeers) return -1;
  if (pairs < 0) pairs = tiles_dev == nullptr && mx_pairs(wfmt, inline_job->n_tiles) ? 1 : 0;
  if (pairs != 0) {
    if (wfmt != HRB_WFMT_MXFP4) return -1;
    if (tiles_dev == nullptr) tiles = mx_job_tiles(*inline_job, true);
    if (nt == 64) return launch_pair<64>(tiles_dev, inline_job, tiles, sm_count, err, s, peers, weights_ready);
    if (nt == 128) return launch_pair<128>(tiles_dev, inline_job, tiles, sm_count, err, s, peers, weights_ready);
    return -1;
  }
  const auto go = [&](auto cfg) {
    using C = decltype(cfg);
    return launch_mx<C::kNt, C::kWp, C::kKb>(tiles_dev, inline_job, tiles, sm_count, err, s,
                                             peers, nullptr, weights_ready);
  };
  switch (wfmt * 1000u + nt) {
    case HRB_WFMT_MXFP4 * 1000u + 64: return go(Pick<64, 1, 4>{});
    case HRB_WFMT_MXFP4 * 1000u + 128: return go(Pick<128, 1, 4>{});
    case HRB_WFMT_W8 * 1000u + 64: return go(Pick<64, 3, 4>{});
    case HRB_WFMT_W8 * 1000u + 128: return go(Pick<128, 3, 4>{});
    case HRB_WFMT_MXFP8 * 1000u + 64: return go(Pick<64, 1, 8>{});
    case HRB_WFMT_MXFP8 * 1000u + 128: return go(Pick<128, 1, 8>{});
    case kTcW8Bf16 * 1000u + kBfNt:
      return launch_w8bf(tiles_dev, inline_job, tiles, sm_count, err, s, peers);
    default: return -1;
  }
}

}  // namespace hrb
