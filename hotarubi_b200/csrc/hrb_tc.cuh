// Tensor-core (tcgen05) GEMM path: declarations shared with capi.cu.
#pragma once

#include <cuda_runtime.h>

#include <cstddef>
#include <cstdint>

#include "hrb_kernels.cuh"

namespace hrb {

// One GEMM for the block-scaled tensor-core kernel (gemm_mxf4.cu), with its
// prepared operands: activation digit planes and translated weight chunks.
// Path formats: the hrb_wfmt values, plus W8 with at most 64 tokens on
// request (hrb_gemm_desc.w8_kernel), whose int8 weights stream from HBM as
// they are and become BF16 in the kernel.
constexpr uint32_t kTcW8Bf16 = 3;
__host__ __device__ constexpr uint32_t tc_path_format(uint32_t wfmt, uint32_t M,
                                                      uint32_t w8_kernel) {
  return wfmt == HRB_WFMT_W8 && M <= 64u && w8_kernel == HRB_W8_BF16 ? kTcW8Bf16 : wfmt;
}

struct TcJob {
  const uint8_t* a_tiles;  // [m_tiles][k_steps][NT rows][128 B]
  const uint8_t* w_tiles;  // [n_tiles][k_steps][chunk]
  const float* bias;       // [N] or null
  // Per-column scale and bias as interleaved pairs [N][2] (hrb_gemm_desc
  // wcol_scale): the epilogue computes out * scale + bias in two roundings.
  // Replaces `bias` when set.
  const float* epv;
  float* c;                // [M][ldc]
  uint32_t M, N, kb, ldc;
  uint32_t wfmt;           // path format (tc_path_format)
  uint32_t accumulate;
  uint32_t m_tiles, n_tiles, k_steps;
  uint32_t tile_begin;     // prefix over the jobs of one launch
  int8_t* cq;              // MXINT8 copy of C [M][ldcq] or null
  uint8_t* cscale;         // [M][ldcq / 32]
  uint32_t cquant;         // hrb_quant of the copy
  uint32_t ldcq;           // row stride of the copy in codes; 0: kpN
  uint32_t relu;           // RELU after the bias (before the copy)
};

// The block-scaled tensor-core path (gemm_mxf4.cu): kind::mxf4 for MXFP4
// weights (their own E2M1 codes) and W8 weights (three E2M1 digit planes),
// kind::mxf8f6f4 for MXFP8 weights (their own E4M3 codes): tokens per tile
// (64 or 128), K steps, prepared operand sizes, the weight translation and
// the launch.
uint32_t mx_tokens_per_tile(uint32_t M);
uint32_t mx_k_steps(uint32_t kb);

// Activation block of one (token tile of nt rows, 256-element K step) for
// the kind::mxf4 kernel.  The three digit planes are stacked as 3 * nt
// operand rows (plane p, token t -> stacked row p * nt + t), 128 bytes each
// in the 128-byte swizzle; the MMAs take the stack 192 rows at a time (one
// MMA for nt = 64, two for nt = 128).  After the rows come the E8M0 scales:
// per 192-row part and 4-block group, two 512-byte chunks (part rows 0-127,
// then 128-191 with 64 unused rows) in the order tcgen05.cp .32x128b.warpx4
// reads them: row i of 32, bytes 4j + s = scale of part row i + 32 j, block s.
__host__ __device__ constexpr uint32_t mx_parts(uint32_t nt) { return 3u * nt / 192u; }
__host__ __device__ constexpr uint32_t mx_act_block_bytes(uint32_t nt) {
  return 3u * nt * 128u + mx_parts(nt) * 2048u;
}
__host__ __device__ inline uint32_t mx_act_sf_offset(uint32_t nt, uint32_t stacked_row,
                                                     uint32_t block_in_step) {
  const uint32_t part = stacked_row / 192u, r = stacked_row % 192u;
  const uint32_t chunk = (part * 2u + block_in_step / 4u) * 2u + r / 128u;
  return 3u * nt * 128u + chunk * 512u + (r % 32u) * 16u + ((r % 128u) / 32u) * 4u +
         block_in_step % 4u;
}

// The same kernel for MXFP8 (E4M3) weights runs kind::mxf8f6f4 with
// 128-element K steps (one 128-byte row of E4M3 per operand row).  The
// activations are two E4M3 digit planes, q = 16 h + l with h, l in [-8, 8]
// (integers E4M3 holds exactly), stacked as 2 nt operand rows (one MMA of
// N = 2 nt per 32 elements of K).  Block: the 2 nt rows, then per 128
// stacked rows one 512-byte scale chunk (the step's 4 blocks), padded to
// 1024 bytes.
uint32_t mx8_k_steps(uint32_t kb);
__host__ __device__ constexpr uint32_t mx8_act_block_bytes(uint32_t nt) {
  return 2u * nt * 128u + 1024u;
}
__host__ __device__ inline uint32_t mx8_act_sf_offset(uint32_t nt, uint32_t stacked_row,
                                                      uint32_t block_in_step) {
  return 2u * nt * 128u + (stacked_row / 128u) * 512u + (stacked_row % 32u) * 16u +
         ((stacked_row % 128u) / 32u) * 4u + block_in_step;
}
// W8 with at most 64 tokens (path format kTcW8Bf16) runs kind::f16 on BF16
// operands, which hold every MXINT8 activation q * 2^(e-6) and every W8
// weight q * 2^(e-133) exactly, so the products are exact as on the other
// kinds.  K steps of 128 elements.  Activations: per (64-row tile, step) two
// 128-byte-swizzled atoms of 64 rows x 64 BF16 values (elements 64 a ..
// 64 a + 63 of the step in atom a), prepared by the encoder.  Weights: per
// (128-column tile, step) the int8 codes as they are, 128 rows x 128 bytes,
// then the rows' scale bytes [128][4] (kMxRawChunk bytes); the kernel
// converts them to BF16 in shared memory.
constexpr uint32_t kMxRawChunk = 128u * 128u + 512u;
__host__ __device__ constexpr uint32_t mxbf_act_block_bytes(uint32_t nt) { return nt * 256u; }

// K steps and activation block bytes of a path format.
uint32_t mx_steps_of(uint32_t wfmt, uint32_t kb);
uint32_t mx_block_bytes_of(uint32_t wfmt, uint32_t nt);

size_t mx_weight_bytes(uint32_t wfmt, uint32_t N, uint32_t kb);
size_t mx_act_bytes(uint32_t wfmt, uint32_t M, uint32_t kb);
void launch_tile_weights_mxf4(uint32_t wfmt, const uint8_t* w, const uint8_t* ws, uint32_t N,
                              uint32_t kb, uint8_t* out, cudaStream_t stream);
// One output tile of a kind::mxf4 launch with its operands located.  Plans
// build the array on the host once, so the kernel's roles read a tile's
// fields with independent loads, one tile ahead, instead of searching jobs.
struct MxTile {
  const uint8_t* w;     // the tile's first weight chunk
  const uint8_t* a;     // its first activation block
  float* c;             // C at the tile's first row and column, or null
  const float* bias;    // bias at the tile's first column, or null
  int8_t* cq;           // MXINT8 copy at the tile's first row and column, or null
  uint8_t* cscale;      // its scale at the tile's first row and block
  uint32_t rows;        // valid token rows
  uint32_t cols_kbq;    // valid weight columns | blocks per cq row << 8
  uint32_t ldc;
  uint32_t flags;       // K steps | (scale, bias) pairs << 28 | RELU << 29 | VEC rule for cq << 30
                        // | accumulate << 31
};
static_assert(sizeof(MxTile) == 64, "MxTile is read as four 16-byte loads");
// Whether MXFP4 GEMMs of n_tiles column tiles run on CTA pairs (two
// adjacent column tiles as one MMA of M = 256; opt-in with the environment
// variable HRB_CTA_PAIRS=1), the tiles of a job in that order, and the tiles
// themselves: mt * n_tiles + nt, or in pairs (tiles 2u, 2u + 1 the column
// tiles 2c, 2c + 1 of one token tile, an odd last one paired with a tile of
// no columns).
bool mx_pairs(uint32_t wfmt, uint32_t n_tiles);
uint32_t mx_job_tiles(const TcJob& job, bool pairs);
void mx_fill_tiles(const TcJob& job, uint32_t nt, MxTile* out, bool pairs = false);
// Peers that receive a copy of every output (the fused all-gather of a
// column- or row-sharded layer): an output byte at address x (C or the
// MXINT8 copy) is also stored at x + delta[i].
constexpr uint32_t kMaxPeers = 7;
struct MxPeers {
  int64_t delta[kMaxPeers];
  uint32_t count;
};

// The gathering variant of the MXFP4 kernel (convolutions whose channel
// planes are 256 wide, so one K step is one (plane, tap)): the activation
// block of each (tile, step) is assembled in shared memory from the input
// map's own operand blocks (map_shift: log2 of their tile height) instead of
// being read as one prepared block.  `rows` = M.
struct MxGather {
  const uint8_t* map_tiles;
  uint32_t map_shift, map_steps, map_block_bytes, rows;
  ConvGeom geom;
};
// One inline job (inline_job.a_tiles unused), nt = 64 or 128.
int launch_mxf4_gather(const TcJob& inline_job, uint32_t nt, uint32_t tiles, int sm_count,
                       uint32_t* err, cudaStream_t stream, const MxGather& gather,
                       const MxPeers* peers = nullptr);

// One launch over `tiles` output tiles: the device array tiles_dev, or, when
// it is null, the tiles of the single *inline_job.  `peers` may be null.
// weights_ready: the weight chunks were written and the stream synchronised
// before (a plan's), so the kernel may read them before its dependency wait.
// pairs: 1 when tiles_dev is in pair order (mx_fill_tiles with pairs; CTA
// pairs run it), 0 when it is not, -1 (the inline job) to decide by
// mx_pairs (the tile count then follows).
int launch_mxf4(const MxTile* tiles_dev, const TcJob* inline_job, uint32_t nt, uint32_t wfmt,
                uint32_t tiles, int sm_count, uint32_t* err, cudaStream_t stream,
                const MxPeers* peers = nullptr, bool weights_ready = false, int pairs = -1);

// Raises `kernel`'s dynamic shared-memory limit to `bytes` on the current
// device, once per (kernel, device).
bool set_smem_limit_once(const void* kernel, uint32_t bytes);

}  // namespace hrb
