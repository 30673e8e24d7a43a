// Device-side job descriptors and kernel launchers shared by the C ABI layer
// (capi.cu) and the kernel files.  Internal to libhrb_gemm.so.
#pragma once

#include <cuda_runtime.h>

#include <cstdint>

#include "hrb_gemm.h"

namespace hrb {

// Unsigned 32-bit division by a divisor fixed for a launch, as a multiply
// and shifts (Granlund and Montgomery, "Division by invariant integers using
// multiplication", PLDI 1994, section 4): for d >= 1 with l = ceil(log2 d),
// m = floor(2^32 (2^l - d) / d) + 1, n / d = (t + ((n - t) >> 1)) >> (l - 1)
// where t = mulhi(m, n); d = 1 takes l = 0 and the shifts degenerate.
struct FastDiv {
  uint32_t d, m, s1, s2;
};
inline FastDiv make_fast_div(uint32_t d) {
  uint32_t l = 0;
  while (l < 32 && (uint64_t{1} << l) < d) ++l;
  FastDiv f;
  f.d = d;
  f.m = static_cast<uint32_t>(((uint64_t{1} << 32) * ((uint64_t{1} << l) - d)) / d + 1);
  f.s1 = l > 0 ? 1u : 0u;
  f.s2 = l > 0 ? l - 1u : 0u;
  return f;
}
__host__ __device__ inline uint32_t fast_div(uint32_t n, const FastDiv& f) {
#ifdef __CUDA_ARCH__
  const uint32_t t = __umulhi(f.m, n);
#else
  const uint32_t t = static_cast<uint32_t>((uint64_t{f.m} * n) >> 32);
#endif
  return (t + ((n - t) >> f.s1)) >> f.s2;
}

// Geometry of a convolution run as a GEMM whose activation rows are
// gathered (hotarubi's ConvEmitter, tools/compiler/sparsedrive_encoder.cpp):
// output row img * Ho * Wo + o reads, for K column (plane, tap, channel in
// plane), channel plane * 32 * bp + channel of the input position under tap
// (ky, kx) = (tap / kh, tap % kh) with padding (kh - 1) / 2, or zero outside
// the map.  Positions are x-major (order 0: x * H + y) or y-major (y * W + x).
// The divisors the index arithmetic needs come precomputed (make_conv_geom).
struct ConvGeom {
  uint32_t images, H, W, Ho, Wo, cin, kh, stride, order;
  uint32_t bp;      // K blocks per channel plane (min(cin, 256) / 32)
  uint32_t kbo;     // gathered K blocks per output row: kh * kh * cin / 32
  FastDiv out_per;  // Ho * Wo
  FastDiv minor;    // Ho (x-major) or Wo (y-major)
  FastDiv kh_div;   // kh
  FastDiv bp_div;   // bp
  FastDiv plane_k;  // kh * kh * bp, gathered blocks per channel plane
  FastDiv kbo_div;  // kbo
};

inline ConvGeom make_conv_geom(uint32_t images, uint32_t H, uint32_t W, uint32_t cin, uint32_t kh,
                               uint32_t stride, uint32_t order) {
  ConvGeom g{};
  g.images = images;
  g.H = H;
  g.W = W;
  g.Ho = H / stride;
  g.Wo = W / stride;
  g.cin = cin;
  g.kh = kh;
  g.stride = stride;
  g.order = order;
  g.bp = (cin < 256u ? cin : 256u) / 32u;
  g.kbo = kh * kh * cin / 32u;
  g.out_per = make_fast_div(g.Ho * g.Wo);
  g.minor = make_fast_div(order == 0 ? g.Ho : g.Wo);
  g.kh_div = make_fast_div(kh);
  g.bp_div = make_fast_div(g.bp);
  g.plane_k = make_fast_div(kh * kh * g.bp);
  g.kbo_div = make_fast_div(g.kbo);
  return g;
}

// Input position of output row `row` under tap `tap`, or -1 outside the map.
__host__ __device__ inline int64_t conv_source_row(const ConvGeom& g, uint32_t row, uint32_t tap) {
  const uint32_t img = fast_div(row, g.out_per), o = row - img * g.out_per.d;
  const uint32_t major = fast_div(o, g.minor), minor = o - major * g.minor.d;
  const uint32_t yo = g.order == 0 ? minor : major;
  const uint32_t xo = g.order == 0 ? major : minor;
  const uint32_t ky = fast_div(tap, g.kh_div), kx = tap - ky * g.kh, pad = (g.kh - 1u) / 2u;
  const int32_t yi = static_cast<int32_t>(g.stride * yo + ky) - static_cast<int32_t>(pad);
  const int32_t xi = static_cast<int32_t>(g.stride * xo + kx) - static_cast<int32_t>(pad);
  if (yi < 0 || yi >= static_cast<int32_t>(g.H) || xi < 0 || xi >= static_cast<int32_t>(g.W)) {
    return -1;
  }
  const uint32_t pos = g.order == 0 ? static_cast<uint32_t>(xi) * g.H + static_cast<uint32_t>(yi)
                                    : static_cast<uint32_t>(yi) * g.W + static_cast<uint32_t>(xi);
  return static_cast<int64_t>(img) * g.H * g.W + pos;
}

// The (input row, input K block) of gathered K block `b` of output row `row`,
// or -1 when it falls outside the map.
__host__ __device__ inline int64_t conv_source_block(const ConvGeom& g, uint32_t row, uint32_t b,
                                                     uint32_t* in_block) {
  const uint32_t plane = fast_div(b, g.plane_k), rem = b - plane * g.plane_k.d;
  const uint32_t tap = fast_div(rem, g.bp_div), cb = rem - tap * g.bp;
  *in_block = plane * g.bp + cb;
  return conv_source_row(g, row, tap);
}

// One FP32 -> MXINT8 encode.  Units are (row, 128-column chunk) pairs;
// `unit_begin` is the prefix sum over the jobs of a launch.
struct QuantJob {
  const float* x;
  int8_t* q;          // [rows][ldq * 32], or null
  uint8_t* scale;     // [rows][ldq], or null
  uint32_t ldq;       // row stride of q and scale in blocks; 0: kb
  // The tensor-core operands (launch_quantize_planes): the activations as
  // digit planes with their E8M0 scales in the activation blocks of
  // hrb_tc.cuh, [row tiles of tile_rows][k_steps][block].  tiles_kind 2:
  // three E2M1 planes, 256-element K steps (kind::mxf4); tiles_kind 3: two
  // E4M3 planes, 128-element K steps (kind::mxf8f6f4); tiles_kind 4: BF16
  // values, 128-element K steps (kind::f16).
  uint8_t* tiles;
  uint64_t unit_begin;
  uint64_t units;     // rows * ceil(kb / 4); planes: rows * 256-element groups
  uint32_t rows, cols, ldx, kb;
  uint32_t vec_rule;  // 0: EncodeMxint8, 1: VEC 'q' pass
  uint32_t vec4;      // x rows are 16-byte aligned: load float4
  uint32_t tile_rows, k_steps;
  uint32_t tiles_kind;
  uint32_t cover_blocks;  // K blocks written (kb plus the steps' zero padding)
  // E2M1 planes: prefix over a launch's jobs of their (row, group of four
  // 256-element steps) items, rows * ceil(k_steps / 4) per job; the
  // specialised encoder's unit of work.
  uint64_t group_begin;
};

constexpr uint32_t kMaxPieces = 64;

// One dense GEMM for the exact kernels.  Tiles are 64 x 64 outputs;
// `tile_begin` is the prefix sum over the GEMMs of a launch.
struct DenseJob {
  const int8_t* aq;       // [M][kp]
  const uint8_t* ascale;  // [M][kb]
  const uint8_t* w;       // format dependent, [N][...]
  const uint8_t* wscale;  // [N][kb]
  const float* bias;      // [N] or null
  const float* colscale;  // [N] or null: the chain times colscale[n], then the bias
  float* c;               // [M][ldc]
  uint32_t tile_begin;
  uint32_t tiles_n;       // column tiles
  uint32_t M, N, kb, ldc;
  uint32_t wfmt;          // 0 MXFP4, 1 W8, 2 MXFP8
  uint32_t accumulate;
  uint32_t npieces;
  uint32_t pieces[kMaxPieces];
};

// The exact chain with its block dots on the tensor cores
// (gemm_exact_tc.cu): a DenseJob whose weights were translated into int8
// chunks by launch_x_translate, in output tiles of 128 weight rows x 64
// tokens (16 for GEMMs of at most 16 tokens).  MXFP4 and W8 only
// (x_supported).
struct XJob {
  DenseJob d;
  const uint8_t* wt;          // [n_tiles][steps][planes] chunks of 128 x 128 int8
  const uint8_t* wsc;         // [n_tiles][steps] 4 blocks x 128 rows of scale bytes
  uint32_t planes, steps;     // 1 (MXFP4) or 2 (W8: HI, LO); ceil(kb / 4)
  uint32_t m_tiles, n_tiles;  // of the launch's token tile
  uint32_t tile_begin;        // prefix over the launch's jobs
};

bool x_supported(uint32_t wfmt);
// Bytes of the translated weights: the chunks (x_code_bytes), then the scales.
size_t x_code_bytes(uint32_t wfmt, uint32_t N, uint32_t kb);
size_t x_weight_bytes(uint32_t wfmt, uint32_t N, uint32_t kb);
// The token tile of a job of M tokens (16 for M <= 16, else 64) and its
// output tiles.
uint32_t x_tok(uint32_t M);
uint32_t x_tiles(uint32_t M, uint32_t N, uint32_t tok);
void launch_x_translate(uint32_t wfmt, const uint8_t* w, const uint8_t* wscale, uint32_t N,
                        uint32_t kb, uint8_t* out, cudaStream_t stream);
// One launch over `tiles` output tiles of jobs_dev (or of *inline_job),
// every job with token tile `tok` (x_tok).
int launch_x_exact(const XJob* jobs_dev, uint32_t njobs, const XJob* inline_job, uint32_t tiles,
                   uint32_t tok, int sm_count, uint32_t* err, cudaStream_t stream);

// Host-side launchers (async on `stream`).  Either jobs_dev points to njobs
// device-resident jobs, or it is null and the single *inline_job travels as
// a kernel parameter (no staging buffer, nothing to keep alive).
void launch_quantize(const QuantJob* jobs_dev, uint32_t njobs, const QuantJob* inline_job,
                     uint64_t total_units, uint32_t* error_flag, int sm_count,
                     cudaStream_t stream);

// The activations of kind::mxf4 GEMMs (tiles_kind 2): E2M1 digit planes and
// their scales, no MXINT8 output.  A unit is one (row, 256-element K step):
// units = rows * k_steps per job, unit_begin the prefix over the launch.
// jobs_host: a host copy of jobs_dev (or null), from which the launch picks
// the specialised encoder when every job allows it.
// MXINT8 activations read where they lie: hotarubi's DMA row format (a
// token's unit of tok x 32 codes then tok scale bytes in one or two 16-byte
// beats, MakeRowFormat, tools/iss/dma_engine.cpp:156-183), its units found
// by position (ROW) or through a list of DDR unit addresses (ROW_INDEXED,
// :231-262), or dense codes [M][kp] with scales [M][kb] (window null).
struct RowsSrc {
  const uint8_t* window;   // device copy of DDR bytes [ddr_base, ddr_base + window_bytes)
  uint64_t ddr_base, window_bytes;
  const uint32_t* index;   // ROW_INDEXED: a DDR unit address per token (0xFFFFFFFF null)
  uint64_t first;          // ROW: window offset of token 0's unit of plane 0
  uint64_t plane_stride, row_stride;
  uint32_t tok, planes, row_tokens, unit_bytes;
  const int8_t* aq;        // dense source
  const uint8_t* ascale;
  uint32_t kp, kb;
};

// Error-flag bits the row kernels set (hrb_sync reports them).
constexpr uint32_t kErrRowOutside = 8u;    // a unit outside the DDR window
constexpr uint32_t kErrScaleRange = 16u;   // a scale byte the tensor-core planes cannot carry

// The tensor-core operand blocks of `job` (tiles, tile_rows, k_steps,
// tiles_kind as tc_quant_job sets them) from MXINT8 activations.
void launch_rows_planes(const RowsSrc& src, const QuantJob& job, uint32_t* error_flag,
                        int sm_count, cudaStream_t stream);
// The same activations as dense codes aq [M][kb * 32] and scales [M][kb].
void launch_rows_dense(const RowsSrc& src, uint32_t M, int8_t* aq, uint8_t* ascale,
                       uint32_t* error_flag, int sm_count, cudaStream_t stream);

void launch_quantize_planes(const QuantJob* jobs_dev, uint32_t njobs, const QuantJob* inline_job,
                            uint64_t total_units, uint32_t* error_flag, int sm_count,
                            cudaStream_t stream, const QuantJob* jobs_host = nullptr);

// The exact (bit-identical) dense GEMM on CUDA cores, all GEMMs of one weight
// format per launch.  Returns the number of kernels launched.
int launch_dense_exact(const DenseJob* jobs_dev, uint32_t njobs, const DenseJob* inline_job,
                       uint32_t total_tiles, uint32_t wfmt, cudaStream_t stream);
// Output tiles of one GEMM for the exact kernel (tiles_n: column tiles).
uint32_t dense_exact_tiles(uint32_t M, uint32_t N, uint32_t& tiles_n);

struct ExecCmd {
  uint32_t a_base, a_stride, kb, m, w_base, w_stride, n8, c_base, wmode, acc;
};

// ExecuteGemm on device-resident memories.
int launch_exec(const ExecCmd& cmd, const uint8_t* abuf, const uint8_t* wbuf, float* fbuf,
                cudaStream_t stream);

}  // namespace hrb

// The argument checks and job builders of the dense entry points, shared
// with hrb_gemm_dense_noalloc (noalloc.cu), which has no context to hold a
// message.
namespace hrb {
hrb_status check_desc_for_noalloc(const hrb_gemm_desc* desc, uint32_t* pieces,
                                  uint32_t* npieces);
QuantJob make_quant_job_for_noalloc(const hrb_gemm_desc* desc, int8_t* q, uint8_t* scale);
// The encoder over C for the MXINT8 copy (desc->cq).
QuantJob make_post_quant_job_for_noalloc(const hrb_gemm_desc* desc);
DenseJob make_dense_job_for_noalloc(const hrb_gemm_desc* desc, const int8_t* aq,
                                    const uint8_t* ascale, const uint32_t* pieces,
                                    uint32_t npieces);
// Context fields for the entry points outside capi.cu (comm.cu): the
// device, and a failure that leaves `message` for hrb_last_error (ctx may
// be null: the calling thread's message).
int ctx_device(const hrb_ctx* ctx);
hrb_status ctx_fail(hrb_ctx* ctx, hrb_status status, const char* message);
// The message of a failed context-free call (hrb_last_error(NULL)).
hrb_status noalloc_fail(hrb_status status, const char* message);
hrb_status noalloc_cuda_fail(cudaError_t err, const char* what);

// Layout translation kernels.
void launch_wbuf_to_dense(const uint8_t* words, uint32_t groups, uint32_t kb, uint8_t* codes,
                          uint8_t* scales, cudaStream_t stream);
void launch_w8_planes_to_dense(const uint8_t* hi, const uint8_t* lo, uint32_t groups,
                               uint32_t kb, int8_t* q, uint8_t* scales, cudaStream_t stream);
void launch_abuf_to_dense(const uint8_t* words, uint32_t quads, uint32_t kb, int8_t* q,
                          uint8_t* scales, cudaStream_t stream);
void launch_dense_to_fbuf(const float* c, uint32_t rows, uint32_t cols, float* words,
                          cudaStream_t stream);

// Convolution helpers (conv.cu): the gathered MXINT8 rows of the exact path,
// the weight matrix reordered to the chain's (plane, tap, channel) order,
// and the VEC RELU pass over an exact output.
void launch_conv_im2col(const int8_t* aq, const uint8_t* ascale, const ConvGeom& g, int8_t* q,
                        uint8_t* scale, cudaStream_t stream);
void launch_conv_weights(const uint8_t* w, const uint8_t* ws, uint32_t N, const ConvGeom& g,
                         uint32_t bytes_per_block, uint8_t* out_w, uint8_t* out_ws,
                         cudaStream_t stream);
void launch_relu_exact(float* c, uint32_t M, uint32_t N, uint32_t ldc, cudaStream_t stream);
// The tensor-core path's gather: the conv GEMM's activation blocks (nt-row
// tiles, `steps` K steps) assembled block by block from the input map's own
// activation blocks (map_nt-row tiles, map_steps K steps), both in the
// layout of hrb_tc.cuh (f8: the two-E4M3-plane layout, else three E2M1).
void launch_conv_gather_tiles(const uint8_t* map_tiles, uint32_t map_nt, uint32_t map_steps,
                              uint8_t* tiles, uint32_t nt, uint32_t steps, uint32_t f8,
                              const ConvGeom& g, cudaStream_t stream);

// GACC in dense form (gacc.cu): see hrb_gacc_desc.
struct GaccJob {
  const uint64_t* entries;  // [tokens][slots][corners]
  const uint32_t* w;        // FP32 bits [tokens][slots][blocks]
  const uint8_t* rows;      // feature rows, row_stride bytes apart
  uint64_t row_stride;
  uint32_t nrows;
  float* out;               // [tokens][blocks * 32]
  uint32_t tokens, slots, corners, blocks, accumulate;
};
void launch_gacc(const GaccJob& job, uint32_t* error_flag, int sm_count, cudaStream_t stream);

// T32_SPLIT8 in dense form (kv_operands.cu).
void launch_t32_split8(const int8_t* vq, const uint8_t* vs, uint32_t tokens, uint32_t hd,
                       uint32_t ldv, int8_t* wq, uint8_t* ws, int sm_count,
                       cudaStream_t stream);

}  // namespace hrb
