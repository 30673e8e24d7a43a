// Device-side job descriptors and kernel launchers shared by the C ABI layer
// (capi.cu) and the kernel files.  Internal to libhrb_gemm.so.
#pragma once

#include <cuda_runtime.h>

#include <cstdint>

#include "hrb_gemm.h"

namespace hrb {

// One FP32 -> MXINT8 encode.  Units are (row, 128-column chunk) pairs;
// `unit_begin` is the prefix sum over the jobs of a launch.
struct QuantJob {
  const float* x;
  int8_t* q;          // [rows][kb * 32], or null
  uint8_t* scale;     // [rows][kb], or null
  // The tensor-core operands (launch_quantize_planes): the activations as
  // digit planes with their E8M0 scales in the activation blocks of
  // hrb_tc.cuh, [row tiles of tile_rows][k_steps][block].  tiles_kind 2:
  // three E2M1 planes, 256-element K steps (kind::mxf4); tiles_kind 3: two
  // E4M3 planes, 128-element K steps (kind::mxf8f6f4).
  uint8_t* tiles;
  uint64_t unit_begin;
  uint64_t units;     // rows * ceil(kb / 4); planes: rows * 256-element groups
  uint32_t rows, cols, ldx, kb;
  uint32_t vec_rule;  // 0: EncodeMxint8, 1: VEC 'q' pass
  uint32_t vec4;      // x rows are 16-byte aligned: load float4
  uint32_t tile_rows, k_steps;
  uint32_t tiles_kind;
  uint32_t cover_blocks;  // K blocks written (kb plus the steps' zero padding)
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
  float* c;               // [M][ldc]
  uint32_t tile_begin;
  uint32_t tiles_n;       // column tiles
  uint32_t M, N, kb, ldc;
  uint32_t wfmt;          // 0 MXFP4, 1 W8, 2 MXFP8
  uint32_t accumulate;
  uint32_t npieces;
  uint32_t pieces[kMaxPieces];
};

// Host-side launchers (async on `stream`).  Either jobs_dev points to njobs
// device-resident jobs, or it is null and the single *inline_job travels as
// a kernel parameter (no staging buffer, nothing to keep alive).
void launch_quantize(const QuantJob* jobs_dev, uint32_t njobs, const QuantJob* inline_job,
                     uint64_t total_units, uint32_t* error_flag, int sm_count,
                     cudaStream_t stream);

// The activations of kind::mxf4 GEMMs (tiles_kind 2): E2M1 digit planes and
// their scales, no MXINT8 output.  A unit is one (row, 256-element K step):
// units = rows * k_steps per job, unit_begin the prefix over the launch.
void launch_quantize_planes(const QuantJob* jobs_dev, uint32_t njobs, const QuantJob* inline_job,
                            uint64_t total_units, uint32_t* error_flag, int sm_count,
                            cudaStream_t stream);

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

// Layout translation kernels.
void launch_wbuf_to_dense(const uint8_t* words, uint32_t groups, uint32_t kb, uint8_t* codes,
                          uint8_t* scales, cudaStream_t stream);
void launch_w8_planes_to_dense(const uint8_t* hi, const uint8_t* lo, uint32_t groups,
                               uint32_t kb, int8_t* q, uint8_t* scales, cudaStream_t stream);
void launch_abuf_to_dense(const uint8_t* words, uint32_t quads, uint32_t kb, int8_t* q,
                          uint8_t* scales, cudaStream_t stream);
void launch_dense_to_fbuf(const float* c, uint32_t rows, uint32_t cols, float* words,
                          cudaStream_t stream);

// T32_SPLIT8 in dense form (kv_operands.cu).
void launch_t32_split8(const int8_t* vq, const uint8_t* vs, uint32_t tokens, uint32_t hd,
                       uint32_t ldv, int8_t* wq, uint8_t* ws, int sm_count,
                       cudaStream_t stream);

}  // namespace hrb
