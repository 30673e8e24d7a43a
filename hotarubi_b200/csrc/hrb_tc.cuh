// Tensor-core (tcgen05) GEMM path: declarations shared with capi.cu.
#pragma once

#include <cuda_runtime.h>

#include <cstddef>
#include <cstdint>

#include "hrb_kernels.cuh"

namespace hrb {

// One GEMM for the tensor-core kernel.  Operands are the prepared tiles of
// gemm_tc.cu: activations as swizzled BF16 tiles, weights as raw chunks.
struct TcJob {
  const uint8_t* a_tiles;  // [m_tiles][k_steps][NT rows][128 B]
  const uint8_t* w_tiles;  // [n_tiles][k_steps][chunk]
  const float* bias;       // [N] or null
  float* c;                // [M][ldc]
  uint32_t M, N, kb, ldc;
  uint32_t wfmt;
  uint32_t accumulate;
  uint32_t m_tiles, n_tiles, k_steps;
  uint32_t tile_begin;     // prefix over the jobs of one launch
};

// Token rows per activation tile for a GEMM of M tokens (64, 128 or 256).
uint32_t tc_tokens_per_tile(uint32_t M);
uint32_t tc_k_steps(uint32_t kb);
size_t tc_weight_tile_bytes(uint32_t wfmt, uint32_t N, uint32_t kb);
size_t tc_act_tile_bytes(uint32_t M, uint32_t kb);
void tc_fill_job(TcJob& t, uint32_t wfmt, uint32_t M, uint32_t N, uint32_t kb);

// The kind::mxf4 path for MXFP4 weights (gemm_mxf4.cu): tokens per tile
// (64 or 128), 256-element K steps, prepared operand sizes, the weight
// translation and the launch.
uint32_t mx_tokens_per_tile(uint32_t M);
uint32_t mx_k_steps(uint32_t kb);
size_t mx_weight_bytes(uint32_t N, uint32_t kb);
size_t mx_act_bytes(uint32_t M, uint32_t kb);
void launch_tile_weights_mxf4(const uint8_t* w, const uint8_t* ws, uint32_t N, uint32_t kb,
                              uint8_t* out, cudaStream_t stream);
int launch_mxf4_jobs(const TcJob* jobs_dev, uint32_t njobs, const TcJob* inline_job, uint32_t nt,
                     uint32_t tiles, int sm_count, uint32_t* err, cudaStream_t stream);

// Dense weights -> the chunk layout the kernel streams.
void launch_tile_weights(const uint8_t* w, const uint8_t* ws, uint32_t N, uint32_t kb,
                         uint32_t wfmt, uint8_t* out, cudaStream_t stream);

// One launch over `njobs` device-resident jobs (or, with jobs_dev null, the
// single *inline_job passed as a kernel parameter) with the same
// tokens-per-tile `nt` and weight format; `tiles` is the total CTA count.
// Returns the number of kernels launched or -1.
int launch_tc_jobs(const TcJob* jobs_dev, uint32_t njobs, const TcJob* inline_job, uint32_t nt,
                   uint32_t wfmt, uint32_t tiles, uint32_t* err, cudaStream_t stream);

}  // namespace hrb
