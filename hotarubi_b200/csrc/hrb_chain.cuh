// One output of hotarubi's GEMM chain recomputed from the dense operands
// with the integer restatements of the reference's adder and multiplier
// (hrb_device.cuh): the slow path the exact kernels take for an output whose
// fast chain met an infinity or NaN (exponent field 255), where the
// hardware add and the reference's adder part ways.  The order is the
// reference's: K pieces, within each the planes (W8: HI, then LO), within
// each the blocks (tools/compiler/kernels.cpp:35-37,343-395); then the
// column scale (Fp32Mul) and the bias (Fp32Add).
#pragma once

#include <cstdint>

#include "hrb_device.cuh"
#include "hrb_kernels.cuh"

namespace hrb {

// Recomputes one output's chain with the integer adder (the rare case of an
// infinity or NaN anywhere in the chain).
template <int WF>
static __device__ __noinline__ uint32_t chain_slow(const DenseJob& job, uint32_t m, uint32_t n) {
  const size_t kp = static_cast<size_t>(job.kb) * 32u;
  uint32_t acc = job.accumulate ? __float_as_uint(job.c[static_cast<size_t>(m) * job.ldc + n]) : 0u;
  const uint32_t planes = WF == 1 ? 2u : 1u;
  uint32_t first = 0;
  for (uint32_t p = 0; p < job.npieces; ++p) {
    for (uint32_t l = 0; l < planes; ++l) {
      const uint32_t mode = WF == 0 ? kModeFp4 : WF == 2 ? kModeE4m3 : (l == 0 ? kModeW8Hi : kModeW8Lo);
      for (uint32_t b = first; b < first + job.pieces[p]; ++b) {
        int32_t sum = 0;
        for (uint32_t k = 0; k < 32; ++k) {
          const int32_t a = job.aq[m * kp + b * 32u + k];
          int32_t w;
          if (WF == 0) {
            const uint32_t byte = job.w[n * (kp / 2) + b * 16u + k / 2];
            const uint32_t nib = (byte >> ((k & 1u) * 4)) & 0xFu;
            // 2 x E2M1 magnitudes {0,1,2,3,4,6,8,12} packed one per nibble.
            const int32_t mag = static_cast<int32_t>((0xC8643210u >> ((nib & 7u) * 4)) & 0xFu);
            w = (nib & 8u) ? -mag : mag;
          } else if (WF == 1) {
            const int8_t q = static_cast<int8_t>(job.w[n * kp + b * 32u + k]);
            w = l == 0 ? (q >> 4) : (q & 15);
          } else {
            w = e4m3_units(job.w[n * kp + b * 32u + k]);
          }
          sum += a * w;
        }
        const int32_t e = static_cast<int32_t>(job.ascale[static_cast<size_t>(m) * job.kb + b]) +
                          static_cast<int32_t>(job.wscale[static_cast<size_t>(n) * job.kb + b]) - 254 +
                          scale_bias(mode);
        acc = iss_add(acc, block_value_wide(sum, e));
      }
    }
    first += job.pieces[p];
  }
  if (job.colscale != nullptr) acc = iss_mul(acc, __float_as_uint(job.colscale[n]));
  if (job.bias != nullptr) acc = iss_add(acc, __float_as_uint(job.bias[n]));
  return acc;
}

}  // namespace hrb
