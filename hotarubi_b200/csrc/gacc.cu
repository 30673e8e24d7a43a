// GACC, the DMA engine's gather-accumulate (DmaEngine::Gather,
// tools/iss/dma_engine.cpp:599-652): deformable sampling for SparseDrive.
// Every output token accumulates, slot by slot and corner by corner, a
// gathered MXINT8 feature row scaled by a coefficient:
//
//   coef_b = ScaleCoefficient(Fp32Mul(w[t][s][b], bw), row scale b)
//   out[t][32b + v] = Fp32Add(out[t][32b + v], Fp32Mul(Int8ToFp32(q_v), coef_b))
//
// with the ISS's FP32 arithmetic, each output's chain in (slot, corner)
// order, so results are bit-identical to the instruction.
//
// k_gacc: one warp per (token, 256 channels); lane l owns channels
// 8l .. 8l+7 (block l / 4) and keeps their eight accumulators in registers
// across the whole chain.  Per entry the warp gathers the row's 256 codes
// (8 bytes per lane, one 256-byte span) and the scale bytes; the entry list
// is read ahead, so the next row's address is known while this one adds.
// Gather (latency) bound: one random row of blocks * 33 bytes per entry.
//
// Arithmetic: FP32 multiplies and adds run on the FMA pipe with flush to
// zero, which for finite normal operands gives the ISS's results except in
// three places handled here: a zero result's sign (the ISS always gives +0),
// an exponent field of 255 in an operand (the ISS reads it as an ordinary
// exponent: the integer restatements iss_mul / iss_add take over), and a
// product just under the normal range that the hardware rounds up to 2^-126
// before flushing while the ISS rounds to 24 bits first (a product equal to
// +-2^-126 is recomputed with iss_mul).
#include <cstdint>

#include "hrb_device.cuh"
#include "hrb_kernels.cuh"

namespace hrb {
namespace {

// Fp32Mul (tools/iss/fp32.hpp:77-92): the 48-bit product of the
// significands rounded once to 24 bits, +0 below the normal range.
__device__ __noinline__ uint32_t iss_mul(uint32_t a, uint32_t b) {
  const uint32_t ea = (a >> 23) & 0xFFu, eb = (b >> 23) & 0xFFu;
  if (ea == 0 || eb == 0) return 0u;
  const uint64_t product = static_cast<uint64_t>((a & 0x7FFFFFu) | 0x800000u) *
                           static_cast<uint64_t>((b & 0x7FFFFFu) | 0x800000u);
  return iss_round_pack((a ^ b) >> 31, product, static_cast<int32_t>(ea + eb) - 300);
}

__device__ __forceinline__ uint32_t gacc_mul(uint32_t a, uint32_t b) {
  const uint32_t ea = (a >> 23) & 0xFFu, eb = (b >> 23) & 0xFFu;
  if (ea == 0 || eb == 0) return 0u;
  if (ea == 0xFFu || eb == 0xFFu) return iss_mul(a, b);
  float r;
  asm("mul.rn.ftz.f32 %0, %1, %2;" : "=f"(r) : "f"(__uint_as_float(a)), "f"(__uint_as_float(b)));
  const uint32_t bits = __float_as_uint(r);
  if ((bits & 0x7FFFFFFFu) == 0x00800000u) return iss_mul(a, b);
  return ((bits >> 23) & 0xFFu) == 0 ? 0u : bits;
}

__device__ __forceinline__ uint32_t gacc_add(uint32_t acc, uint32_t p) {
  if (((acc >> 23) & 0xFFu) == 0xFFu || ((p >> 23) & 0xFFu) == 0xFFu) return iss_add(acc, p);
  return __float_as_uint(add_rn_ftz(__uint_as_float(acc), __uint_as_float(p)));
}

// ScaleCoefficient (dma_engine.cpp:516-528).
__device__ __forceinline__ uint32_t scale_coefficient(uint32_t c, uint32_t scale) {
  const uint32_t field = (c >> 23) & 0xFFu;
  const int32_t e = static_cast<int32_t>(field + scale) - 133;
  if (field == 0 || e <= 0) return 0u;
  const uint32_t sign = c & 0x80000000u;
  if (e >= 255) return sign | 0x7F7FFFFFu;
  return sign | (static_cast<uint32_t>(e) << 23) | (c & 0x7FFFFFu);
}

// Int8ToFp32 (dma_engine.cpp:504-514) is the exact conversion.
__device__ __forceinline__ uint32_t int8_bits(uint32_t byte) {
  return __float_as_uint(static_cast<float>(static_cast<int8_t>(byte)));
}

constexpr uint32_t kNull = 0xFFFFFFFFu;

__global__ void __launch_bounds__(256)
    k_gacc(const GaccJob j, uint32_t* __restrict__ error_flag) {
  const uint32_t lane = threadIdx.x & 31u;
  const uint32_t octets = (j.blocks + 7u) / 8u;
  const uint64_t warps = static_cast<uint64_t>(j.tokens) * octets;
  const uint64_t first = (static_cast<uint64_t>(blockIdx.x) * blockDim.x + threadIdx.x) >> 5;
  const uint64_t stride = (static_cast<uint64_t>(gridDim.x) * blockDim.x) >> 5;
  const uint32_t channels = j.blocks * 32u;
  for (uint64_t wi = first; wi < warps; wi += stride) {
    const uint32_t t = static_cast<uint32_t>(wi / octets), oct = static_cast<uint32_t>(wi % octets);
    const uint32_t b = oct * 8u + lane / 4u;  // this lane's block
    const bool mine = b < j.blocks;
    const uint32_t c0 = oct * 256u + lane * 8u;
    float* out = j.out + static_cast<size_t>(t) * channels + c0;
    uint32_t acc[8];
#pragma unroll
    for (uint32_t i = 0; i < 8; ++i) {
      acc[i] = (mine && j.accumulate) ? __float_as_uint(out[i]) : 0u;
    }
    const uint64_t* list = j.entries + static_cast<size_t>(t) * j.slots * j.corners;
    const uint32_t* wt = j.w + static_cast<size_t>(t) * j.slots * j.blocks;
    const uint32_t n = j.slots * j.corners;
    bool bad = false;
    uint64_t next = n != 0 ? __ldg(list) : 0;
    for (uint32_t e = 0; e < n; ++e) {
      const uint64_t entry = next;
      if (e + 1 < n) next = __ldg(list + e + 1);
      const uint32_t index = static_cast<uint32_t>(entry);
      if (index == kNull) continue;
      if (index >= j.nrows) {  // an address outside the feature rows
        bad = true;
        continue;
      }
      const uint8_t* row = j.rows + static_cast<uint64_t>(index) * j.row_stride;
      if (!mine) continue;
      const uint2 q = __ldg(reinterpret_cast<const uint2*>(row + c0));
      const uint32_t scale = row[channels + b];
      const uint32_t s = e / j.corners;
      const uint32_t coef =
          scale_coefficient(gacc_mul(__ldg(wt + static_cast<size_t>(s) * j.blocks + b),
                                     static_cast<uint32_t>(entry >> 32)),
                            scale);
#pragma unroll
      for (uint32_t i = 0; i < 8; ++i) {
        const uint32_t byte = ((i < 4 ? q.x : q.y) >> (8u * (i % 4u))) & 0xFFu;
        acc[i] = gacc_add(acc[i], gacc_mul(int8_bits(byte), coef));
      }
    }
    if (mine) {
#pragma unroll
      for (uint32_t i = 0; i < 8; ++i) {
        // The ISS's zero is +0.
        out[i] = __uint_as_float((acc[i] & 0x7FFFFFFFu) == 0 ? 0u : acc[i]);
      }
    }
    if (__any_sync(0xFFFFFFFFu, bad) && lane == 0) atomicOr(error_flag, 4u);
  }
}

}  // namespace

void launch_gacc(const GaccJob& job, uint32_t* error_flag, int sm_count, cudaStream_t stream) {
  const uint64_t warps = static_cast<uint64_t>(job.tokens) * ((job.blocks + 7u) / 8u);
  uint64_t grid = (warps + 7u) / 8u;
  const uint64_t cap = static_cast<uint64_t>(sm_count > 0 ? sm_count : 148) * 16u;
  if (grid > cap) grid = cap;
  k_gacc<<<static_cast<unsigned>(grid ? grid : 1), 256, 0, stream>>>(job, error_flag);
}

}  // namespace hrb
