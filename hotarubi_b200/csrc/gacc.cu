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
// (8 bytes per lane, one 256-byte span) and the scale bytes.  Entries go in
// chunks of eight: a chunk's gathers are issued together, one chunk ahead of
// the adds, and the entry list is read a chunk ahead of the gathers.  With
// one chain per (token, 256 channels) and nothing to split a chain, the
// kernel is bound by the issue latency of few long chains (928 warps for
// SparseDrive's detection head).
// Gather (latency) bound: one random row of blocks * 33 bytes per entry.
//
// Arithmetic: FP32 multiplies and adds run on the FMA pipe with flush to
// zero, which for finite normal operands gives the ISS's results except in
// three places handled here: a zero result's sign (the ISS always gives +0:
// outputs are made +0 at the end), an exponent field of 255 (the ISS reads
// it as an ordinary exponent: a lane whose chain ends at exponent 255 redoes
// it with the integer restatements iss_mul / iss_add), and a product just
// under the normal range that the hardware rounds up to 2^-126 before
// flushing while the ISS rounds to 24 bits first (w * bw equal to +-2^-126
// is recomputed with iss_mul; int8 x coefficient products cannot land
// there).
#include <cstdint>

#include "hrb_device.cuh"
#include "hrb_kernels.cuh"

namespace hrb {
namespace {

__device__ __forceinline__ uint32_t gacc_mul(uint32_t a, uint32_t b) { return iss_mul_fast(a, b); }

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
constexpr uint32_t kAhead = 8;  // entries whose loads are in flight together
constexpr uint32_t kLaneCh = 8;                     // channels per lane
constexpr uint32_t kWarpBlocks = 32 * kLaneCh / 32;  // 32-channel blocks per warp

// One lane's eight accumulators over the whole chain with the integer
// restatements of the ISS's multiply and add: the rare path, taken when the
// FMA-pipe chain reached an exponent field of 255 (an overflow, or an
// infinity or NaN read from the coefficients).
__device__ __noinline__ void gacc_chain_exact(const GaccJob& j, uint32_t t, uint32_t b,
                                              uint32_t c0, uint32_t (&acc)[kLaneCh]) {
  const uint32_t channels = j.blocks * 32u;
  const float* out = j.out + static_cast<size_t>(t) * channels + c0;
#pragma unroll
  for (uint32_t i = 0; i < kLaneCh; ++i) acc[i] = j.accumulate ? __float_as_uint(out[i]) : 0u;
  const uint64_t* list = j.entries + static_cast<size_t>(t) * j.slots * j.corners;
  const uint32_t* wt = j.w + static_cast<size_t>(t) * j.slots * j.blocks;
  for (uint32_t e = 0; e < j.slots * j.corners; ++e) {
    const uint64_t entry = list[e];
    const uint32_t index = static_cast<uint32_t>(entry);
    if (index == kNull || index >= j.nrows) continue;
    const uint8_t* row = j.rows + static_cast<uint64_t>(index) * j.row_stride;
    const uint32_t coef = scale_coefficient(
        iss_mul(wt[static_cast<size_t>(e / j.corners) * j.blocks + b],
                static_cast<uint32_t>(entry >> 32)),
        row[channels + b]);
#pragma unroll
    for (uint32_t i = 0; i < kLaneCh; ++i) {
      acc[i] = iss_add(acc[i], iss_mul(int8_bits(row[c0 + i]), coef));
    }
  }
}

__global__ void __launch_bounds__(256)
    k_gacc(const GaccJob j, uint32_t* __restrict__ error_flag) {
  const uint32_t lane = threadIdx.x & 31u;
  const uint32_t groups = (j.blocks + kWarpBlocks - 1u) / kWarpBlocks;
  const uint64_t warps = static_cast<uint64_t>(j.tokens) * groups;
  const uint64_t first = (static_cast<uint64_t>(blockIdx.x) * blockDim.x + threadIdx.x) >> 5;
  const uint64_t stride = (static_cast<uint64_t>(gridDim.x) * blockDim.x) >> 5;
  const uint32_t channels = j.blocks * 32u;
  for (uint64_t wi = first; wi < warps; wi += stride) {
    const uint32_t t = static_cast<uint32_t>(wi / groups), grp = static_cast<uint32_t>(wi % groups);
    const uint32_t b = grp * kWarpBlocks + lane / (32u / kLaneCh);  // this lane's block
    const bool mine = b < j.blocks;
    const uint32_t c0 = grp * kWarpBlocks * 32u + lane * kLaneCh;
    float* out = j.out + static_cast<size_t>(t) * channels + c0;
    float acc[kLaneCh];
#pragma unroll
    for (uint32_t i = 0; i < kLaneCh; ++i) acc[i] = (mine && j.accumulate) ? out[i] : 0.0f;
    const uint64_t* list = j.entries + static_cast<size_t>(t) * j.slots * j.corners;
    const uint32_t* wt = j.w + static_cast<size_t>(t) * j.slots * j.blocks;
    const uint32_t n = j.slots * j.corners;
    bool bad = false;
    // Entries in chunks of kAhead: a chunk's rows, scales and coefficients
    // are all loaded (independent loads in flight together) before its
    // entries are added in order.
    struct Chunk {
      uint64_t cur[kAhead];
      uint32_t q[kAhead][kLaneCh / 4];
      uint32_t sc[kAhead], wv[kAhead];
    };
    uint64_t ent[kAhead];
#pragma unroll
    for (uint32_t u = 0; u < kAhead; ++u) ent[u] = u < n ? __ldg(list + u) : kNull;
    // Issues chunk `e0`'s gathers from `ent` into c, then reads the list
    // entries of the chunk after it into `ent`.
    auto issue = [&](Chunk& c, uint32_t e0) {
#pragma unroll
      for (uint32_t u = 0; u < kAhead; ++u) {
        const uint32_t index = static_cast<uint32_t>(ent[u]);
        c.cur[u] = ent[u];
        c.q[u][0] = 0;
        c.q[u][kLaneCh / 4 - 1] = 0;
        c.sc[u] = 0;
        c.wv[u] = 0;
        if (mine && index != kNull && index < j.nrows) {
          const uint8_t* row = j.rows + static_cast<uint64_t>(index) * j.row_stride;
          const uint2 v = __ldg(reinterpret_cast<const uint2*>(row + c0));
          c.q[u][0] = v.x;
          c.q[u][kLaneCh / 4 - 1] = v.y;
          c.sc[u] = row[channels + b];
          c.wv[u] = __ldg(wt + static_cast<size_t>((e0 + u) / j.corners) * j.blocks + b);
        }
      }
#pragma unroll
      for (uint32_t u = 0; u < kAhead; ++u) {
        ent[u] = e0 + kAhead + u < n ? __ldg(list + e0 + kAhead + u) : kNull;
      }
    };
    auto add = [&](const Chunk& c) {
#pragma unroll
      for (uint32_t u = 0; u < kAhead; ++u) {
        const uint32_t index = static_cast<uint32_t>(c.cur[u]);
        if (index == kNull) continue;
        if (index >= j.nrows) {  // an address outside the feature rows
          bad = true;
          continue;
        }
        if (!mine) continue;
        const uint32_t coef =
            scale_coefficient(gacc_mul(c.wv[u], static_cast<uint32_t>(c.cur[u] >> 32)), c.sc[u]);
        if (coef == 0) continue;  // every product is a zero: the chain keeps its values
        const float cf = __uint_as_float(coef);
#pragma unroll
        for (uint32_t i = 0; i < kLaneCh; ++i) {
          const uint32_t byte = (c.q[u][i / 4u] >> (8u * (i % 4u))) & 0xFFu;
          float p;
          asm("mul.rn.ftz.f32 %0, %1, %2;"
              : "=f"(p)
              : "f"(static_cast<float>(static_cast<int8_t>(byte))), "f"(cf));
          acc[i] = add_rn_ftz(acc[i], p);
        }
      }
    };
    // Two chunks in flight: the next chunk's gathers are issued before this
    // one's adds.
    Chunk ca, cb;
    issue(ca, 0);
    for (uint32_t e0 = 0; e0 < n; e0 += 2 * kAhead) {
      const bool second = e0 + kAhead < n;
      if (second) issue(cb, e0 + kAhead);
      add(ca);
      if (e0 + 2 * kAhead < n) issue(ca, e0 + 2 * kAhead);
      if (second) add(cb);
    }
    if (mine) {
      uint32_t bits[kLaneCh];
      bool wide = false;
#pragma unroll
      for (uint32_t i = 0; i < kLaneCh; ++i) {
        bits[i] = __float_as_uint(acc[i]);
        wide |= ((bits[i] >> 23) & 0xFFu) == 0xFFu;
      }
      if (wide) gacc_chain_exact(j, t, b, c0, bits);
#pragma unroll
      for (uint32_t i = 0; i < kLaneCh; ++i) {
        // The ISS's zero is +0.
        out[i] = __uint_as_float((bits[i] & 0x7FFFFFFFu) == 0 ? 0u : bits[i]);
      }
    }
    if (__any_sync(0xFFFFFFFFu, bad) && lane == 0) atomicOr(error_flag, 4u);
  }
}

}  // namespace

void launch_gacc(const GaccJob& job, uint32_t* error_flag, int sm_count, cudaStream_t stream) {
  const uint64_t warps =
      static_cast<uint64_t>(job.tokens) * ((job.blocks + kWarpBlocks - 1u) / kWarpBlocks);
  uint64_t grid = (warps + 7u) / 8u;
  const uint64_t cap = static_cast<uint64_t>(sm_count > 0 ? sm_count : 148) * 16u;
  if (grid > cap) grid = cap;
  k_gacc<<<static_cast<unsigned>(grid ? grid : 1), 256, 0, stream>>>(job, error_flag);
}

}  // namespace hrb
