// Convolution as hotarubi's compiler lowers it (ConvEmitter,
// tools/compiler/sparsedrive_encoder.cpp): one GEMM per (channel plane, tap)
// over activation rows gathered per tap ("faces", :114-168; a position
// outside the map is the DMA engine's null entry, a zero token with scale
// byte 127, tools/iss/dma_engine.cpp:247-256), all chaining into the same
// outputs (:384-398), then ADDP of the bias and optionally RELU (:399-420).
// Here that is one GEMM over K = (plane, tap, channel in plane) whose
// activation rows are gathered:
//
//   * tensor-core path: the input map is encoded once into its own operand
//     blocks (the digit planes of hrb_tc.cuh, one row per position), and
//     k_conv_gather_tiles assembles the GEMM's operand blocks from them, one
//     32-element block (16 or 32 bytes per plane and a scale byte) at a time:
//     every input element is encoded once, not once per tap;
//   * exact path: k_conv_im2col gathers the MXINT8 map's rows into the dense
//     activations of the exact chain.
//
// Weights arrive as the conv matrix [cout][kh * kh * cin] with tap-major
// columns (ConvTile, tools/compiler/sparsedrive_common.cpp:136-158); with
// more than one channel plane they are reordered to the chain's K order once
// (k_conv_weights).
#include <cstdint>

#include "hrb_device.cuh"
#include "hrb_kernels.cuh"
#include "hrb_tc.cuh"

namespace hrb {
namespace {

unsigned grid_of(uint64_t n) {
  uint64_t g = (n + 255) / 256;
  if (g > 148u * 16u) g = 148u * 16u;
  return static_cast<unsigned>(g ? g : 1);
}

// One thread per (output row, gathered K block): 32 codes (two 16-byte
// loads) and the scale byte, or zeros and scale 127 outside the map.
__global__ void k_conv_im2col(const int8_t* __restrict__ aq, const uint8_t* __restrict__ as,
                              const ConvGeom g, int8_t* __restrict__ q,
                              uint8_t* __restrict__ scale) {
  const uint32_t kbi = g.cin / 32u;
  const uint64_t rows = static_cast<uint64_t>(g.images) * g.Ho * g.Wo;
  const uint64_t total = rows * g.kbo;
  for (uint64_t i = blockIdx.x * static_cast<uint64_t>(blockDim.x) + threadIdx.x; i < total;
       i += static_cast<uint64_t>(gridDim.x) * blockDim.x) {
    const uint64_t row64 = i / g.kbo;
    const uint32_t row = static_cast<uint32_t>(row64), b = static_cast<uint32_t>(i - row64 * g.kbo);
    uint32_t ib = 0;
    const int64_t src = conv_source_block(g, row, b, &ib);
    uint4 lo = make_uint4(0, 0, 0, 0), hi = lo;
    uint8_t s = 127;
    if (src >= 0) {
      const uint4* from = reinterpret_cast<const uint4*>(aq + (static_cast<size_t>(src) * kbi + ib) * 32u);
      lo = __ldg(from);
      hi = __ldg(from + 1);
      s = as[static_cast<size_t>(src) * kbi + ib];
    }
    uint4* to = reinterpret_cast<uint4*>(q + i * 32u);
    to[0] = lo;
    to[1] = hi;
    scale[i] = s;
  }
}

// One thread per (weight row, K block): the block of chain position b is
// conv-matrix block tap * cin / 32 + plane * bp + channel block.
__global__ void k_conv_weights(const uint8_t* __restrict__ w, const uint8_t* __restrict__ ws,
                               uint32_t N, const ConvGeom g, uint32_t bpb,
                               uint8_t* __restrict__ out_w, uint8_t* __restrict__ out_ws) {
  const uint32_t kbi = g.cin / 32u, taps = g.kh * g.kh, kbo = taps * kbi;
  const uint64_t total = static_cast<uint64_t>(N) * kbo;
  for (uint64_t i = blockIdx.x * static_cast<uint64_t>(blockDim.x) + threadIdx.x; i < total;
       i += static_cast<uint64_t>(gridDim.x) * blockDim.x) {
    const uint64_t n = i / kbo;
    const uint32_t b = static_cast<uint32_t>(i % kbo);
    const uint32_t per_plane = taps * g.bp;
    const uint32_t plane = b / per_plane, rem = b - plane * per_plane;
    const uint32_t tap = rem / g.bp, cb = rem - tap * g.bp;
    const uint64_t src = n * kbo + tap * kbi + plane * g.bp + cb;
    const uint4* from = reinterpret_cast<const uint4*>(w + src * bpb);
    uint4* to = reinterpret_cast<uint4*>(out_w + i * bpb);
    to[0] = __ldg(from);
    if (bpb == 32u) to[1] = __ldg(from + 1);
    out_ws[i] = ws[src];
  }
}

// The VEC RELU pass (post op kMax against +0 then + 0, tools/iss/lane.cpp:
// 57-70,322-326): x unless x is negative with a nonzero magnitude, else +0,
// through the reference's FP32 adder.
__global__ void k_relu_exact(float* __restrict__ c, uint32_t M, uint32_t N, uint32_t ldc) {
  const uint64_t total = static_cast<uint64_t>(M) * N;
  for (uint64_t i = blockIdx.x * static_cast<uint64_t>(blockDim.x) + threadIdx.x; i < total;
       i += static_cast<uint64_t>(gridDim.x) * blockDim.x) {
    float* p = c + (i / N) * ldc + i % N;
    const uint32_t x = __float_as_uint(*p);
    const bool keep = (x >> 31) == 0 || (x & 0x7FFFFFFFu) == 0;
    *p = __uint_as_float(iss_add(keep ? x : 0u, 0u));
  }
}

// One thread per (output row, gathered K block).  Per digit plane the
// block's 16 (E2M1) or 32 (E4M3) bytes move from the source position's row
// to the output row's, each 16-byte chunk re-swizzled (stored chunk
// = logical chunk ^ row % 8 on both sides), and its scale byte with it; a
// block outside the map becomes zeros with scale byte 0.
__global__ void k_conv_gather_tiles(const uint8_t* __restrict__ map_tiles, uint32_t map_nt,
                                    uint32_t map_steps, uint8_t* __restrict__ tiles, uint32_t nt,
                                    uint32_t steps, uint32_t f8, const ConvGeom g) {
  const uint32_t bps = f8 ? 4u : 8u;        // blocks per K step
  const uint32_t bps_shift = f8 ? 2u : 3u;
  const uint32_t nt_shift = nt == 64u ? 6u : 7u, map_shift = map_nt == 64u ? 6u : 7u;
  const uint32_t planes = f8 ? 2u : 3u;
  const uint32_t chunks = f8 ? 2u : 1u;     // 16-byte chunks per block and plane
  const uint32_t bb = f8 ? mx8_act_block_bytes(nt) : mx_act_block_bytes(nt);
  const uint32_t mbb = f8 ? mx8_act_block_bytes(map_nt) : mx_act_block_bytes(map_nt);
  // 32-bit indices (the launch keeps rows * kbo below 2^32).
  const uint32_t total = g.images * g.Ho * g.Wo * g.kbo;
  for (uint32_t i = blockIdx.x * blockDim.x + threadIdx.x; i < total; i += gridDim.x * blockDim.x) {
    const uint32_t row = fast_div(i, g.kbo_div), b = i - row * g.kbo;
    uint32_t ib = 0;
    const int64_t src = conv_source_block(g, row, b, &ib);
    // Tile heights (64 or 128) and blocks per step (4 or 8) are powers of 2.
    const uint32_t dr = row & (nt - 1u), db = b & (bps - 1u);
    uint8_t* dblk = tiles + (static_cast<size_t>(row >> nt_shift) * steps + (b >> bps_shift)) * bb;
    const uint8_t* sblk = nullptr;
    uint32_t sr = 0, sb = 0;
    if (src >= 0) {
      const uint32_t pos = static_cast<uint32_t>(src);
      sr = pos & (map_nt - 1u);
      sb = ib & (bps - 1u);
      sblk = map_tiles +
             (static_cast<size_t>(pos >> map_shift) * map_steps + (ib >> bps_shift)) * mbb;
    }
    for (uint32_t p = 0; p < planes; ++p) {
      for (uint32_t c = 0; c < chunks; ++c) {
        const uint32_t logical = db * chunks + c;
        uint4 v = make_uint4(0, 0, 0, 0);
        if (sblk != nullptr) {
          const uint32_t sl = sb * chunks + c;
          v = *reinterpret_cast<const uint4*>(sblk + (p * map_nt + sr) * 128u +
                                              ((sl ^ (sr & 7u)) << 4));
        }
        *reinterpret_cast<uint4*>(dblk + (p * nt + dr) * 128u + ((logical ^ (dr & 7u)) << 4)) = v;
      }
      const uint32_t dsf = f8 ? mx8_act_sf_offset(nt, p * nt + dr, db)
                              : mx_act_sf_offset(nt, p * nt + dr, db);
      uint8_t sf = 0;
      if (sblk != nullptr) {
        sf = sblk[f8 ? mx8_act_sf_offset(map_nt, p * map_nt + sr, sb)
                     : mx_act_sf_offset(map_nt, p * map_nt + sr, sb)];
      }
      dblk[dsf] = sf;
    }
  }
}

}  // namespace

void launch_conv_gather_tiles(const uint8_t* map_tiles, uint32_t map_nt, uint32_t map_steps,
                              uint8_t* tiles, uint32_t nt, uint32_t steps, uint32_t f8,
                              const ConvGeom& g, cudaStream_t stream) {
  const uint64_t total =
      static_cast<uint64_t>(g.images) * g.Ho * g.Wo * (g.kh * g.kh * g.cin / 32u);
  k_conv_gather_tiles<<<grid_of(total), 256, 0, stream>>>(map_tiles, map_nt, map_steps, tiles, nt,
                                                          steps, f8, g);
}

void launch_conv_im2col(const int8_t* aq, const uint8_t* ascale, const ConvGeom& g, int8_t* q,
                        uint8_t* scale, cudaStream_t stream) {
  const uint64_t total =
      static_cast<uint64_t>(g.images) * g.Ho * g.Wo * (g.kh * g.kh * g.cin / 32u);
  k_conv_im2col<<<grid_of(total), 256, 0, stream>>>(aq, ascale, g, q, scale);
}

void launch_conv_weights(const uint8_t* w, const uint8_t* ws, uint32_t N, const ConvGeom& g,
                         uint32_t bytes_per_block, uint8_t* out_w, uint8_t* out_ws,
                         cudaStream_t stream) {
  const uint64_t total = static_cast<uint64_t>(N) * (g.kh * g.kh * g.cin / 32u);
  k_conv_weights<<<grid_of(total), 256, 0, stream>>>(w, ws, N, g, bytes_per_block, out_w, out_ws);
}

void launch_relu_exact(float* c, uint32_t M, uint32_t N, uint32_t ldc, cudaStream_t stream) {
  k_relu_exact<<<grid_of(static_cast<uint64_t>(M) * N), 256, 0, stream>>>(c, M, N, ldc);
}

}  // namespace hrb
