// Test infrastructure only.  This file is compiled together with hotarubi's
// own sources (left where they lie in the reference checkout) into
// oracle/_ref/libhrb_ref.so.  It gives the Python tests a C entry point to
// the reference's GEMM executor and its helpers so that they can check the
// C restatement in oracle/hrb_oracle.c and generate the golden fixtures.  The
// product never links or loads it.
//
// Each wrapper names the reference function it calls.
#include <algorithm>
#include <cstddef>
#include <cstdint>
#include <cstring>
#include <atomic>
#include <memory>
#include <random>
#include <thread>
#include <span>
#include <vector>

#include "ddr.hpp"             // tools/iss/ddr.hpp
#include "dma_engine.hpp"      // tools/iss/dma_engine.hpp
#include "fp32.hpp"            // tools/iss/fp32.hpp
#include "gemm_array.hpp"      // tools/iss/gemm_array.hpp
#include "hotarubi/exact.hpp"  // include/hotarubi/exact.hpp
#include "hotarubi/formats.hpp"
#include "hotarubi/json.hpp"  // include/hotarubi/json.hpp
#include "lane.hpp"       // tools/iss/lane.hpp
#include "memories.hpp"   // tools/iss/memories.hpp
#include "reference.hpp"  // tools/iss/reference.hpp
#include "timing.hpp"     // tools/iss/timing.hpp
#include "tensors.hpp"    // tools/compiler/tensors.hpp
#include "weights.hpp"    // tools/compiler/weights.hpp

#include "tb_types.hpp"

// Declarations of tb/fp32_ref.hpp and tb/gemm_ref.hpp, restated because the
// real headers include the Verilator-dependent word headers.
namespace hotarubi::tb {
uint32_t Fp32Add(uint32_t a, uint32_t b);
void ReferenceGemm(const GemmArgs& args, const std::vector<AbufWord>& abuf,
                   const std::vector<WbufWord>& wbuf,
                   std::vector<FbufWord>& fbuf);
}  // namespace hotarubi::tb

namespace {

using hotarubi::iss::GemmCommand;
using hotarubi::iss::Memories;

GemmCommand Command(const uint32_t* f) {
  return {.a_base = f[0],
          .a_stride = f[1],
          .kb = f[2],
          .m = f[3],
          .w_base = f[4],
          .w_stride = f[5],
          .n8 = f[6],
          .c_base = f[7],
          .wmode = f[8],
          .acc = f[9] != 0};
}

template <size_t N>
void StoreBits(const std::bitset<N>& bits, uint8_t* out) {
  for (size_t i = 0; i < N; ++i) {
    out[i] = bits.test(i) ? 1 : 0;
  }
}

}  // namespace

extern "C" {

// hotarubi::iss::ExecuteGemm (tools/iss/gemm_array.cpp:112-149) on a full set
// of GEMM memories.  abuf: 8192 words of 132 bytes, wbuf: 2048 words of 144
// bytes, fbuf: 4096 words of 32 FP32 bit patterns (updated in place).  When
// log is not null it receives one byte per word: ABUF reads [8192], WBUF
// reads [2048], FBUF reads [4096], FBUF writes [4096].
void hrbref_execute_gemm(const uint32_t* fields, const uint8_t* abuf,
                         const uint8_t* wbuf, uint32_t* fbuf, uint8_t* log) {
  static Memories memories;
  memories.log.Clear();
  for (size_t i = 0; i < hotarubi::iss::kAbufDepth; ++i) {
    std::memcpy(memories.abuf[i].data(), abuf + (i * 132), 132);
  }
  for (size_t i = 0; i < hotarubi::iss::kWbufDepth; ++i) {
    std::memcpy(memories.wbuf[i].data(), wbuf + (i * 144), 144);
  }
  for (size_t i = 0; i < hotarubi::iss::kFbufDepth; ++i) {
    std::memcpy(memories.fbuf[i].data(), fbuf + (i * 32), 128);
  }
  hotarubi::iss::ExecuteGemm(Command(fields), memories);
  for (size_t i = 0; i < hotarubi::iss::kFbufDepth; ++i) {
    std::memcpy(fbuf + (i * 32), memories.fbuf[i].data(), 128);
  }
  if (log != nullptr) {
    StoreBits(memories.log.reads.abuf, log);
    StoreBits(memories.log.reads.wbuf, log + 8192);
    StoreBits(memories.log.reads.fbuf, log + 8192 + 2048);
    StoreBits(memories.log.writes.fbuf, log + 8192 + 2048 + 4096);
  }
}

// hotarubi::tb::ReferenceGemm (tb/gemm_ref.cpp:47-68).  Word arrays use the
// DDR word layout of 144 bytes (tb/npu_data.cpp): ABUF bytes 0..127 int8,
// 128..131 scales; WBUF bytes 0..127 packed nibbles (low nibble first),
// 128..135 scales.
void hrbref_reference_gemm(const uint32_t* fields, const uint8_t* abuf,
                           uint32_t a_words, const uint8_t* wbuf,
                           uint32_t w_words, uint32_t* fbuf, uint32_t f_words) {
  std::vector<hotarubi::tb::AbufWord> a(a_words);
  std::vector<hotarubi::tb::WbufWord> w(w_words);
  std::vector<hotarubi::tb::FbufWord> c(f_words);
  for (uint32_t i = 0; i < a_words; ++i) {
    std::memcpy(a[i].q.data(), abuf + (size_t{i} * 144), 128);
    std::memcpy(a[i].scale.data(), abuf + (size_t{i} * 144) + 128, 4);
  }
  for (uint32_t i = 0; i < w_words; ++i) {
    const uint8_t* word = wbuf + (size_t{i} * 144);
    for (uint32_t n = 0; n < 256; ++n) {
      w[i].nibble[n] = (word[n / 2] >> (4 * (n % 2))) & 0xFU;
    }
    std::memcpy(w[i].scale.data(), word + 128, 8);
  }
  for (uint32_t i = 0; i < f_words; ++i) {
    std::memcpy(c[i].data(), fbuf + (size_t{i} * 32), 128);
  }
  const hotarubi::tb::GemmArgs args{.a_base = fields[0],
                                    .a_stride = fields[1],
                                    .kb = fields[2],
                                    .m = fields[3],
                                    .w_base = fields[4],
                                    .w_stride = fields[5],
                                    .n8 = fields[6],
                                    .c_base = fields[7],
                                    .wmode = fields[8],
                                    .acc = fields[9] != 0};
  hotarubi::tb::ReferenceGemm(args, a, w, c);
  for (uint32_t i = 0; i < f_words; ++i) {
    std::memcpy(fbuf + (size_t{i} * 32), c[i].data(), 128);
  }
}

// tools/iss/fp32.hpp:46-75
uint32_t hrbref_fp32_add(uint32_t a, uint32_t b) {
  return hotarubi::iss::Fp32Add(a, b);
}

// tb/fp32_ref.cpp:64-88
uint32_t hrbref_tb_fp32_add(uint32_t a, uint32_t b) {
  return hotarubi::tb::Fp32Add(a, b);
}

// tools/iss/reference.cpp: exact-real model of the FP32 adder.
uint32_t hrbref_exact_add(uint32_t a, uint32_t b) {
  return hotarubi::iss::reference::Add(a, b);
}

// reference::Round(Integer(sum) * 2^exponent): the exact model the ISS unit
// test uses for one block product (tools/iss/gemm_array_test.cpp:91-98).
uint32_t hrbref_exact_round(int64_t sum, int64_t exponent) {
  return hotarubi::iss::reference::Round(
      hotarubi::exact::Real::Integer(sum).Scaled(exponent));
}

// tools/iss/gemm_array.cpp:84-97 and :99-110
int32_t hrbref_weight_value(uint32_t nibble, uint32_t wmode) {
  return hotarubi::iss::WeightValue(nibble,
                                    hotarubi::iss::DecodeWeightMode(wmode));
}

uint32_t hrbref_block_value(int32_t sum, uint32_t a_scale, uint32_t w_scale,
                            uint32_t wmode) {
  return hotarubi::iss::BlockValue(sum, a_scale, w_scale,
                                   hotarubi::iss::DecodeWeightMode(wmode));
}

// hotarubi::EncodeMxint8 (tools/runtime/formats.cpp:138-162).  bits is a
// rows x cols FP32 matrix; q receives rows x padded-cols int8 and e receives
// rows x blocks exponents (scale byte = e + 127).
void hrbref_encode_mxint8(const uint32_t* bits, uint32_t rows, uint32_t cols,
                          int8_t* q, int32_t* e) {
  hotarubi::Matrix m{.rows = rows,
                     .cols = cols,
                     .bits = std::vector<uint32_t>(
                         bits, bits + (static_cast<size_t>(rows) * cols))};
  const hotarubi::Mxint8Matrix out = hotarubi::EncodeMxint8(m);
  std::copy(out.q.begin(), out.q.end(), q);
  std::copy(out.e.begin(), out.e.end(), e);
}

// hotarubi::PackAbuf (tools/runtime/formats.cpp:114-136): 144-byte words.
void hrbref_pack_abuf(const int8_t* q, const int32_t* e, uint32_t rows,
                      uint32_t cols, uint8_t* out) {
  const size_t blocks = cols / 32;
  hotarubi::Mxint8Matrix m{
      .rows = rows,
      .cols = cols,
      .q = std::vector<int8_t>(q, q + (static_cast<size_t>(rows) * cols)),
      .e = std::vector<int32_t>(e, e + (rows * blocks))};
  const std::vector<std::byte> bytes = hotarubi::PackAbuf(m);
  std::memcpy(out, bytes.data(), bytes.size());
}

// hotarubi::iss::QuantizeBlock (tools/iss/lane.cpp:406-423): four FBUF words
// (32 FP32 each) -> one 132-byte ABUF word, the VEC 'q' pass.
void hrbref_quantize_block(const uint32_t* words, uint8_t* out) {
  std::array<hotarubi::iss::FbufWord, 4> in{};
  for (size_t i = 0; i < 4; ++i) {
    std::memcpy(in[i].data(), words + (i * 32), 128);
  }
  const hotarubi::iss::AbufWord word =
      hotarubi::iss::QuantizeBlock(std::span<const hotarubi::iss::FbufWord, 4>(in));
  std::memcpy(out, word.data(), word.size());
}

// hotarubi::compiler::CanonicalMxfp4 (tools/compiler/weights.cpp:39-70).
void hrbref_canonical_mxfp4(const uint8_t* code, const int32_t* e,
                            uint32_t rows, uint32_t cols, int32_t shift,
                            uint32_t out_rows, uint8_t* code_out,
                            int32_t* e_out) {
  const size_t blocks = cols / 32;
  hotarubi::compiler::Mxfp4Matrix m{
      .rows = rows,
      .cols = cols,
      .code = std::vector<uint8_t>(code, code + (static_cast<size_t>(rows) * cols)),
      .e = std::vector<int32_t>(e, e + (rows * blocks))};
  const hotarubi::compiler::Mxfp4Matrix out =
      hotarubi::compiler::CanonicalMxfp4(m, shift, out_rows);
  std::copy(out.code.begin(), out.code.end(), code_out);
  std::copy(out.e.begin(), out.e.end(), e_out);
}

// hotarubi::compiler::SplitW8 (tools/compiler/weights.cpp:72-88).
void hrbref_split_w8(const int8_t* q, uint32_t rows, uint32_t cols,
                     uint8_t* hi, uint8_t* lo) {
  hotarubi::Mxint8Matrix m{
      .rows = rows,
      .cols = cols,
      .q = std::vector<int8_t>(q, q + (static_cast<size_t>(rows) * cols)),
      .e = std::vector<int32_t>(static_cast<size_t>(rows) * (cols / 32))};
  const hotarubi::compiler::W8Planes planes = hotarubi::compiler::SplitW8(m);
  std::copy(planes.hi.code.begin(), planes.hi.code.end(), hi);
  std::copy(planes.lo.code.begin(), planes.lo.code.end(), lo);
}

// hotarubi::compiler::PackWbuf (tools/compiler/tensors.cpp:66-90).
void hrbref_pack_wbuf(const uint8_t* code, const int32_t* e, uint32_t rows,
                      uint32_t cols, uint8_t* out) {
  const size_t blocks = cols / 32;
  hotarubi::compiler::Mxfp4Matrix m{
      .rows = rows,
      .cols = cols,
      .code = std::vector<uint8_t>(code, code + (static_cast<size_t>(rows) * cols)),
      .e = std::vector<int32_t>(e, e + (rows * blocks))};
  const std::vector<std::byte> bytes = hotarubi::compiler::PackWbuf(m);
  std::memcpy(out, bytes.data(), bytes.size());
}

// Element-wise array forms of the three adders and of the exact rounding.
void hrbref_fp32_add_n(const uint32_t* a, const uint32_t* b, uint32_t* out,
                       size_t n) {
  for (size_t i = 0; i < n; ++i) out[i] = hotarubi::iss::Fp32Add(a[i], b[i]);
}

// tools/iss/fp32.hpp:77-92
void hrbref_fp32_mul_n(const uint32_t* a, const uint32_t* b, uint32_t* out,
                       size_t n) {
  for (size_t i = 0; i < n; ++i) out[i] = hotarubi::iss::Fp32Mul(a[i], b[i]);
}

void hrbref_tb_fp32_add_n(const uint32_t* a, const uint32_t* b, uint32_t* out,
                          size_t n) {
  for (size_t i = 0; i < n; ++i) out[i] = hotarubi::tb::Fp32Add(a[i], b[i]);
}

void hrbref_exact_add_n(const uint32_t* a, const uint32_t* b, uint32_t* out,
                        size_t n) {
  for (size_t i = 0; i < n; ++i) out[i] = hotarubi::iss::reference::Add(a[i], b[i]);
}

void hrbref_exact_round_n(const int64_t* sum, const int32_t* exponent,
                          uint32_t* out, size_t n) {
  for (size_t i = 0; i < n; ++i) {
    out[i] = hotarubi::iss::reference::Round(
        hotarubi::exact::Real::Integer(sum[i]).Scaled(exponent[i]));
  }
}

// ---------------------------------------------------------------------------
// Input generators of the reference's own GEMM tests, restated so that the
// golden fixtures carry exactly the inputs those tests feed the reference.
// They draw from std::mt19937 with the same distributions in the same order.

// GemmArrayTest::Fill (tools/iss/gemm_array_test.cpp:45-70) over full
// memories (ABUF 8192 x 132, WBUF 2048 x 144, FBUF 4096 x 32).
void hrbref_fill_gemm_array_test(uint32_t seed, uint8_t* abuf, uint8_t* wbuf,
                                 uint32_t* fbuf) {
  std::mt19937 generator(seed);
  std::uniform_int_distribution<uint32_t> byte(0, 255);
  std::uniform_int_distribution<uint32_t> scale(118, 136);
  for (size_t w = 0; w < hotarubi::iss::kAbufDepth; ++w) {
    uint8_t* word = abuf + (w * 132);
    for (size_t i = 0; i < 128; ++i) word[i] = static_cast<uint8_t>(byte(generator));
    for (size_t t = 0; t < 4; ++t) word[128 + t] = static_cast<uint8_t>(scale(generator));
  }
  for (size_t w = 0; w < hotarubi::iss::kWbufDepth; ++w) {
    uint8_t* word = wbuf + (w * 144);
    for (size_t i = 0; i < 128; ++i) word[i] = static_cast<uint8_t>(byte(generator));
    for (size_t c = 0; c < 8; ++c) word[128 + c] = static_cast<uint8_t>(scale(generator));
    for (size_t i = 136; i < 144; ++i) word[i] = 0;
  }
  for (size_t w = 0; w < hotarubi::iss::kFbufDepth; ++w) {
    for (size_t e = 0; e < 32; ++e) {
      fbuf[(w * 32) + e] = 0x3F000000U + (byte(generator) << 16);
    }
  }
}

// RandomAbuf / RandomWbuf / RandomFbuf (tb/gemm_test.cpp:31-65) and
// RandomFp32 (tb/npu_data.cpp:112-118) on a caller-held generator.  The words
// use the 144-byte DDR layout.
void* hrbref_tb_rng_new(uint32_t seed) { return new std::mt19937(seed); }
void hrbref_tb_rng_free(void* rng) { delete static_cast<std::mt19937*>(rng); }

void hrbref_tb_random_abuf(void* handle, uint32_t count, uint8_t* out) {
  std::mt19937& rng = *static_cast<std::mt19937*>(handle);
  for (uint32_t w = 0; w < count; ++w) {
    uint8_t* word = out + (size_t{w} * 144);
    std::memset(word, 0, 144);
    for (size_t i = 0; i < 128; ++i) {
      word[i] = static_cast<uint8_t>(static_cast<int8_t>(static_cast<int>(rng() % 256) - 128));
    }
    for (size_t t = 0; t < 4; ++t) word[128 + t] = static_cast<uint8_t>(118 + (rng() % 18));
  }
}

void hrbref_tb_random_wbuf(void* handle, uint32_t count, uint8_t* out) {
  std::mt19937& rng = *static_cast<std::mt19937*>(handle);
  for (uint32_t w = 0; w < count; ++w) {
    uint8_t* word = out + (size_t{w} * 144);
    std::memset(word, 0, 144);
    for (size_t n = 0; n < 256; ++n) {
      const auto nibble = static_cast<uint8_t>(rng() % 16);
      word[n / 2] = static_cast<uint8_t>(word[n / 2] | (nibble << (4 * (n % 2))));
    }
    for (size_t c = 0; c < 8; ++c) word[128 + c] = static_cast<uint8_t>(118 + (rng() % 18));
  }
}

void hrbref_tb_random_fbuf(void* handle, uint32_t count, uint32_t* out) {
  std::mt19937& rng = *static_cast<std::mt19937*>(handle);
  for (uint32_t i = 0; i < count * 32; ++i) {
    const auto exponent = static_cast<uint32_t>(-6 + 127 + static_cast<int>(rng() % 13));
    const uint32_t sign = rng() & 1U;
    out[i] = (sign << 31) | (exponent << 23) | (rng() & 0x7FFFFFU);
  }
}

// ---------------------------------------------------------------------------
// The CPU baseline: a dense GEMM run through the reference's ExecuteGemm,
// tiled into legal GEMM instructions the way hotarubi's compiler tiles a
// Linear (one weight tile loaded per plane, planes accumulating in order,
// tools/compiler/kernels.cpp:343-395), with independent (row chunk, column
// tile) units spread over `threads` std::threads, each owning a Memories.
//
// a_words: PackAbuf words (144 bytes) of the rows, [ceil(M/4)][kb].
// planes: PackWbuf words of each plane, [N/8][kb] per plane, planes back to
// back (1 plane: FP4, mode 0; 2 planes: W8 HI then LO, modes 1 and 2).
// c: M x N FP32 bits, row-major.  Only rows [row0, row1) are computed;
// row0 must be a multiple of 4.  Returns 0, or -1 when kb does not fit.
int hrbref_dense_gemm_iss(uint32_t nplanes, uint32_t M, uint32_t N,
                          uint32_t kb, const uint8_t* a_words,
                          const uint8_t* planes, uint32_t* c, uint32_t threads,
                          uint32_t row0, uint32_t row1) {
  using hotarubi::iss::kAbufDepth;
  using hotarubi::iss::kFbufDepth;
  using hotarubi::iss::kWbufDepth;
  if (kb == 0 || kb > kWbufDepth || N % 8 != 0 || row0 % 4 != 0) return -1;
  const uint32_t groups_total = N / 8;
  uint32_t tile_groups = std::min<uint32_t>(255, kWbufDepth / kb);
  uint32_t chunk_quads = std::min<uint32_t>(248, kAbufDepth / kb);
  chunk_quads -= chunk_quads % 8;
  if (tile_groups == 0 || chunk_quads == 0) return -1;
  while (chunk_quads * tile_groups > kFbufDepth) {
    if (tile_groups > 8) {
      tile_groups /= 2;
    } else {
      chunk_quads -= 8;
    }
  }
  row1 = std::min(row1, M);
  if (row1 <= row0) return 0;
  const uint32_t quad0 = row0 / 4;
  const uint32_t quads = (row1 - row0 + 3) / 4;
  const uint32_t chunks = (quads + chunk_quads - 1) / chunk_quads;
  const uint32_t tiles = (groups_total + tile_groups - 1) / tile_groups;
  const size_t plane_bytes = size_t{groups_total} * kb * 144;
  std::atomic<uint32_t> next{0};
  auto worker = [&]() {
    auto memories = std::make_unique<Memories>();
    for (;;) {
      const uint32_t unit = next.fetch_add(1);
      if (unit >= chunks * tiles) break;
      const uint32_t chunk = unit / tiles;
      const uint32_t tile = unit % tiles;
      const uint32_t q_first = quad0 + chunk * chunk_quads;
      const uint32_t q_count = std::min(chunk_quads, quad0 + quads - q_first);
      const uint32_t m = ((q_count * 4) + 31) / 32 * 32;
      const uint32_t g_first = tile * tile_groups;
      const uint32_t g_count = std::min(tile_groups, groups_total - g_first);
      for (uint32_t q = 0; q < m / 4; ++q) {
        for (uint32_t b = 0; b < kb; ++b) {
          auto& word = memories->abuf[(q * kb) + b];
          if (q < q_count) {
            std::memcpy(word.data(), a_words + ((size_t{q_first + q} * kb) + b) * 144, 132);
          } else {
            std::fill(word.begin(), word.end(), 0);
          }
        }
      }
      for (uint32_t l = 0; l < nplanes; ++l) {
        for (uint32_t g = 0; g < g_count; ++g) {
          for (uint32_t b = 0; b < kb; ++b) {
            std::memcpy(memories->wbuf[(g * kb) + b].data(),
                        planes + (l * plane_bytes) + ((size_t{g_first + g} * kb) + b) * 144,
                        144);
          }
        }
        const GemmCommand command{.a_base = 0,
                                  .a_stride = kb,
                                  .kb = kb,
                                  .m = m,
                                  .w_base = 0,
                                  .w_stride = kb,
                                  .n8 = g_count,
                                  .c_base = 0,
                                  .wmode = nplanes == 1 ? 0U : l + 1,
                                  .acc = l > 0};
        hotarubi::iss::ExecuteGemm(command, *memories);
      }
      for (uint32_t q = 0; q < q_count; ++q) {
        for (uint32_t g = 0; g < g_count; ++g) {
          const auto& word = memories->fbuf[(q * g_count) + g];
          for (uint32_t t = 0; t < 4; ++t) {
            const uint32_t row = ((q_first + q) * 4) + t;
            if (row < row0 || row >= row1) continue;
            for (uint32_t col = 0; col < 8; ++col) {
              c[(size_t{row} * N) + ((g_first + g) * 8) + col] = word[(t * 8) + col];
            }
          }
        }
      }
      memories->log.Clear();
    }
  };
  std::vector<std::thread> pool;
  for (uint32_t t = 1; t < std::max<uint32_t>(threads, 1); ++t) pool.emplace_back(worker);
  worker();
  for (auto& thread : pool) thread.join();
  return 0;
}

// The same dense GEMM through tb/gemm_ref's ReferenceGemm (the model the
// RTL is checked against, tb/gemm_ref.cpp:47-68): one instruction per (row
// chunk, column tile) unit and plane, the instruction's words converted to
// the tb's word types (nibbles unpacked), on `threads` std::threads.  The
// tiling is hrbref_dense_gemm_iss's; all M rows are computed.
int hrbref_dense_gemm_tb(uint32_t nplanes, uint32_t M, uint32_t N, uint32_t kb,
                         const uint8_t* a_words, const uint8_t* planes, uint32_t* c,
                         uint32_t threads) {
  using hotarubi::iss::kAbufDepth;
  using hotarubi::iss::kFbufDepth;
  using hotarubi::iss::kWbufDepth;
  if (kb == 0 || kb > kWbufDepth || N % 8 != 0) return -1;
  const uint32_t groups_total = N / 8;
  uint32_t tile_groups = std::min<uint32_t>(255, kWbufDepth / kb);
  uint32_t chunk_quads = std::min<uint32_t>(248, kAbufDepth / kb);
  chunk_quads -= chunk_quads % 8;
  if (tile_groups == 0 || chunk_quads == 0) return -1;
  while (chunk_quads * tile_groups > kFbufDepth) {
    if (tile_groups > 8) {
      tile_groups /= 2;
    } else {
      chunk_quads -= 8;
    }
  }
  const uint32_t quads = (M + 3) / 4;
  const uint32_t chunks = (quads + chunk_quads - 1) / chunk_quads;
  const uint32_t tiles = (groups_total + tile_groups - 1) / tile_groups;
  const size_t plane_bytes = size_t{groups_total} * kb * 144;
  std::atomic<uint32_t> next{0};
  auto worker = [&]() {
    std::vector<hotarubi::tb::AbufWord> a;
    std::vector<hotarubi::tb::WbufWord> w;
    std::vector<hotarubi::tb::FbufWord> f;
    for (;;) {
      const uint32_t unit = next.fetch_add(1);
      if (unit >= chunks * tiles) break;
      const uint32_t q_first = (unit / tiles) * chunk_quads;
      const uint32_t q_count = std::min(chunk_quads, quads - q_first);
      const uint32_t m = ((q_count * 4) + 31) / 32 * 32;
      const uint32_t g_first = (unit % tiles) * tile_groups;
      const uint32_t g_count = std::min(tile_groups, groups_total - g_first);
      a.assign(size_t{m / 4} * kb, hotarubi::tb::AbufWord{});
      for (uint32_t q = 0; q < q_count; ++q) {
        for (uint32_t b = 0; b < kb; ++b) {
          const uint8_t* src = a_words + ((size_t{q_first + q} * kb) + b) * 144;
          std::memcpy(a[(q * kb) + b].q.data(), src, 128);
          std::memcpy(a[(q * kb) + b].scale.data(), src + 128, 4);
        }
      }
      f.assign(size_t{m / 4} * g_count, hotarubi::tb::FbufWord{});
      w.resize(size_t{g_count} * kb);
      for (uint32_t l = 0; l < nplanes; ++l) {
        for (uint32_t g = 0; g < g_count; ++g) {
          for (uint32_t b = 0; b < kb; ++b) {
            const uint8_t* src = planes + (l * plane_bytes) + ((size_t{g_first + g} * kb) + b) * 144;
            auto& word = w[(g * kb) + b];
            for (uint32_t n = 0; n < 256; ++n) word.nibble[n] = (src[n / 2] >> (4 * (n % 2))) & 0xFU;
            std::memcpy(word.scale.data(), src + 128, 8);
          }
        }
        const hotarubi::tb::GemmArgs args{.a_base = 0, .a_stride = kb, .kb = kb, .m = m,
                                          .w_base = 0, .w_stride = kb, .n8 = g_count,
                                          .c_base = 0, .wmode = nplanes == 1 ? 0U : l + 1,
                                          .acc = l > 0};
        hotarubi::tb::ReferenceGemm(args, a, w, f);
      }
      for (uint32_t q = 0; q < q_count; ++q) {
        for (uint32_t g = 0; g < g_count; ++g) {
          for (uint32_t t = 0; t < 4; ++t) {
            const uint32_t row = ((q_first + q) * 4) + t;
            if (row >= M) continue;
            for (uint32_t col = 0; col < 8; ++col) {
              c[(size_t{row} * N) + ((g_first + g) * 8) + col] = f[(q * g_count) + g][(t * 8) + col];
            }
          }
        }
      }
    }
  };
  std::vector<std::thread> pool;
  for (uint32_t t = 1; t < std::max<uint32_t>(threads, 1); ++t) pool.emplace_back(worker);
  worker();
  for (auto& thread : pool) thread.join();
  return 0;
}

// iss::AlignElement (tools/iss/dma_engine.cpp:532-544).
uint8_t hrbref_align_element(uint8_t value, uint32_t shift) {
  return hotarubi::iss::AlignElement(value, shift);
}

// DmaEngine::Execute (tools/iss/dma_engine.cpp) of one load into WBUF of kind
// `kind` (include/hotarubi/isa.hpp:66-67: 3 = SPLIT8, 4 = T32_SPLIT8):
// `rows` DDR rows of `row_words` 144-byte MXINT8 words, `stride` bytes apart,
// starting at byte 0 of `ddr` (`ddr_bytes` long), to WBUF word `onchip`.
// `wbuf` (2048 x 144 bytes) holds WBUF before the load and receives it after.
void hrbref_dma_load_wbuf(uint32_t kind, uint8_t* ddr, uint32_t ddr_bytes,
                          uint32_t rows, uint32_t row_words, uint32_t stride,
                          uint32_t onchip, uint8_t* wbuf) {
  namespace iss = hotarubi::iss;
  constexpr uint64_t kBase = 0x20000000;
  iss::Ddr bus(std::span(reinterpret_cast<std::byte*>(ddr), ddr_bytes), kBase);
  auto memories = std::make_unique<iss::Memories>();
  for (uint32_t i = 0; i < iss::kWbufDepth; ++i) {
    std::memcpy(memories->wbuf[i].data(), wbuf + size_t{i} * iss::kWbufWordBytes,
                iss::kWbufWordBytes);
  }
  iss::DmaCommand command{};
  command.ddr_addr = static_cast<uint32_t>(kBase / 16);
  command.mem = 1;  // WBUF (isa::Mem::kWbuf)
  command.onchip = onchip;
  command.rows = rows;
  command.row_words = row_words;
  command.ddr_stride = stride / 16;
  command.kind = kind;
  iss::DmaEngine engine;
  engine.Execute(command, bus, *memories);
  for (uint32_t i = 0; i < iss::kWbufDepth; ++i) {
    std::memcpy(wbuf + size_t{i} * iss::kWbufWordBytes, memories->wbuf[i].data(),
                iss::kWbufWordBytes);
  }
}

// A convolution lowered the way the compiler's ConvEmitter lowers it
// (tools/compiler/sparsedrive_encoder.cpp) and run on the reference's own DMA
// engine and GEMM array, one output tile of 64 positions at a time:
//
//   * faces and taps as MakeSrc builds them (:78-111), their index lists as
//     FaceListS1 / FaceListStrided write them (:114-150, restated here: both
//     are file-local in the reference), the map in DDR row format
//     (TokenBytes, sparsedrive_common.cpp:28-33);
//   * each face gathered into ABUF by DmaEngine::Execute with a ROW_INDEXED
//     load (dma_engine.cpp:231-262, null entries included);
//   * per (plane, face, tap) job one ExecuteGemm with the fields of
//     ConvEmitter::Group (:384-398), the weight tile being the conv matrix's
//     columns [tap*cin + c0, +channels) (ConvTile, sparsedrive_common.cpp:
//     136-158, restated) packed by the reference's PackWbuf;
//   * then ADDP of the bias and, with relu, the RELU pass (restated from
//     lane.cpp:57-70,325 around the reference's Fp32Add).
//
// One x-major map (position x*H + y) of H x W x cin MXINT8 codes aq and
// scale bytes ascale; FP4 weight codes wcode [cout][kh*kh*cin] (one code per
// byte) with exponents we [cout][kh*kh*cin/32]; bias [cout] FP32 bits;
// residual (or null) and c: [Ho*Wo][cout] FP32 bits.  Returns 0, or -1 for a
// shape the emitter rejects.  W8 (hrbref_conv_iss_w8): HI and LO nibble
// codes of the same geometry, each job chained HI then LO (W8Planes,
// smolvla_common.cpp:95-103; kernels.cpp:35-37).
static int conv_iss(uint32_t H, uint32_t W, uint32_t cin, uint32_t cout, uint32_t kh,
                    uint32_t stride, const int8_t* aq, const uint8_t* ascale, uint32_t nplanes,
                    const uint8_t* const* wcodes, const int32_t* we, const uint32_t* bias,
                    const uint32_t* residual, int relu, uint32_t* c) {
  namespace iss = hotarubi::iss;
  if (H % 4 != 0 || cin % 32 != 0 || (cin > 256 && cin % 256 != 0) ||
      (kh != 1 && kh != 3) || (stride != 1 && stride != 2) || cout % 8 != 0 ||
      (cout > 256 && cout % 256 != 0)) {
    return -1;
  }
  struct Face { int32_t dy; bool strided; int32_t dx; };
  struct Tap { uint32_t ky, kx, qoff; };
  std::vector<Face> faces;
  std::vector<std::vector<Tap>> taps;
  if (kh == 1) {
    faces.push_back({0, true, 0});
    taps.push_back({{0, 0, 0}});
  } else if (stride == 1) {
    for (int32_t dy = -1; dy <= 1; ++dy) {
      faces.push_back({dy, false, 0});
      std::vector<Tap> row;
      for (int32_t dx = -1; dx <= 1; ++dx) {
        row.push_back({static_cast<uint32_t>(dy + 1), static_cast<uint32_t>(dx + 1),
                       static_cast<uint32_t>(dx + 1) * H / 4});
      }
      taps.push_back(row);
    }
  } else {
    for (int32_t dy = -1; dy <= 1; ++dy) {
      for (int32_t dx = -1; dx <= 1; ++dx) {
        faces.push_back({dy, true, dx});
        taps.push_back({{static_cast<uint32_t>(dy + 1), static_cast<uint32_t>(dx + 1), 0}});
      }
    }
  }
  constexpr uint32_t mt = 64;
  constexpr uint64_t kBase = 0x20000000;
  const uint32_t plane = std::min(cin, 256u), planes = cin / plane, tok = plane / 32;
  const uint64_t tb = uint64_t{tok} * 32 + (tok + 15) / 16 * 16;
  const uint32_t tokens = H * W, ho = H / stride, wo = W / stride, n_out = ho * wo;
  const uint32_t nt = std::min(cout, 256u), n8 = nt / 8;
  const uint32_t face_tokens = (kh == 3 && stride == 1) ? mt + 2 * H : mt;
  const uint32_t face_words = face_tokens / 4 * tok;
  if (uint64_t{planes} * faces.size() * face_words > iss::kAbufDepth) return -1;
  const uint64_t map_bytes = (uint64_t{tokens} + 64) * tb;
  const uint64_t list_off = planes * map_bytes;
  std::vector<std::byte> bytes(list_off + (uint64_t{face_tokens} * 4 + 15) / 16 * 16 + 64);
  for (uint32_t p = 0; p < planes; ++p) {
    for (uint32_t j = 0; j < tokens; ++j) {
      std::byte* tokp = bytes.data() + p * map_bytes + j * tb;
      for (uint32_t k = 0; k < plane; ++k) {
        tokp[k] = static_cast<std::byte>(aq[size_t{j} * cin + p * plane + k]);
      }
      for (uint32_t b = 0; b < tok; ++b) {
        tokp[tok * 32 + b] = static_cast<std::byte>(ascale[size_t{j} * (cin / 32) + p * tok + b]);
      }
    }
  }
  iss::Ddr ddr{std::span<std::byte>(bytes), kBase};
  auto memories = std::make_unique<iss::Memories>();
  iss::DmaEngine engine;
  const uint32_t kbw = kh * kh * cin / 32;  // weight blocks per row
  for (uint32_t i0 = 0; i0 < n_out; i0 += mt) {
    // LoadFaces: every (plane, face) gathered into its own ABUF range.
    for (uint32_t p = 0; p < planes; ++p) {
      for (size_t f = 0; f < faces.size(); ++f) {
        std::vector<uint32_t> list;
        const Face& face = faces[f];
        auto entry = [&](int64_t token) {
          return static_cast<uint32_t>((kBase + p * map_bytes + token * tb) / 16);
        };
        if (!face.strided) {
          for (int64_t e = 0; e < face_tokens; ++e) {
            const int64_t j = int64_t{i0} - H + e;
            const bool ok = j >= 0 && j < tokens && (j % H) + face.dy >= 0 &&
                            (j % H) + face.dy < H;
            list.push_back(ok ? entry(j + face.dy) : hotarubi::isa::kNullEntry);
          }
        } else {
          for (int64_t o = i0; o < int64_t{i0} + mt; ++o) {
            const int64_t xo = o / ho, yo = o % ho;
            const int64_t yi = int64_t{stride} * yo + face.dy;
            const int64_t xi = int64_t{stride} * xo + face.dx;
            const bool ok = o < int64_t{ho} * wo && yi >= 0 && yi < H && xi >= 0 && xi < W;
            list.push_back(ok ? entry(xi * H + yi) : hotarubi::isa::kNullEntry);
          }
        }
        for (size_t u = 0; u < list.size(); ++u) {
          for (uint32_t b = 0; b < 4; ++b) {
            bytes[list_off + u * 4 + b] = static_cast<std::byte>((list[u] >> (8 * b)) & 0xFF);
          }
        }
        iss::DmaCommand command{};
        command.ddr_addr = static_cast<uint32_t>((kBase + list_off) / 16);
        command.mem = 0;  // ABUF
        command.onchip = static_cast<uint32_t>((p * faces.size() + f) * face_words);
        command.rows = 1;
        command.row_words = face_tokens;
        command.kind = hotarubi::isa::dma::kKindRowIndexed;
        command.tok = tok;
        engine.Execute(command, ddr, *memories);
      }
    }
    for (uint32_t n0 = 0; n0 < cout; n0 += nt) {
      if (residual != nullptr) {
        for (uint32_t r = 0; r < mt; ++r) {
          for (uint32_t n = 0; n < nt; ++n) {
            const uint32_t o = i0 + r;
            memories->fbuf[(r / 4) * n8 + n / 8][(r % 4) * 8 + n % 8] =
                o < n_out ? residual[size_t{o} * cout + n0 + n] : 0;
          }
        }
      }
      uint32_t k = 0;
      for (uint32_t p = 0; p < planes; ++p) {
        for (size_t f = 0; f < faces.size(); ++f) {
          for (const Tap& tap : taps[f]) {
            for (uint32_t wp = 0; wp < nplanes; ++wp) {
              const uint8_t* wcode = wcodes[wp];
              const uint32_t first = (tap.ky * kh + tap.kx) * cin + p * plane;
              hotarubi::compiler::Mxfp4Matrix tile{.rows = nt, .cols = plane, .code = {}, .e = {}};
              for (uint32_t r = n0; r < n0 + nt; ++r) {
                tile.code.insert(tile.code.end(), wcode + size_t{r} * kh * kh * cin + first,
                                 wcode + size_t{r} * kh * kh * cin + first + plane);
                for (uint32_t b = 0; b < tok; ++b) tile.e.push_back(we[size_t{r} * kbw + first / 32 + b]);
              }
              const std::vector<std::byte> words = hotarubi::compiler::PackWbuf(tile);
              for (size_t wd = 0; wd < words.size() / iss::kWbufWordBytes; ++wd) {
                std::memcpy(memories->wbuf[wd].data(), words.data() + wd * iss::kWbufWordBytes,
                            iss::kWbufWordBytes);
              }
              const GemmCommand gemm{
                  .a_base = static_cast<uint32_t>((p * faces.size() + f) * face_words + tap.qoff * tok),
                  .a_stride = tok,
                  .kb = tok,
                  .m = mt,
                  .w_base = 0,
                  .w_stride = tok,
                  .n8 = n8,
                  .c_base = 0,
                  .wmode = nplanes == 1 ? 0u : 1u + wp,
                  .acc = k > 0 || residual != nullptr};
              iss::ExecuteGemm(gemm, *memories);
              ++k;
            }
          }
        }
      }
      for (uint32_t r = 0; r < mt && i0 + r < n_out; ++r) {
        for (uint32_t n = 0; n < nt; ++n) {
          uint32_t v = memories->fbuf[(r / 4) * n8 + n / 8][(r % 4) * 8 + n % 8];
          v = iss::Fp32Add(v, bias[n0 + n]);
          if (relu) {
            const bool keep = (v >> 31) == 0 || (v & 0x7FFFFFFFu) == 0;
            v = iss::Fp32Add(keep ? v : 0u, 0u);
          }
          c[size_t{i0 + r} * cout + n0 + n] = v;
        }
      }
    }
  }
  return 0;
}

int hrbref_conv_iss(uint32_t H, uint32_t W, uint32_t cin, uint32_t cout, uint32_t kh,
                    uint32_t stride, const int8_t* aq, const uint8_t* ascale,
                    const uint8_t* wcode, const int32_t* we, const uint32_t* bias,
                    const uint32_t* residual, int relu, uint32_t* c) {
  const uint8_t* const planes[1] = {wcode};
  return conv_iss(H, W, cin, cout, kh, stride, aq, ascale, 1, planes, we, bias, residual, relu,
                  c);
}

int hrbref_conv_iss_w8(uint32_t H, uint32_t W, uint32_t cin, uint32_t cout, uint32_t kh,
                       uint32_t stride, const int8_t* aq, const uint8_t* ascale,
                       const uint8_t* hi, const uint8_t* lo, const int32_t* we,
                       const uint32_t* bias, const uint32_t* residual, int relu, uint32_t* c) {
  const uint8_t* const planes[2] = {hi, lo};
  return conv_iss(H, W, cin, cout, kh, stride, aq, ascale, 2, planes, we, bias, residual, relu,
                  c);
}

// A GEMM whose activations come from DDR in the DMA row format, as a
// compiled program feeds the GEMM array: per chunk of 32-token groups and
// per plane one LoadRows (DmaEngine::Execute with kind ROW, one command per
// DDR row segment, or ROW_INDEXED over the plane's entry list,
// dma_engine.cpp:156-195,231-262) into an ABUF region of its own, then per
// plane (one K piece of tok blocks) the GEMM instructions of each weight
// plane (W8: HI then LO), accumulating in order, over column tiles.
//
// ddr: the DDR window [ddr_base, ddr_base + ddr_bytes).  Token m's unit of
// plane 0: ROW at ddr_base + m0 + (m / row_tokens) * row_stride +
// (m % row_tokens) * unit bytes, where m0 = first_unit * 16 - ddr_base;
// ROW_INDEXED (index != null) at index[m] * 16 (0xFFFFFFFF: null).  Plane p
// adds p * plane_stride.  Weights as hrbref_dense_gemm_iss's (nplanes 1 FP4,
// 2 W8), kb = planes * tok.  c: M x N FP32 bits.  ROW needs M a multiple of
// 32 tokens (the ISS's m) and row_tokens of 4; -1 on a rejected shape.
int hrbref_rows_gemm_iss(const uint8_t* ddr, uint64_t ddr_bytes, uint64_t ddr_base,
                         uint32_t first_unit, uint32_t tok, uint32_t planes,
                         uint64_t plane_stride, uint32_t row_tokens, uint64_t row_stride,
                         const uint32_t* index, uint32_t M, uint32_t N, uint32_t nplanes,
                         const uint8_t* wplanes, uint32_t* c) {
  namespace iss = hotarubi::iss;
  using hotarubi::isa::kNullEntry;
  namespace dma = hotarubi::isa::dma;
  const uint32_t kb = planes * tok;
  if (tok == 0 || tok > 32 || planes == 0 || N % 8 != 0 || kb > iss::kWbufDepth) return -1;
  if (index == nullptr && (M % 32 != 0 || row_tokens % 4 != 0 || row_tokens == 0)) return -1;
  const uint32_t unit_bytes = tok * 32 + (tok > 16 ? 32 : 16);
  std::vector<std::byte> bytes(ddr_bytes + 64 * 1024);
  std::memcpy(bytes.data(), ddr, ddr_bytes);
  // Index lists of each chunk go past the window's end.
  const uint64_t list_off = ddr_bytes;
  iss::Ddr mem{std::span<std::byte>(bytes), ddr_base};
  auto memories = std::make_unique<iss::Memories>();
  iss::DmaEngine engine;
  const uint32_t groups_total = N / 8;
  const uint32_t tile_groups = std::max<uint32_t>(1, std::min<uint32_t>(32, iss::kWbufDepth / kb));
  // Tokens per chunk: every plane's quads in ABUF, FBUF for a tile.
  uint32_t chunk = std::min<uint32_t>(iss::kAbufDepth / kb * 4, iss::kFbufDepth / tile_groups * 4);
  chunk -= chunk % 32;
  if (chunk == 0) return -1;
  const size_t plane_bytes = size_t{groups_total} * kb * 144;
  for (uint32_t t0 = 0; t0 < M; t0 += chunk) {
    const uint32_t count = std::min(chunk, M - t0);
    const uint32_t m = (count + 31) / 32 * 32;
    const uint32_t quads = m / 4;
    for (uint32_t p = 0; p < planes; ++p) {
      const uint32_t region = p * quads * tok;
      if (index != nullptr) {
        for (uint32_t u = 0; u < m; ++u) {
          uint32_t e = kNullEntry;
          if (t0 + u < M && index[t0 + u] != kNullEntry) {
            e = static_cast<uint32_t>(index[t0 + u] + p * (plane_stride / 16));
          }
          std::memcpy(bytes.data() + list_off + u * 4, &e, 4);
        }
        iss::DmaCommand command{};
        command.ddr_addr = static_cast<uint32_t>((ddr_base + list_off) / 16);
        command.mem = 0;
        command.onchip = region;
        command.rows = 1;
        command.row_words = m;
        command.kind = dma::kKindRowIndexed;
        command.tok = tok;
        engine.Execute(command, mem, *memories);
      } else {
        // One command per row segment [a, b) of the chunk's tokens.
        for (uint32_t a = t0; a < t0 + m;) {
          const uint32_t b = std::min(t0 + m, (a / row_tokens + 1) * row_tokens);
          const uint64_t addr = uint64_t{first_unit} * 16 + p * plane_stride +
                                uint64_t{a / row_tokens} * row_stride +
                                uint64_t{a % row_tokens} * unit_bytes;
          iss::DmaCommand command{};
          command.ddr_addr = static_cast<uint32_t>(addr / 16);
          command.mem = 0;
          command.onchip = region + (a - t0) / 4 * tok;
          command.rows = 1;
          command.row_words = b - a;
          command.kind = dma::kKindRow;
          command.tok = tok;
          engine.Execute(command, mem, *memories);
          a = b;
        }
      }
    }
    for (uint32_t g0 = 0; g0 < groups_total; g0 += tile_groups) {
      const uint32_t gc = std::min(tile_groups, groups_total - g0);
      uint32_t k = 0;
      for (uint32_t p = 0; p < planes; ++p) {
        for (uint32_t l = 0; l < nplanes; ++l) {
          for (uint32_t g = 0; g < gc; ++g) {
            for (uint32_t b = 0; b < tok; ++b) {
              std::memcpy(memories->wbuf[(g * tok) + b].data(),
                          wplanes + (l * plane_bytes) +
                              ((size_t{g0 + g} * kb) + p * tok + b) * 144,
                          144);
            }
          }
          const GemmCommand gemm{.a_base = p * quads * tok,
                                 .a_stride = tok,
                                 .kb = tok,
                                 .m = m,
                                 .w_base = 0,
                                 .w_stride = tok,
                                 .n8 = gc,
                                 .c_base = 0,
                                 .wmode = nplanes == 1 ? 0U : l + 1,
                                 .acc = k > 0};
          iss::ExecuteGemm(gemm, *memories);
          ++k;
        }
      }
      for (uint32_t r = 0; r < count; ++r) {
        for (uint32_t g = 0; g < gc; ++g) {
          for (uint32_t col = 0; col < 8; ++col) {
            c[size_t{t0 + r} * N + (g0 + g) * 8 + col] =
                memories->fbuf[(r / 4) * gc + g][(r % 4) * 8 + col];
          }
        }
      }
    }
  }
  return 0;
}

// CostModel::Gemm (tools/iss/timing.cpp:89-93, default TimingParameters):
// the NPU cycles of one GEMM instruction; *array receives GemmArrayCycles
// (:65-67).
uint64_t hrbref_gemm_cycles(const uint32_t* fields, uint64_t* array) {
  const GemmCommand command = Command(fields);
  if (array != nullptr) *array = hotarubi::iss::GemmArrayCycles(command);
  return hotarubi::iss::CostModel{}.Gemm(command).cycles;
}

// NPU cycles of a dense GEMM as hrbref_dense_gemm_iss tiles it into GEMM
// instructions (every row chunk x column tile, each weight plane), summed
// over CostModel::Gemm (tools/iss/timing.cpp:89-93).  0 when kb does not fit.
uint64_t hrbref_dense_gemm_cycles(uint32_t nplanes, uint32_t M, uint32_t N, uint32_t kb) {
  using hotarubi::iss::kAbufDepth;
  using hotarubi::iss::kFbufDepth;
  using hotarubi::iss::kWbufDepth;
  if (kb == 0 || kb > kWbufDepth || N % 8 != 0) return 0;
  const uint32_t groups_total = N / 8;
  uint32_t tile_groups = std::min<uint32_t>(255, kWbufDepth / kb);
  uint32_t chunk_quads = std::min<uint32_t>(248, kAbufDepth / kb);
  chunk_quads -= chunk_quads % 8;
  if (tile_groups == 0 || chunk_quads == 0) return 0;
  while (chunk_quads * tile_groups > kFbufDepth) {
    if (tile_groups > 8) {
      tile_groups /= 2;
    } else {
      chunk_quads -= 8;
    }
  }
  const uint32_t quads = (M + 3) / 4;
  const hotarubi::iss::CostModel model;
  uint64_t cycles = 0;
  for (uint32_t q_first = 0; q_first < quads; q_first += chunk_quads) {
    const uint32_t q_count = std::min(chunk_quads, quads - q_first);
    const uint32_t m = ((q_count * 4) + 31) / 32 * 32;
    for (uint32_t g_first = 0; g_first < groups_total; g_first += tile_groups) {
      const uint32_t g_count = std::min(tile_groups, groups_total - g_first);
      for (uint32_t l = 0; l < nplanes; ++l) {
        const GemmCommand command{.a_base = 0, .a_stride = kb, .kb = kb, .m = m, .w_base = 0,
                                  .w_stride = kb, .n8 = g_count, .c_base = 0,
                                  .wmode = nplanes == 1 ? 0U : l + 1, .acc = l > 0};
        cycles += model.Gemm(command).cycles;
      }
    }
  }
  return cycles;
}

// GACC through the reference's DmaEngine::Execute (tools/iss/dma_engine.cpp:
// 599-652): the dense operands of hrbo_gacc_dense (tokens a multiple of 4,
// 4 corners, 1..8 blocks) laid out in a DDR image as the DMA engine reads
// them (the index list of 64-bit entries after a weights pointer, the
// coefficient banks per 8-slot group and block, feature rows in row format),
// one GACC command per 4 tokens; slots [0, split) and [split, slots) as two
// commands, the second continuing the first's accumulators (acc), flushed to
// FBUF.  out: FP32 bits [tokens][blocks * 32].  Returns 0, or -1 for a shape
// outside the instruction.
int hrbref_gacc_iss(uint32_t tokens, uint32_t slots, uint32_t blocks, const uint64_t* entries,
                    const uint32_t* w, const uint8_t* rows, uint32_t nrows, uint32_t split,
                    uint32_t* out) {
  namespace iss = hotarubi::iss;
  if (tokens % 4 != 0 || blocks < 1 || blocks > 8 || slots < 1 || slots > 2047 ||
      split > slots) {
    return -1;
  }
  constexpr uint64_t kBase = 0x20000000;
  const uint64_t row_bytes = (2ull * blocks + 1) * 16;
  const uint32_t groups = (slots + 7) / 8;
  const uint64_t feat_off = 0;
  const uint64_t bank_off = (feat_off + nrows * row_bytes + 127) / 128 * 128;
  const uint64_t bank_bytes = uint64_t{groups} * 128 * blocks;
  const uint64_t list_off = (bank_off + bank_bytes + 127) / 128 * 128;
  const uint64_t list_bytes = 16 + uint64_t{slots} * 16 * 8;
  std::vector<std::byte> bytes(list_off + list_bytes + 64);
  std::memcpy(bytes.data() + feat_off, rows, nrows * row_bytes);
  iss::Ddr ddr{std::span<std::byte>(bytes), kBase};
  auto memories = std::make_unique<iss::Memories>();
  iss::DmaEngine engine;
  auto put = [&](uint64_t off, uint64_t v, int n) {
    for (int i = 0; i < n; ++i) bytes[off + i] = static_cast<std::byte>((v >> (8 * i)) & 0xFF);
  };
  for (uint32_t tg = 0; tg < tokens / 4; ++tg) {
    // Coefficient banks: block i, group g at bank + (i * groups + g) * 128,
    // element t * 8 + s % 8.
    for (uint32_t i = 0; i < blocks; ++i) {
      for (uint32_t s = 0; s < slots; ++s) {
        for (uint32_t t = 0; t < 4; ++t) {
          const uint64_t at = bank_off + (uint64_t{i} * groups + s / 8) * 128 + 4 * (t * 8 + s % 8);
          put(at, w[((size_t{tg} * 4 + t) * slots + s) * blocks + i], 4);
        }
      }
    }
    put(list_off, (kBase + bank_off) / 16, 8);
    for (uint32_t s = 0; s < slots; ++s) {
      for (uint32_t t = 0; t < 4; ++t) {
        for (uint32_t k = 0; k < 4; ++k) {
          const uint64_t e = entries[((size_t{tg} * 4 + t) * slots + s) * 4 + k];
          const uint32_t index = static_cast<uint32_t>(e);
          const uint64_t unit = index == 0xFFFFFFFFu
                                    ? 0xFFFFFFFFull
                                    : (kBase + feat_off + index * row_bytes) / 16;
          put(list_off + 16 + ((uint64_t{s} * 16) + t * 4 + k) * 8, unit | (e & ~0xFFFFFFFFull), 8);
        }
      }
    }
    // Two commands: slots [0, split) and [split, slots); the list of the
    // second starts `split` slots in, its banks `split / 8` groups in
    // (split is a multiple of 8 or the whole list).
    const uint32_t parts[2][2] = {{0, split}, {split, slots}};
    for (int c = 0; c < 2; ++c) {
      const uint32_t first = parts[c][0], count = parts[c][1] - parts[c][0];
      if (count == 0) continue;
      if (c == 1) {
        put(list_off + uint64_t{first} * 16 * 8, (kBase + bank_off + (first / 8) * 128) / 16, 8);
      }
      iss::DmaCommand command{};
      command.ddr_addr = static_cast<uint32_t>((kBase + list_off + uint64_t{first} * 16 * 8) / 16);
      command.mem = 2;  // FBUF
      command.onchip = 0;
      command.rows = count;
      command.row_words = blocks;
      command.ddr_stride = groups * 8;
      command.kind = hotarubi::isa::dma::kKindGacc;
      command.acc = c == 1 && split != 0;
      command.flush = c == 1 || split == slots;
      engine.Execute(command, ddr, *memories);
    }
    for (uint32_t g = 0; g < blocks * 4; ++g) {
      for (uint32_t t = 0; t < 4; ++t) {
        for (uint32_t cc = 0; cc < 8; ++cc) {
          out[(size_t{tg} * 4 + t) * blocks * 32 + g * 8 + cc] = memories->fbuf[g][t * 8 + cc];
        }
      }
    }
  }
  return 0;
}


// The regions part of a meta.json as the compiler writes it (MetaJson,
// tools/compiler/output.cpp:57-89: base, instr_off, n_instr, image_bytes,
// listings, then "regions": name -> [offset, size]) with hotarubi's Json
// writer; returns the text length, or -1 when `cap` is too small.
int64_t hrbref_meta_json(const char* const* names, const uint64_t* offsets,
                         const uint64_t* sizes, uint32_t n, uint64_t image_bytes, char* out,
                         size_t cap) {
  using hotarubi::Json;
  Json::Object regions;
  for (uint32_t i = 0; i < n; ++i) {
    regions.emplace_back(names[i], Json(Json::Array{Json(static_cast<double>(offsets[i])),
                                                    Json(static_cast<double>(sizes[i]))}));
  }
  Json::Object meta = {{"base", Json(static_cast<double>(0x40000000ULL))},
                       {"instr_off", Json(0.0)},
                       {"n_instr", Json(0.0)},
                       {"image_bytes", Json(static_cast<double>(image_bytes))}};
  meta.emplace_back("listings", Json(Json::Object{{"main", Json(std::string("main.listing.json"))}}));
  meta.emplace_back("regions", Json(std::move(regions)));
  const std::string text = Json(std::move(meta)).Dump() + "\n";
  if (text.size() + 1 > cap) return -1;
  std::memcpy(out, text.c_str(), text.size() + 1);
  return static_cast<int64_t>(text.size());
}

// A region of a meta.json as LoadProgram reads it (tools/runtime/runtime.cpp:
// 132-150): Json::Parse, then regions -> name -> [offset, size].  0 when
// found, 1 when missing, 2 when the text does not parse.
int hrbref_find_region(const char* meta, const char* name, uint64_t* offset, uint64_t* size) {
  auto json = hotarubi::Json::Parse(meta);
  if (!json) return 2;
  const hotarubi::Json* regions = json->Find("regions");
  if (regions == nullptr) return 1;
  const hotarubi::Json* r = regions->Find(name);
  if (r == nullptr || !r->IsArray() || r->Items().size() != 2) return 1;
  *offset = static_cast<uint64_t>(r->Items()[0].Number());
  *size = static_cast<uint64_t>(r->Items()[1].Number());
  return 0;
}

}  // extern "C"
