// Test infrastructure only (oracle/_ref build of the reference sources).
//
// hotarubi's tb/gemm_ref.cpp includes tb/npu_data.hpp and tb/npu_isa.hpp,
// which pull in Verilator's generated Vnpu_top.h through tb/npu_bench.hpp.
// Verilator is not installed, so this header is force-included (-include)
// when compiling tb/gemm_ref.cpp and tb/fp32_ref.cpp: it claims both include
// guards and supplies only the four word types the reference GEMM uses, with
// the field layout of tb/npu_data.hpp:19-31 and tb/npu_isa.hpp:50-62.
#ifndef HRB_ORACLE_TB_TYPES_HPP_
#define HRB_ORACLE_TB_TYPES_HPP_

#define HOTARUBI_TB_NPU_DATA_HPP_
#define HOTARUBI_TB_NPU_ISA_HPP_

#include <array>
#include <cstdint>

namespace hotarubi::tb {

struct AbufWord {
  std::array<int8_t, 128> q{};
  std::array<uint8_t, 4> scale{};
};

struct WbufWord {
  std::array<uint8_t, 256> nibble{};
  std::array<uint8_t, 8> scale{};
};

using FbufWord = std::array<uint32_t, 32>;

struct GemmArgs {
  uint32_t a_base = 0;
  uint32_t a_stride = 0;
  uint32_t kb = 0;
  uint32_t m = 0;
  uint32_t w_base = 0;
  uint32_t w_stride = 0;
  uint32_t n8 = 0;
  uint32_t c_base = 0;
  uint32_t wmode = 0;
  bool acc = false;
  uint32_t wait = 0;
};

}  // namespace hotarubi::tb

#endif  // HRB_ORACLE_TB_TYPES_HPP_
