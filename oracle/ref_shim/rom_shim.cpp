// Test infrastructure only (oracle/_ref build of the reference sources).
//
// hotarubi generates tools/iss/rom.cpp from rtl/vec_rom_pkg.sv with a CMake
// script (tools/iss/CMakeLists.txt:1-8).  The ROM holds the VEC program
// library that Memories() copies into CBUF (tools/iss/memories.cpp).  The GEMM
// path never reads CBUF, so the checker links an all-zero ROM of the declared
// size instead of running the reference's build system.
#include "rom.hpp"

namespace hotarubi::iss {

const std::array<Word128, kRomWords> kRom = {};

}  // namespace hotarubi::iss
