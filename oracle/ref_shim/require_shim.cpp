// Test infrastructure only: part of the build of the reference's own GEMM
// sources into oracle/_ref/ (the checker), never linked into the product.
//
// Stand-in for hotarubi's tools/runtime/require.cpp:10-13, which prints with
// <print> (GCC 14) before aborting.  Same behaviour on g++ 13: the message
// goes to stderr prefixed with "error: ", then abort().
#include <cstdio>
#include <cstdlib>
#include <string_view>

namespace hotarubi {

[[noreturn]] void Fail(std::string_view message) {
  std::fprintf(stderr, "error: %.*s\n", static_cast<int>(message.size()),
               message.data());
  std::abort();
}

}  // namespace hotarubi
