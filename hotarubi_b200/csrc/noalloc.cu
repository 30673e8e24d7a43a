// hrb_gemm_dense_noalloc: the dense GEMM for callers that cannot allocate
// device memory.
//
// Some hosts of this library may not call cudaMalloc at all: a simulator
// plugin that runs inside a process whose device memory is owned and
// accounted by someone else, code that runs while a CUDA graph is being
// captured, or a real-time loop where an allocation (and the implicit
// synchronisation it can bring) is not allowed.  They pass device pointers
// for every input and output and get a GEMM that needs no allocation: the
// only scratch — the MXINT8 encoding of FP32 activations — lives in the
// file-scope device array below, which every GPU that loads this library
// holds until the process exits.
//
// Limits and sharing:
//   * The scratch holds HRB_NOALLOC_SCRATCH_BYTES (4 MiB): an FP32-input GEMM
//     needs M * kp bytes of codes plus M * kp / 32 scale bytes (each part
//     rounded up to 256 bytes); larger requests fail with HRB_EINVAL before
//     anything is launched.  MXINT8-input GEMMs need no scratch.
//   * Every call shares the one array and it keeps the last call's
//     contents.  Nothing in it has to start at zero (the encoder writes every
//     byte a GEMM later reads), so calls do not clear it, but two calls
//     whose work overlaps on the GPU (different streams, or different host
//     threads) race on it: serialise them on one stream.
//   * The first call on a device looks the array's device address up with
//     cudaGetSymbolAddress (host code cannot use the symbol itself as a
//     device pointer) with that device current, and caches it per device
//     ordinal; make that first call before any stream capture.  The address
//     belongs to the context current at that moment: the runtime's primary
//     context, the only one this entry point supports.  A host that makes
//     its own driver context current, or resets the device
//     (cudaDeviceReset), must not use it afterwards: the cached address is
//     not looked up again.
//   * A CUDA error already pending on the calling thread (an earlier launch
//     of someone else's that failed) is not taken for this call's: the call
//     returns HRB_ECUDA naming it, launches nothing and leaves it pending.
//   * Non-finite activations are not reported (there is no context to hold
//     the flag); hrb_gemm_dense reports them through hrb_sync.
#include <cuda_runtime.h>

#include <cstdint>
#include <cstdio>
#include <mutex>

#include "hrb_gemm.h"
#include "hrb_kernels.cuh"
#include "hrb_tc.cuh"

namespace {

constexpr size_t kScratchBytes = HRB_NOALLOC_SCRATCH_BYTES;
constexpr size_t kFlagBytes = 256;  // the encoder's Inf/NaN flag word
constexpr int kMaxDevices = 64;

static __device__ __align__(256) uint8_t g_noalloc_scratch[kScratchBytes + kFlagBytes];

struct DeviceSetup {
  uint8_t* scratch = nullptr;  // device address of g_noalloc_scratch
  int sm_count = 0;
};

std::mutex g_setup_mutex;
DeviceSetup g_setup[kMaxDevices];

size_t align_up(size_t x, size_t a) { return (x + a - 1) / a * a; }

// Once per device, with that device current: the array's device address.
hrb_status setup_device(int device, DeviceSetup* out) {
  if (device < 0 || device >= kMaxDevices) {
    return hrb::noalloc_fail(HRB_EINVAL, "hrb_gemm_dense_noalloc: device ordinal out of range");
  }
  std::lock_guard<std::mutex> lock(g_setup_mutex);
  DeviceSetup& s = g_setup[device];
  if (s.scratch == nullptr) {
    void* ptr = nullptr;
    const cudaError_t e = cudaGetSymbolAddress(&ptr, g_noalloc_scratch);
    if (e != cudaSuccess || ptr == nullptr) {
      return hrb::noalloc_cuda_fail(e, "hrb_gemm_dense_noalloc: cudaGetSymbolAddress of the scratch");
    }
    int sms = 0;
    const cudaError_t a = cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, device);
    if (a != cudaSuccess) {
      return hrb::noalloc_cuda_fail(a, "hrb_gemm_dense_noalloc: SM count");
    }
    s.sm_count = sms;
    s.scratch = static_cast<uint8_t*>(ptr);
  }
  *out = s;
  return HRB_OK;
}

}  // namespace

extern "C" hrb_status hrb_gemm_dense_noalloc(const hrb_gemm_desc* desc, void* stream) {
  uint32_t pieces[hrb::kMaxPieces];
  uint32_t npieces = 0;
  hrb_status st = hrb::check_desc_for_noalloc(desc, pieces, &npieces);
  if (st != HRB_OK) return st;
  if (desc->c == nullptr) {  // the exact kernel writes C
    return hrb::noalloc_fail(HRB_EINVAL, "hrb_gemm_dense_noalloc: c is required");
  }
  const uint32_t kb = (desc->K + 31u) / 32u;
  const size_t code_bytes = align_up(size_t{desc->M} * kb * 32u, 256);
  const size_t scale_bytes = align_up(size_t{desc->M} * kb, 256);
  if (desc->a != nullptr && code_bytes + scale_bytes > kScratchBytes) {
    char msg[160];
    std::snprintf(msg, sizeof msg,
                  "hrb_gemm_dense_noalloc: activation encoding needs %zu bytes, scratch holds %zu",
                  code_bytes + scale_bytes, kScratchBytes);
    return hrb::noalloc_fail(HRB_EINVAL, msg);
  }
  const cudaError_t pending = cudaPeekAtLastError();
  if (pending != cudaSuccess) {
    return hrb::noalloc_cuda_fail(pending, "hrb_gemm_dense_noalloc: an earlier CUDA error is pending");
  }
  int device = 0;
  const cudaError_t g = cudaGetDevice(&device);
  if (g != cudaSuccess) return hrb::noalloc_cuda_fail(g, "hrb_gemm_dense_noalloc: cudaGetDevice");
  DeviceSetup setup;
  st = setup_device(device, &setup);
  if (st != HRB_OK) return st;
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  const int8_t* aq = desc->aq;
  const uint8_t* ascale = desc->ascale;
  if (desc->a != nullptr) {
    auto* q = reinterpret_cast<int8_t*>(setup.scratch);
    uint8_t* sc = setup.scratch + code_bytes;
    auto* flag = reinterpret_cast<uint32_t*>(setup.scratch + kScratchBytes);
    const hrb::QuantJob j = hrb::make_quant_job_for_noalloc(desc, q, sc);
    hrb::launch_quantize(nullptr, 1, &j, j.units, flag, setup.sm_count, s);
    aq = q;
    ascale = sc;
  }
  // Both modes run the exact kernel here: the tensor-core path needs its
  // weights translated into scratch the size of the weights, which a fixed
  // array cannot hold; the exact result is within the fast mode's tolerance.
  hrb::DenseJob job = hrb::make_dense_job_for_noalloc(desc, aq, ascale, pieces, npieces);
  uint32_t tiles_n = 0;
  const uint32_t tiles = hrb::dense_exact_tiles(job.M, job.N, tiles_n);
  job.tiles_n = tiles_n;
  job.tile_begin = 0;
  hrb::launch_dense_exact(nullptr, 1, &job, tiles, job.wfmt, s);
  if (desc->cq != nullptr) {
    // The MXINT8 copy of C, encoded after the GEMM (its flag word is the
    // scratch's, unreported as above).
    const hrb::QuantJob pq = hrb::make_post_quant_job_for_noalloc(desc);
    hrb::launch_quantize(nullptr, 1, &pq, pq.units,
                         reinterpret_cast<uint32_t*>(setup.scratch + kScratchBytes),
                         setup.sm_count, s);
  }
  const cudaError_t e = cudaGetLastError();
  return e == cudaSuccess ? HRB_OK : hrb::noalloc_cuda_fail(e, "hrb_gemm_dense_noalloc: launch");
}
