// The communicator of the multi-GPU paths (include/hrb_gemm.h section 8),
// for hosts that bring no framework: one process per GPU, NCCL over NVLink.
//
// hotarubi itself runs on one NPU and has no collective; what the sharded
// GEMMs and convolutions need around their kernels is the plumbing:
//   * bootstrap: rank 0 makes a unique id (hrb_comm_id_new) and hands the
//     128 bytes to the other ranks by its own means (a pipe, a file, MPI);
//     every rank then calls hrb_comm_create;
//   * hrb_comm_exchange: a small record of every rank on every rank (the
//     IPC handles of the buffers the fused all-gather stores into);
//   * hrb_comm_barrier: every rank's queued work finished (host side);
//   * hrb_comm_fence: the same as a stream dependency (device side): the end
//     of a sharded step, after which every rank holds every peer store;
//   * hrb_comm_allgather: byte ranges that each rank computed in place in
//     one buffer, made whole on every rank (the library all-gather the fused
//     peer stores are measured against, and the gather of row-sharded
//     convolutions' outputs on hosts that do not map peers).
//
// NCCL is loaded at the first call (dlopen of libnccl.so.2), so the library
// itself loads, and runs every single-GPU path, without it.
#include <cuda_runtime.h>
#include <dlfcn.h>
#include <nccl.h>

#include <cstdint>
#include <cstdio>
#include <cstring>
#include <mutex>
#include <new>
#include <string>
#include <vector>

#include "hrb_gemm.h"
#include "hrb_kernels.cuh"

static_assert(sizeof(ncclUniqueId) <= sizeof(hrb_comm_id), "NCCL unique id size");

struct hrb_comm {
  hrb_ctx* ctx = nullptr;
  ncclComm_t comm = nullptr;
  uint32_t rank = 0, ranks = 0;
  void* d_scratch = nullptr;  // staging of hrb_comm_exchange / hrb_comm_barrier
  size_t scratch_bytes = 0;
  uint8_t* d_fence = nullptr;  // one byte per rank for hrb_comm_fence
};

namespace {

struct Nccl {
  ncclResult_t (*get_unique_id)(ncclUniqueId*) = nullptr;
  ncclResult_t (*init_rank)(ncclComm_t*, int, ncclUniqueId, int) = nullptr;
  ncclResult_t (*destroy)(ncclComm_t) = nullptr;
  ncclResult_t (*all_gather)(const void*, void*, size_t, ncclDataType_t, ncclComm_t,
                             cudaStream_t) = nullptr;
  ncclResult_t (*broadcast)(const void*, void*, size_t, ncclDataType_t, int, ncclComm_t,
                            cudaStream_t) = nullptr;
  ncclResult_t (*group_start)() = nullptr;
  ncclResult_t (*group_end)() = nullptr;
  const char* (*error_string)(ncclResult_t) = nullptr;
  std::string missing;  // why NCCL is unusable, or empty
};

template <typename F>
bool bind(void* lib, const char* name, F* fn) {
  *fn = reinterpret_cast<F>(dlsym(lib, name));
  return *fn != nullptr;
}

const Nccl& nccl() {
  static Nccl n;
  static std::once_flag once;
  std::call_once(once, [] {
    void* lib = dlopen("libnccl.so.2", RTLD_NOW | RTLD_GLOBAL);
    if (lib == nullptr) lib = dlopen("libnccl.so", RTLD_NOW | RTLD_GLOBAL);
    if (lib == nullptr) {
      n.missing = std::string("NCCL not found: ") + dlerror();
      return;
    }
    const bool ok = bind(lib, "ncclGetUniqueId", &n.get_unique_id) &&
                    bind(lib, "ncclCommInitRank", &n.init_rank) &&
                    bind(lib, "ncclCommDestroy", &n.destroy) &&
                    bind(lib, "ncclAllGather", &n.all_gather) &&
                    bind(lib, "ncclBroadcast", &n.broadcast) &&
                    bind(lib, "ncclGroupStart", &n.group_start) &&
                    bind(lib, "ncclGroupEnd", &n.group_end) &&
                    bind(lib, "ncclGetErrorString", &n.error_string);
    if (!ok) n.missing = "NCCL lacks an entry point this library uses";
  });
  return n;
}

hrb_status nccl_fail(hrb_ctx* ctx, ncclResult_t r, const char* what) {
  char msg[256];
  std::snprintf(msg, sizeof msg, "%s: %s", what,
                nccl().error_string != nullptr ? nccl().error_string(r) : "NCCL error");
  return hrb::ctx_fail(ctx, HRB_ECUDA, msg);
}

hrb_status cuda_fail(hrb_ctx* ctx, cudaError_t e, const char* what) {
  char msg[256];
  std::snprintf(msg, sizeof msg, "%s: %s", what, cudaGetErrorString(e));
  return hrb::ctx_fail(ctx, e == cudaErrorMemoryAllocation ? HRB_ENOMEM : HRB_ECUDA, msg);
}

#define HRB_COMM_CUDA(ctx, call)                                        \
  do {                                                                  \
    const cudaError_t e_ = (call);                                      \
    if (e_ != cudaSuccess) return cuda_fail(ctx, e_, #call);            \
  } while (0)

#define HRB_COMM_NCCL(ctx, call)                                        \
  do {                                                                  \
    const ncclResult_t r_ = (call);                                     \
    if (r_ != ncclSuccess) return nccl_fail(ctx, r_, #call);            \
  } while (0)

hrb_status grow_scratch(hrb_comm* c, size_t bytes) {
  if (c->scratch_bytes >= bytes) return HRB_OK;
  if (c->d_scratch != nullptr) cudaFree(c->d_scratch);
  c->d_scratch = nullptr;
  c->scratch_bytes = 0;
  HRB_COMM_CUDA(c->ctx, cudaMalloc(&c->d_scratch, bytes));
  c->scratch_bytes = bytes;
  return HRB_OK;
}

}  // namespace

extern "C" {

hrb_status hrb_comm_id_new(hrb_comm_id* out) {
  if (out == nullptr) return HRB_EINVAL;
  const Nccl& n = nccl();
  if (!n.missing.empty()) return hrb::ctx_fail(nullptr, HRB_ENOTSUP, n.missing.c_str());
  ncclUniqueId id;
  const ncclResult_t r = n.get_unique_id(&id);
  if (r != ncclSuccess) return nccl_fail(nullptr, r, "ncclGetUniqueId");
  std::memset(out, 0, sizeof(*out));
  std::memcpy(out->bytes, &id, sizeof(id));
  return HRB_OK;
}

hrb_status hrb_comm_create(hrb_ctx* ctx, const hrb_comm_id* id, uint32_t rank, uint32_t ranks,
                           hrb_comm** out) {
  if (ctx == nullptr || id == nullptr || out == nullptr) return HRB_EINVAL;
  *out = nullptr;
  if (ranks == 0 || rank >= ranks) {
    return hrb::ctx_fail(ctx, HRB_EINVAL, "rank out of range");
  }
  const Nccl& n = nccl();
  if (!n.missing.empty()) return hrb::ctx_fail(ctx, HRB_ENOTSUP, n.missing.c_str());
  HRB_COMM_CUDA(ctx, cudaSetDevice(hrb::ctx_device(ctx)));
  auto* c = new (std::nothrow) hrb_comm;
  if (c == nullptr) return hrb::ctx_fail(ctx, HRB_ENOMEM, "communicator");
  c->ctx = ctx;
  c->rank = rank;
  c->ranks = ranks;
  ncclUniqueId uid;
  std::memcpy(&uid, id->bytes, sizeof(uid));
  // Blocks until every rank has called it with the same id.
  const ncclResult_t r =
      n.init_rank(&c->comm, static_cast<int>(ranks), uid, static_cast<int>(rank));
  if (r != ncclSuccess) {
    delete c;
    return nccl_fail(ctx, r, "ncclCommInitRank");
  }
  const cudaError_t e = cudaMalloc(&c->d_fence, ranks);
  if (e != cudaSuccess) {
    n.destroy(c->comm);
    delete c;
    return cuda_fail(ctx, e, "communicator fence buffer");
  }
  *out = c;
  return HRB_OK;
}

hrb_status hrb_comm_fence(hrb_comm* comm, void* stream) {
  if (comm == nullptr) return HRB_EINVAL;
  hrb_ctx* ctx = comm->ctx;
  HRB_COMM_CUDA(ctx, cudaSetDevice(hrb::ctx_device(ctx)));
  auto s = stream != nullptr ? static_cast<cudaStream_t>(stream)
                             : static_cast<cudaStream_t>(hrb_get_stream(ctx));
  // One byte per rank, gathered in place: it completes on a rank once every
  // rank's stream has reached it.
  HRB_COMM_NCCL(ctx, nccl().all_gather(comm->d_fence + comm->rank, comm->d_fence, 1, ncclInt8,
                                       comm->comm, s));
  return HRB_OK;
}

hrb_status hrb_comm_destroy(hrb_comm* comm) {
  if (comm == nullptr) return HRB_OK;
  cudaSetDevice(hrb::ctx_device(comm->ctx));
  cudaStreamSynchronize(static_cast<cudaStream_t>(hrb_get_stream(comm->ctx)));
  if (comm->comm != nullptr) nccl().destroy(comm->comm);
  if (comm->d_scratch != nullptr) cudaFree(comm->d_scratch);
  if (comm->d_fence != nullptr) cudaFree(comm->d_fence);
  delete comm;
  return HRB_OK;
}

hrb_status hrb_comm_exchange(hrb_comm* comm, const void* mine, void* all, size_t bytes) {
  if (comm == nullptr || mine == nullptr || all == nullptr || bytes == 0) return HRB_EINVAL;
  hrb_ctx* ctx = comm->ctx;
  HRB_COMM_CUDA(ctx, cudaSetDevice(hrb::ctx_device(ctx)));
  const hrb_status st = grow_scratch(comm, bytes * comm->ranks);
  if (st != HRB_OK) return st;
  auto s = static_cast<cudaStream_t>(hrb_get_stream(ctx));
  auto* base = static_cast<uint8_t*>(comm->d_scratch);
  HRB_COMM_CUDA(ctx, cudaMemcpyAsync(base + bytes * comm->rank, mine, bytes,
                                     cudaMemcpyHostToDevice, s));
  HRB_COMM_NCCL(ctx, nccl().all_gather(base + bytes * comm->rank, base, bytes, ncclInt8,
                                       comm->comm, s));
  HRB_COMM_CUDA(ctx, cudaMemcpyAsync(all, base, bytes * comm->ranks, cudaMemcpyDeviceToHost, s));
  HRB_COMM_CUDA(ctx, cudaStreamSynchronize(s));
  return HRB_OK;
}

hrb_status hrb_comm_barrier(hrb_comm* comm) {
  if (comm == nullptr) return HRB_EINVAL;
  hrb_ctx* ctx = comm->ctx;
  HRB_COMM_CUDA(ctx, cudaSetDevice(hrb::ctx_device(ctx)));
  HRB_COMM_CUDA(ctx, cudaStreamSynchronize(static_cast<cudaStream_t>(hrb_get_stream(ctx))));
  std::vector<uint8_t> all(comm->ranks);
  const uint8_t one = 1;
  return hrb_comm_exchange(comm, &one, all.data(), 1);
}

hrb_status hrb_comm_allgather(hrb_comm* comm, void* buf, const uint64_t* offsets, void* stream) {
  if (comm == nullptr || buf == nullptr || offsets == nullptr) return HRB_EINVAL;
  hrb_ctx* ctx = comm->ctx;
  const uint32_t G = comm->ranks;
  for (uint32_t r = 0; r < G; ++r) {
    if (offsets[r + 1] < offsets[r]) return hrb::ctx_fail(ctx, HRB_EINVAL, "offsets decrease");
  }
  HRB_COMM_CUDA(ctx, cudaSetDevice(hrb::ctx_device(ctx)));
  auto s = stream != nullptr ? static_cast<cudaStream_t>(stream)
                             : static_cast<cudaStream_t>(hrb_get_stream(ctx));
  auto* base = static_cast<uint8_t*>(buf);
  const uint64_t part = offsets[1] - offsets[0];
  bool equal = true;
  for (uint32_t r = 0; r < G; ++r) equal &= offsets[r + 1] - offsets[r] == part;
  if (equal) {
    if (part == 0) return HRB_OK;
    // In place: rank r's part already sits at its offset of the output.
    HRB_COMM_NCCL(ctx, nccl().all_gather(base + offsets[comm->rank], base + offsets[0], part,
                                         ncclInt8, comm->comm, s));
    return HRB_OK;
  }
  // Ragged parts: one broadcast per rank, rooted at its owner, in a group.
  HRB_COMM_NCCL(ctx, nccl().group_start());
  for (uint32_t r = 0; r < G; ++r) {
    const uint64_t bytes = offsets[r + 1] - offsets[r];
    if (bytes == 0) continue;
    const ncclResult_t res = nccl().broadcast(base + offsets[r], base + offsets[r], bytes,
                                              ncclInt8, static_cast<int>(r), comm->comm, s);
    if (res != ncclSuccess) {
      nccl().group_end();
      return nccl_fail(ctx, res, "ncclBroadcast");
    }
  }
  HRB_COMM_NCCL(ctx, nccl().group_end());
  return HRB_OK;
}

void hrb_shard_rows(uint32_t units, uint32_t rank, uint32_t ranks, uint32_t* u0, uint32_t* u1) {
  if (u0 == nullptr || u1 == nullptr) return;
  if (ranks == 0 || rank >= ranks) {
    *u0 = *u1 = 0;
    return;
  }
  *u0 = static_cast<uint32_t>(static_cast<uint64_t>(units) * rank / ranks);
  *u1 = static_cast<uint32_t>(static_cast<uint64_t>(units) * (rank + 1) / ranks);
}

}  // extern "C"
