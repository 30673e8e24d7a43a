// The C++ host side of the sharded GEMMs and convolutions: RAII over the C
// ABI's communicator (hrb_comm_*) and IPC buffers (hrb_shared_alloc,
// hrb_peer_open), for hosts that run one process per GPU without a
// framework.  A rank:
//
//   hrb::host::Comm comm(ctx, id, rank, ranks);      // id from rank 0
//   hrb::host::PeerBuffer out(ctx, comm, bytes);     // mapped on every rank
//   ... plan over this rank's columns (hrb_shard_columns) or images
//   (hrb_shard_rows), outputs at their place in out.local() ...
//   hrb_plan_set_peers(plan, out.local(), out.peers().data(), out.peers().size());
//   hrb_plan_run(plan, stream, nullptr);
//   comm.fence(stream);                              // every rank holds all
//
// Errors become hrb::host::Error exceptions here, on the host side of the
// ABI; nothing throws across it.
#pragma once

#include <cstdint>
#include <cstring>
#include <stdexcept>
#include <string>
#include <vector>

#include "hrb_gemm.h"

namespace hrb::host {

class Error : public std::runtime_error {
 public:
  Error(hrb_status status, const std::string& what)
      : std::runtime_error(what), status_(status) {}
  hrb_status status() const { return status_; }

 private:
  hrb_status status_;
};

inline void check(hrb_status st, const hrb_ctx* ctx, const char* what) {
  if (st != HRB_OK) {
    throw Error(st, std::string(what) + ": " + hrb_status_string(st) + ": " + hrb_last_error(ctx));
  }
}

class Comm {
 public:
  Comm(hrb_ctx* ctx, const hrb_comm_id& id, uint32_t rank, uint32_t ranks)
      : ctx_(ctx), rank_(rank), ranks_(ranks) {
    check(hrb_comm_create(ctx, &id, rank, ranks, &comm_), ctx, "hrb_comm_create");
  }
  ~Comm() { hrb_comm_destroy(comm_); }
  Comm(const Comm&) = delete;
  Comm& operator=(const Comm&) = delete;

  // Every rank's record of `bytes`, in rank order.
  std::vector<std::vector<uint8_t>> exchange(const void* mine, size_t bytes) {
    std::vector<uint8_t> all(bytes * ranks_);
    check(hrb_comm_exchange(comm_, mine, all.data(), bytes), ctx_, "hrb_comm_exchange");
    std::vector<std::vector<uint8_t>> out(ranks_);
    for (uint32_t r = 0; r < ranks_; ++r) {
      out[r].assign(all.begin() + r * bytes, all.begin() + (r + 1) * bytes);
    }
    return out;
  }
  void barrier() { check(hrb_comm_barrier(comm_), ctx_, "hrb_comm_barrier"); }
  void fence(void* stream = nullptr) {
    check(hrb_comm_fence(comm_, stream), ctx_, "hrb_comm_fence");
  }
  void allgather(void* buf, const std::vector<uint64_t>& offsets, void* stream = nullptr) {
    if (offsets.size() != ranks_ + 1u) throw Error(HRB_EINVAL, "allgather: ranks + 1 offsets");
    check(hrb_comm_allgather(comm_, buf, offsets.data(), stream), ctx_, "hrb_comm_allgather");
  }
  uint32_t rank() const { return rank_; }
  uint32_t ranks() const { return ranks_; }
  hrb_comm* get() const { return comm_; }

 private:
  hrb_ctx* ctx_;
  hrb_comm* comm_ = nullptr;
  uint32_t rank_, ranks_;
};

// A device buffer on every rank, each mapped into every other rank: the
// target of the fused all-gather's peer stores.
class PeerBuffer {
 public:
  PeerBuffer(hrb_ctx* ctx, Comm& comm, size_t bytes) : ctx_(ctx) {
    hrb_ipc_handle mine;
    check(hrb_shared_alloc(ctx, bytes, &local_, &mine), ctx, "hrb_shared_alloc");
    const auto all = comm.exchange(&mine, sizeof(mine));
    for (uint32_t r = 0; r < comm.ranks(); ++r) {
      if (r == comm.rank()) continue;
      hrb_ipc_handle h;
      std::memcpy(&h, all[r].data(), sizeof(h));
      void* p = nullptr;
      check(hrb_peer_open(ctx, &h, &p), ctx, "hrb_peer_open");
      peers_.push_back(p);
    }
  }
  ~PeerBuffer() {
    for (void* p : peers_) hrb_peer_close(ctx_, p);
    if (local_ != nullptr) hrb_shared_free(ctx_, local_);
  }
  PeerBuffer(const PeerBuffer&) = delete;
  PeerBuffer& operator=(const PeerBuffer&) = delete;

  void* local() const { return local_; }
  // The other ranks' buffers, in rank order without this rank.
  const std::vector<void*>& peers() const { return peers_; }

 private:
  hrb_ctx* ctx_;
  void* local_ = nullptr;
  std::vector<void*> peers_;
};

// Byte offsets of every rank's rows, for Comm::allgather: `units` units of
// `unit_bytes`, split by hrb_shard_rows.
inline std::vector<uint64_t> row_offsets(uint32_t units, uint64_t unit_bytes, uint32_t ranks) {
  std::vector<uint64_t> out;
  for (uint32_t r = 0; r < ranks; ++r) {
    uint32_t u0 = 0, u1 = 0;
    hrb_shard_rows(units, r, ranks, &u0, &u1);
    out.push_back(u0 * unit_bytes);
  }
  out.push_back(static_cast<uint64_t>(units) * unit_bytes);
  return out;
}

}  // namespace hrb::host
