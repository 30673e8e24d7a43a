// Test program for the C++ host side of the sharded paths
// (hotarubi_b200/host/shard_host.hpp over the C ABI), with no framework.
//
//   test_shard_host <ranks>
//
// The parent forks one process per GPU before any CUDA call and hands rank
// 0's communicator id to the others through pipes.  Each rank then checks,
// on its own GPU, against the unsharded result computed there:
//   * a column-sharded MXFP4 GEMM (hrb_shard_columns) whose epilogue stores
//     every output into all ranks' C (hrb_plan_set_peers), bit for bit;
//   * a row-sharded 3x3 convolution (hrb_shard_rows over the images) whose
//     epilogue stores its FP32 output and MXINT8 copy into all ranks
//     (hrb_conv_plan_set_peers), bit for bit;
//   * the communicator's in-place all-gather of the convolution's row
//     ranges (hrb_comm_allgather), bit for bit.
// Exit status 0 when every rank passed; the parent kills the ranks after
// 240 s.
#include <cuda_runtime.h>
#include <signal.h>
#include <sys/wait.h>
#include <unistd.h>

#include <chrono>
#include <cstdio>
#include <cstdlib>
#include <cstring>
#include <random>
#include <thread>
#include <vector>

#include "shard_host.hpp"

namespace host = hrb::host;

namespace {

#define CUDA_OK(call)                                                              \
  do {                                                                             \
    const cudaError_t e_ = (call);                                                 \
    if (e_ != cudaSuccess) throw host::Error(HRB_ECUDA, std::string(#call) + ": " + \
                                             cudaGetErrorString(e_));              \
  } while (0)

struct Dev {
  void* p = nullptr;
  explicit Dev(size_t bytes) { CUDA_OK(cudaMalloc(&p, bytes)); }
  ~Dev() { cudaFree(p); }
  template <typename T>
  T* as() const { return static_cast<T*>(p); }
};

template <typename T>
Dev upload(const std::vector<T>& v) {
  Dev d(v.size() * sizeof(T));
  CUDA_OK(cudaMemcpy(d.p, v.data(), v.size() * sizeof(T), cudaMemcpyHostToDevice));
  return d;
}

std::vector<uint8_t> download(const void* p, size_t bytes) {
  std::vector<uint8_t> v(bytes);
  CUDA_OK(cudaMemcpy(v.data(), p, bytes, cudaMemcpyDeviceToHost));
  return v;
}

std::vector<float> normal(size_t n, uint32_t seed) {
  std::mt19937 gen(seed);
  std::normal_distribution<float> d(0.0f, 1.0f);
  std::vector<float> v(n);
  for (auto& x : v) x = d(gen);
  return v;
}

// MXFP4 weights: any byte is two valid E2M1 codes; scale bytes 117..123.
void mxfp4(uint32_t n, uint32_t k, uint32_t seed, std::vector<uint8_t>& w,
           std::vector<uint8_t>& ws) {
  std::mt19937 gen(seed);
  std::uniform_int_distribution<uint32_t> byte(0, 255), scale(117, 123);
  w.resize(static_cast<size_t>(n) * k / 2);
  ws.resize(static_cast<size_t>(n) * k / 32);
  for (auto& b : w) b = static_cast<uint8_t>(byte(gen));
  for (auto& s : ws) s = static_cast<uint8_t>(scale(gen));
}

void expect_equal(const std::vector<uint8_t>& got, const std::vector<uint8_t>& want,
                  const char* what, uint32_t rank) {
  if (got != want) {
    size_t i = 0;
    while (i < got.size() && got[i] == want[i]) ++i;
    throw host::Error(HRB_EDATA, std::string(what) + ": rank " + std::to_string(rank) +
                                     " differs from the unsharded result at byte " +
                                     std::to_string(i));
  }
}

void columns(hrb_ctx* ctx, host::Comm& comm) {
  const uint32_t M = 96, N = 1000, K = 768, kb = K / 32;
  const auto x = normal(static_cast<size_t>(M) * K, 11);
  std::vector<uint8_t> w, ws;
  mxfp4(N, K, 12, w, ws);
  Dev dx = upload(x), dw = upload(w), dws = upload(ws), ref(M * N * 4);
  hrb_gemm_desc d{};
  d.wfmt = HRB_WFMT_MXFP4;
  d.mode = HRB_MODE_FAST;
  d.M = M;
  d.N = N;
  d.K = K;
  d.a = dx.as<float>();
  d.lda = K;
  d.w = dw.as<uint8_t>();
  d.wscale = dws.as<uint8_t>();
  d.c = ref.as<float>();
  d.ldc = N;
  hrb_plan* full = nullptr;
  host::check(hrb_plan_create(ctx, &d, 1, &full), ctx, "plan (full)");
  host::check(hrb_plan_run(full, nullptr, nullptr), ctx, "run (full)");
  host::check(hrb_sync(ctx), ctx, "sync");
  host::PeerBuffer out(ctx, comm, static_cast<size_t>(M) * N * 4);
  CUDA_OK(cudaMemset(out.local(), 0, static_cast<size_t>(M) * N * 4));
  uint32_t n0 = 0, n1 = 0;
  hrb_shard_columns(N, comm.rank(), comm.ranks(), &n0, &n1);
  hrb_plan* mine = nullptr;
  if (n1 > n0) {
    hrb_gemm_desc s = d;
    s.N = n1 - n0;
    s.w = dw.as<uint8_t>() + static_cast<size_t>(n0) * K / 2;
    s.wscale = dws.as<uint8_t>() + static_cast<size_t>(n0) * kb;
    s.c = static_cast<float*>(out.local()) + n0;
    host::check(hrb_plan_create(ctx, &s, 1, &mine), ctx, "plan (shard)");
    host::check(hrb_plan_set_peers(mine, out.local(), out.peers().data(),
                                   static_cast<uint32_t>(out.peers().size())),
                ctx, "hrb_plan_set_peers");
  }
  CUDA_OK(cudaDeviceSynchronize());
  comm.barrier();
  if (mine != nullptr) host::check(hrb_plan_run(mine, nullptr, nullptr), ctx, "run (shard)");
  comm.fence();
  host::check(hrb_sync(ctx), ctx, "sync");
  expect_equal(download(out.local(), M * N * 4), download(ref.p, M * N * 4), "column shard",
               comm.rank());
  comm.barrier();
  hrb_plan_destroy(mine);
  hrb_plan_destroy(full);
  comm.barrier();
}

void rows(hrb_ctx* ctx, host::Comm& comm) {
  const uint32_t images = 6, H = 8, W = 12, cin = 256, cout = 256, kh = 3;
  const uint32_t hw = H * W, per = hw, M = images * per, K = kh * kh * cin;
  const uint32_t kpn = cout, kbn = kpn / 32;
  const auto x = normal(static_cast<size_t>(images) * hw * cin, 21);
  auto bias = normal(cout, 22);
  for (auto& b : bias) b *= 0.01f;
  std::vector<uint8_t> w, ws;
  mxfp4(cout, K, 23, w, ws);
  Dev dx = upload(x), dw = upload(w), dws = upload(ws), db = upload(bias);
  const size_t c_bytes = static_cast<size_t>(M) * cout * 4;
  const size_t q_bytes = static_cast<size_t>(M) * kpn, s_bytes = static_cast<size_t>(M) * kbn;
  Dev ref(c_bytes), ref_q(q_bytes), ref_s(s_bytes);
  hrb_conv_desc d{};
  d.wfmt = HRB_WFMT_MXFP4;
  d.mode = HRB_MODE_FAST;
  d.images = images;
  d.H = H;
  d.W = W;
  d.cin = cin;
  d.cout = cout;
  d.kh = kh;
  d.stride = 1;
  d.order = HRB_CONV_YMAJOR;
  d.a = dx.as<float>();
  d.w = dw.as<uint8_t>();
  d.wscale = dws.as<uint8_t>();
  d.bias = db.as<float>();
  d.c = ref.as<float>();
  d.relu = 1;
  d.cq = ref_q.as<int8_t>();
  d.cscale = ref_s.as<uint8_t>();
  d.cquant = HRB_QUANT_VEC;
  hrb_conv_plan* full = nullptr;
  host::check(hrb_conv_plan_create(ctx, &d, &full), ctx, "conv plan (full)");
  host::check(hrb_conv_plan_run(full, nullptr, nullptr), ctx, "conv run (full)");
  host::check(hrb_sync(ctx), ctx, "sync");
  // FP32 rows, then the MXINT8 codes and scales, in one shared buffer.
  const size_t oq = (c_bytes + 255) / 256 * 256, os = oq + (q_bytes + 255) / 256 * 256;
  host::PeerBuffer out(ctx, comm, os + s_bytes);
  auto* base = static_cast<uint8_t*>(out.local());
  CUDA_OK(cudaMemset(base, 0, os + s_bytes));
  uint32_t i0 = 0, i1 = 0;
  hrb_shard_rows(images, comm.rank(), comm.ranks(), &i0, &i1);
  const size_t r0 = static_cast<size_t>(i0) * per;
  hrb_conv_plan* mine = nullptr;
  if (i1 > i0) {
    hrb_conv_desc s = d;
    s.images = i1 - i0;
    s.a = dx.as<float>() + static_cast<size_t>(i0) * hw * cin;
    s.c = reinterpret_cast<float*>(base) + r0 * cout;
    s.cq = reinterpret_cast<int8_t*>(base + oq) + r0 * kpn;
    s.cscale = base + os + r0 * kbn;
    host::check(hrb_conv_plan_create(ctx, &s, &mine), ctx, "conv plan (shard)");
    host::check(hrb_conv_plan_set_peers(mine, base, out.peers().data(),
                                        static_cast<uint32_t>(out.peers().size())),
                ctx, "hrb_conv_plan_set_peers");
  }
  CUDA_OK(cudaDeviceSynchronize());
  comm.barrier();
  if (mine != nullptr) host::check(hrb_conv_plan_run(mine, nullptr, nullptr), ctx, "conv run");
  comm.fence();
  host::check(hrb_sync(ctx), ctx, "sync");
  expect_equal(download(base, c_bytes), download(ref.p, c_bytes), "row shard (FP32)",
               comm.rank());
  expect_equal(download(base + oq, q_bytes), download(ref_q.p, q_bytes), "row shard (codes)",
               comm.rank());
  expect_equal(download(base + os, s_bytes), download(ref_s.p, s_bytes), "row shard (scales)",
               comm.rank());
  // The communicator's all-gather of the same row ranges.
  Dev loose(c_bytes);
  CUDA_OK(cudaMemset(loose.p, 0, c_bytes));
  const size_t row_bytes = static_cast<size_t>(cout) * 4;
  CUDA_OK(cudaMemcpy(loose.as<uint8_t>() + r0 * row_bytes, ref.as<uint8_t>() + r0 * row_bytes,
                     (static_cast<size_t>(i1) * per - r0) * row_bytes, cudaMemcpyDeviceToDevice));
  comm.barrier();
  comm.allgather(loose.p, host::row_offsets(images, per * row_bytes, comm.ranks()));
  host::check(hrb_sync(ctx), ctx, "sync");
  expect_equal(download(loose.p, c_bytes), download(ref.p, c_bytes), "communicator all-gather",
               comm.rank());
  comm.barrier();
  hrb_conv_plan_destroy(mine);
  hrb_conv_plan_destroy(full);
  comm.barrier();
}

int rank_main(uint32_t rank, uint32_t ranks, const std::vector<int>& to_rank, int from_zero) {
  hrb_comm_id id{};
  if (rank == 0) {
    host::check(hrb_comm_id_new(&id), nullptr, "hrb_comm_id_new");
    for (uint32_t r = 1; r < ranks; ++r) {
      if (write(to_rank[r], id.bytes, sizeof(id.bytes)) != static_cast<ssize_t>(sizeof(id.bytes))) {
        std::fprintf(stderr, "rank 0: pipe write failed\n");
        return 2;
      }
    }
  } else {
    size_t got = 0;
    while (got < sizeof(id.bytes)) {
      const ssize_t n = read(from_zero, id.bytes + got, sizeof(id.bytes) - got);
      if (n <= 0) {
        std::fprintf(stderr, "rank %u: no id from rank 0\n", rank);
        return 2;
      }
      got += static_cast<size_t>(n);
    }
  }
  hrb_ctx* ctx = nullptr;
  host::check(hrb_create(static_cast<int>(rank), &ctx), nullptr, "hrb_create");
  {
    host::Comm comm(ctx, id, rank, ranks);
    columns(ctx, comm);
    rows(ctx, comm);
    comm.barrier();
  }
  hrb_destroy(ctx);
  std::printf("rank %u ok\n", rank);
  return 0;
}

}  // namespace

int main(int argc, char** argv) {
  const uint32_t ranks = argc > 1 ? static_cast<uint32_t>(std::atoi(argv[1])) : 2u;
  if (ranks < 1 || ranks > 8) {
    std::fprintf(stderr, "usage: test_shard_host <ranks 1..8>\n");
    return 2;
  }
  // No CUDA call before the fork: each rank initialises its own GPU.
  std::vector<int> rd(ranks, -1), wr(ranks, -1);
  for (uint32_t r = 1; r < ranks; ++r) {
    int fd[2];
    if (pipe(fd) != 0) return 2;
    rd[r] = fd[0];
    wr[r] = fd[1];
  }
  std::vector<pid_t> pids;
  for (uint32_t r = 0; r < ranks; ++r) {
    const pid_t pid = fork();
    if (pid < 0) return 2;
    if (pid == 0) {
      // Only rank 0 writes: the others drop the write ends, so that a read
      // sees the end of the pipe if rank 0 dies.
      if (r != 0) {
        for (uint32_t q = 1; q < ranks; ++q) close(wr[q]);
      }
      int rc = 1;
      try {
        rc = rank_main(r, ranks, wr, rd[r]);
      } catch (const std::exception& e) {
        std::fprintf(stderr, "rank %u: %s\n", r, e.what());
        rc = 1;
      }
      std::fflush(stdout);
      std::fflush(stderr);
      _exit(rc);
    }
    pids.push_back(pid);
  }
  for (uint32_t r = 1; r < ranks; ++r) {
    close(rd[r]);
    close(wr[r]);
  }
  int failed = 0;
  const auto deadline = std::chrono::steady_clock::now() + std::chrono::seconds(240);
  size_t done = 0;
  std::vector<bool> finished(ranks, false);
  while (done < ranks) {
    for (uint32_t r = 0; r < ranks; ++r) {
      if (finished[r]) continue;
      int status = 0;
      if (waitpid(pids[r], &status, WNOHANG) == pids[r]) {
        finished[r] = true;
        ++done;
        if (!WIFEXITED(status) || WEXITSTATUS(status) != 0) {
          std::fprintf(stderr, "rank %u failed (status %d)\n", r, status);
          failed = 1;
        }
      }
    }
    if (done < ranks && std::chrono::steady_clock::now() > deadline) {
      std::fprintf(stderr, "ranks did not finish in 240 s\n");
      for (uint32_t r = 0; r < ranks; ++r) {
        if (!finished[r]) kill(pids[r], SIGKILL);
      }
      for (uint32_t r = 0; r < ranks; ++r) {
        if (!finished[r]) waitpid(pids[r], nullptr, 0);
      }
      return 3;
    }
    std::this_thread::sleep_for(std::chrono::milliseconds(20));
  }
  return failed;
}
