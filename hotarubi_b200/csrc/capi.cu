// The C ABI of include/hrb_gemm.h: argument checks, contexts, memory
// staging, plans, and the dispatch onto the kernels.
//
// Error convention: where hotarubi's ExecuteGemm / EncodeMxint8 call Require()
// (tools/iss/gemm_array.cpp:113-119, tools/runtime/formats.cpp:37) the entry
// points return HRB_EINVAL / HRB_EDATA with the same message text; nothing
// aborts inside the library.
#include <cuda_runtime.h>

#include <algorithm>
#include <cstdarg>
#include <cstdint>
#include <cstdio>
#include <cstdlib>
#include <cstring>
#include <mutex>
#include <new>
#include <string>
#include <vector>

#include "hrb_gemm.h"
#include "hrb_kernels.cuh"
#include "hrb_tc.cuh"

struct hrb_ctx {
  int device = 0;
  cudaStream_t stream = nullptr;
  bool own_stream = false;
  int sm_count = 148;
  std::string last_error;
  uint64_t launches = 0;
  // ISS memories mirrored on the device for hrb_gemm_exec.
  uint8_t* d_abuf = nullptr;
  uint8_t* d_wbuf = nullptr;
  float* d_fbuf = nullptr;
  // Scratch: the MXINT8 activations of an FP32-input GEMM.
  void* scratch = nullptr;
  size_t scratch_bytes = 0;
  // Operand staging for hrb_gemm_dense_host.
  void* staging = nullptr;
  size_t staging_bytes = 0;
  // The int8 weight chunks of the tensor-core exact GEMM (launch_x_translate).
  void* xscratch = nullptr;
  size_t xscratch_bytes = 0;
  // Bit 0: the encoder met Inf/NaN; bit 1: a tensor-core kernel gave up
  // waiting (it then leaves its outputs unwritten).
  uint32_t* d_error = nullptr;
};

struct hrb_conv_plan {
  hrb_ctx* ctx = nullptr;
  hrb_conv_desc desc{};
  void* d_scratch = nullptr;
  // Peers that receive every output (hrb_conv_plan_set_peers).
  hrb::MxPeers peers{};
};

struct hrb_plan {
  hrb_ctx* ctx = nullptr;
  void* d_jobs = nullptr;   // QuantJobs then DenseJobs
  void* d_scratch = nullptr;
  uint32_t nquant = 0;
  uint64_t quant_units = 0;
  const hrb::QuantJob* d_quant = nullptr;
  // Activations of kind::mxf4 GEMMs: the digit-plane encoder's jobs.
  uint32_t nplanes = 0;
  uint64_t plane_units = 0;
  uint64_t plane_groups = 0;  // the same jobs counted in 4-step groups
  const hrb::QuantJob* d_planes = nullptr;
  std::vector<hrb::QuantJob> d_planes_host;  // the same jobs on the host
  // MXINT8 copies of the exact GEMMs' outputs, encoded after them.
  uint32_t npost = 0;
  uint64_t post_units = 0;
  const hrb::QuantJob* d_post = nullptr;
  struct Group {
    uint32_t wfmt;
    uint32_t kind;  // 0 exact kernel, 1 exact tensor-core kernel, 2 block-scaled tensor-core kernel
    uint32_t nt, njobs, tiles;
    const void* d_jobs;  // DenseJob (kind 0), XJob (kind 1) or TcJob (kind 2) array
    const hrb::MxTile* d_tiles;  // kind 2: the launch's output tiles
    bool pairs = false;          // kind 2: d_tiles in pair order (CTA pairs)
  };
  std::vector<Group> groups;
  // Per GEMM, in creation order: the device activations and output the
  // descriptor names, for hrb_plan_run_host.
  struct Io {
    void* a;          // FP32 [M][lda], or MXINT8 codes [M][kp] when a is not given
    size_t a_bytes;
    void* ascale;     // MXINT8 scales [M][kb] (MXINT8 input only)
    size_t ascale_bytes;
    void* c;          // [M][ldc]
    size_t c_bytes;
    uint32_t tile_begin, tiles;  // output tiles in the kind::mxf4 group
  };
  std::vector<Io> io;
  // hrb_plan_run_host pipelines chunks of GEMMs (copy in / compute / copy
  // out on three streams) when the plan is one kind::mxf4 group fed by the
  // digit-plane encoder; created on first use.
  cudaStream_t s_in = nullptr, s_out = nullptr;
  std::vector<cudaEvent_t> events;
  // Peers that receive every output (hrb_plan_set_peers).
  hrb::MxPeers peers{};
};

namespace {

// Messages of calls made without a context (hrb_last_error(NULL)).
thread_local std::string t_last_error;

hrb_status fail(hrb_ctx* ctx, hrb_status status, const char* fmt, ...) {
  char buf[512];
  va_list ap;
  va_start(ap, fmt);
  std::vsnprintf(buf, sizeof buf, fmt, ap);
  va_end(ap);
  (ctx != nullptr ? ctx->last_error : t_last_error) = buf;
  return status;
}

hrb_status cuda_fail(hrb_ctx* ctx, cudaError_t err, const char* what) {
  return fail(ctx, err == cudaErrorMemoryAllocation ? HRB_ENOMEM : HRB_ECUDA, "%s: %s", what,
              cudaGetErrorString(err));
}

#define HRB_CUDA(ctx, call)                                   \
  do {                                                        \
    const cudaError_t err_ = (call);                          \
    if (err_ != cudaSuccess) return cuda_fail(ctx, err_, #call); \
  } while (0)

cudaStream_t pick(hrb_ctx* ctx, void* stream) {
  return stream != nullptr ? static_cast<cudaStream_t>(stream) : ctx->stream;
}

// Grows a device buffer owned by the context (synchronous allocation).
hrb_status grow(hrb_ctx* ctx, void** buf, size_t* have, size_t need) {
  if (*have >= need) return HRB_OK;
  if (*buf != nullptr) {
    HRB_CUDA(ctx, cudaStreamSynchronize(ctx->stream));
    HRB_CUDA(ctx, cudaFree(*buf));
    *buf = nullptr;
    *have = 0;
  }
  const size_t bytes = std::max<size_t>(need, 1u << 20);
  HRB_CUDA(ctx, cudaMalloc(buf, bytes));
  *have = bytes;
  return HRB_OK;
}

size_t align_up(size_t x, size_t a) { return (x + a - 1) / a * a; }

uint32_t blocks_of(uint32_t k) { return (k + 31u) / 32u; }

size_t weight_row_bytes(uint32_t wfmt, uint32_t kb) {
  return wfmt == HRB_WFMT_MXFP4 ? size_t{kb} * 16u : size_t{kb} * 32u;
}

bool aligned(const void* p, uintptr_t a) { return (reinterpret_cast<uintptr_t>(p) % a) == 0; }

// Checks of one dense descriptor; fills the piece list.
hrb_status check_desc(hrb_ctx* ctx, const hrb_gemm_desc* d, uint32_t* pieces,
                      uint32_t* npieces) {
  if (d == nullptr) return fail(ctx, HRB_EINVAL, "null GEMM descriptor");
  if (d->wfmt > HRB_WFMT_MXFP8) return fail(ctx, HRB_EINVAL, "unknown weight format %u", d->wfmt);
  if (d->mode > HRB_MODE_FAST) return fail(ctx, HRB_EINVAL, "unknown mode %u", d->mode);
  if (d->M == 0 || d->N == 0 || d->K == 0) {
    return fail(ctx, HRB_EINVAL, "empty GEMM %u x %u x %u", d->M, d->N, d->K);
  }
  const uint32_t kb = blocks_of(d->K);
  if (d->a != nullptr) {
    if (d->aq != nullptr || d->ascale != nullptr) {
      return fail(ctx, HRB_EINVAL, "give either FP32 activations or MXINT8 ones, not both");
    }
    if (d->lda < d->K) return fail(ctx, HRB_EINVAL, "lda %u < K %u", d->lda, d->K);
    if (d->quant > HRB_QUANT_VEC) return fail(ctx, HRB_EINVAL, "unknown quantizer %u", d->quant);
    if (!aligned(d->a, 4)) return fail(ctx, HRB_EINVAL, "activations are not 4-byte aligned");
  } else {
    if (d->aq == nullptr || d->ascale == nullptr) {
      return fail(ctx, HRB_EINVAL, "no activations");
    }
    if (!aligned(d->aq, 16)) return fail(ctx, HRB_EINVAL, "MXINT8 activations are not 16-byte aligned");
  }
  if (d->w == nullptr || d->wscale == nullptr) {
    return fail(ctx, HRB_EINVAL, "missing weights or weight scales");
  }
  if ((d->cq == nullptr) != (d->cscale == nullptr)) {
    return fail(ctx, HRB_EINVAL, "give both MXINT8 output codes and scales, or neither");
  }
  if (d->cq != nullptr && d->cquant > HRB_QUANT_VEC) {
    return fail(ctx, HRB_EINVAL, "unknown output quantizer %u", d->cquant);
  }
  if (d->ldcq != 0 &&
      (d->cq == nullptr || d->ldcq % 32u != 0 || d->ldcq < blocks_of(d->N) * 32u)) {
    return fail(ctx, HRB_EINVAL, "ldcq %u: needs cq, a multiple of 32 and at least N rounded up "
                                 "to 32 (%u)", d->ldcq, blocks_of(d->N) * 32u);
  }
  if (d->c == nullptr) {
    // Only the fused re-quantisation may stand in for the FP32 output.
    if (d->cq == nullptr || d->mode != HRB_MODE_FAST || d->a == nullptr || d->accumulate) {
      return fail(ctx, HRB_EINVAL, "missing output (an MXINT8-only output needs HRB_MODE_FAST, "
                                   "FP32 activations and no accumulate)");
    }
  }
  if (!aligned(d->w, 16)) return fail(ctx, HRB_EINVAL, "weights are not 16-byte aligned");
  if (d->w8_kernel > HRB_W8_BF16) {
    return fail(ctx, HRB_EINVAL, "unknown W8 kernel %u", d->w8_kernel);
  }
  if (d->wcol_scale != nullptr) {
    if (d->accumulate) {
      return fail(ctx, HRB_EINVAL, "per-column weight scales do not combine with accumulate");
    }
    if (!aligned(d->wcol_scale, 4)) {
      return fail(ctx, HRB_EINVAL, "per-column weight scales are not 4-byte aligned");
    }
  }
  if (d->c != nullptr && d->ldc < d->N) {
    return fail(ctx, HRB_EINVAL, "ldc %u < N %u", d->ldc, d->N);
  }
  if (d->pieces == nullptr || d->npieces == 0) {
    pieces[0] = kb;
    *npieces = 1;
    return HRB_OK;
  }
  if (d->npieces > hrb::kMaxPieces) {
    return fail(ctx, HRB_EINVAL, "%u K pieces (at most %u)", d->npieces, hrb::kMaxPieces);
  }
  uint32_t total = 0;
  for (uint32_t p = 0; p < d->npieces; ++p) {
    if (d->pieces[p] == 0) return fail(ctx, HRB_EINVAL, "K piece %u is empty", p);
    pieces[p] = d->pieces[p];
    total += d->pieces[p];
  }
  if (total != kb) {
    return fail(ctx, HRB_EINVAL, "K pieces cover %u blocks, the GEMM has %u", total, kb);
  }
  *npieces = d->npieces;
  return HRB_OK;
}

hrb::DenseJob make_dense_job(const hrb_gemm_desc* d, const int8_t* aq, const uint8_t* ascale,
                             const uint32_t* pieces, uint32_t npieces) {
  hrb::DenseJob j{};
  j.aq = aq;
  j.ascale = ascale;
  j.w = d->w;
  j.wscale = d->wscale;
  j.bias = d->bias;
  j.colscale = d->wcol_scale;
  j.c = d->c;
  j.M = d->M;
  j.N = d->N;
  j.kb = blocks_of(d->K);
  j.ldc = d->ldc;
  j.wfmt = d->wfmt;
  j.accumulate = d->accumulate != 0;
  j.npieces = npieces;
  for (uint32_t p = 0; p < npieces; ++p) j.pieces[p] = pieces[p];
  return j;
}

hrb::QuantJob make_quant_job(const float* x, uint32_t rows, uint32_t cols, uint32_t ldx,
                             uint32_t quant, int8_t* q, uint8_t* scale) {
  hrb::QuantJob j{};
  j.x = x;
  j.q = q;
  j.scale = scale;
  j.rows = rows;
  j.cols = cols;
  j.ldx = ldx;
  j.kb = blocks_of(cols);
  j.cover_blocks = j.kb;
  j.units = static_cast<uint64_t>(rows) * ((j.kb + 3u) / 4u);
  j.vec_rule = quant == HRB_QUANT_VEC;
  j.vec4 = aligned(x, 16) && (ldx % 4u) == 0;
  return j;
}

// Bytes of MXINT8 scratch for an M x K activation: q then scales, 256-aligned.
size_t act_scratch_bytes(uint32_t M, uint32_t K) {
  const size_t kb = blocks_of(K);
  return align_up(size_t{M} * kb * 32u, 256) + align_up(size_t{M} * kb, 256);
}

// The MXINT8 copy of C for GEMMs that do not take the tensor-core path (its
// epilogue makes the copy itself): the encoder over C, after the GEMM.
hrb::QuantJob post_quant_job(const hrb_gemm_desc* d) {
  hrb::QuantJob j = make_quant_job(d->c, d->M, d->N, d->ldc, d->cquant, d->cq, d->cscale);
  j.ldq = d->ldcq / 32u;
  return j;
}

// The exact GEMM, once activations are MXINT8 on the device.
// MXFP4 and W8 run their block dots on the tensor cores (k_exact_tc) unless
// HRB_EXACT_TC=0; MXFP8 and that switch take k_dense_exact.  Both give the
// same bits.
bool exact_tc(uint32_t wfmt) {
  static const bool on = [] {
    const char* e = std::getenv("HRB_EXACT_TC");
    return e == nullptr || std::strcmp(e, "0") != 0;
  }();
  return on && hrb::x_supported(wfmt);
}

// The tensor-core job of a dense exact job whose weights were translated
// into xw, in tiles of hrb::x_tok(job.M) tokens.
hrb::XJob x_job(const hrb::DenseJob& job, const uint8_t* xw, uint32_t tile_begin) {
  const uint32_t tok = hrb::x_tok(job.M);
  hrb::XJob x{};
  x.d = job;
  x.wt = xw;
  x.wsc = xw + hrb::x_code_bytes(job.wfmt, job.N, job.kb);
  x.planes = job.wfmt == 1 ? 2u : 1u;
  x.steps = (job.kb + 3u) / 4u;
  x.m_tiles = (job.M + tok - 1u) / tok;
  x.n_tiles = (job.N + 127u) / 128u;
  x.tile_begin = tile_begin;
  return x;
}

hrb_status run_dense(hrb_ctx* ctx, const hrb::DenseJob& job, cudaStream_t s) {
  if (exact_tc(job.wfmt)) {
    hrb_status st = grow(ctx, &ctx->xscratch, &ctx->xscratch_bytes,
                         hrb::x_weight_bytes(job.wfmt, job.N, job.kb));
    if (st != HRB_OK) return st;
    uint8_t* xw = static_cast<uint8_t*>(ctx->xscratch);
    hrb::launch_x_translate(job.wfmt, job.w, job.wscale, job.N, job.kb, xw, s);
    const hrb::XJob x = x_job(job, xw, 0);
    const uint32_t tok = hrb::x_tok(job.M);
    const int n = hrb::launch_x_exact(nullptr, 1, &x, hrb::x_tiles(job.M, job.N, tok), tok,
                                      ctx->sm_count, ctx->d_error, s);
    if (n < 0) return fail(ctx, HRB_ECUDA, "k_exact_tc launch failed");
    ctx->launches += 1u + static_cast<uint64_t>(n);
    HRB_CUDA(ctx, cudaGetLastError());
    return HRB_OK;
  }
  hrb::DenseJob one = job;
  uint32_t tiles_n = 0;
  const uint32_t tiles = hrb::dense_exact_tiles(job.M, job.N, tiles_n);
  one.tiles_n = tiles_n;
  one.tile_begin = 0;
  ctx->launches += static_cast<uint64_t>(
      hrb::launch_dense_exact(nullptr, 1, &one, tiles, job.wfmt, s));
  HRB_CUDA(ctx, cudaGetLastError());
  return HRB_OK;
}

// The tensor-core path serves HRB_MODE_FAST GEMMs whose activations arrive
// as FP32 (the encoder then writes the digit planes it streams); MXINT8 input
// runs the exact kernel, whose results are within any tolerance.
bool use_tc(const hrb_gemm_desc* d) { return d->mode == HRB_MODE_FAST && d->a != nullptr; }

// The tensor-core path format of a GEMM (hrb_tc.cuh): its weight format,
// or kTcW8Bf16 for W8 with at most 64 tokens and w8_kernel HRB_W8_BF16.
// Convolutions keep the weight format (their operand gathering writes digit
// planes).
uint32_t tc_fmt(const hrb_gemm_desc* d) {
  return hrb::tc_path_format(d->wfmt, d->M, d->w8_kernel);
}

// Tensor-core bytes of one GEMM in path format pf: prepared activations then
// weight chunks.
size_t tc_act_bytes(const hrb_gemm_desc* d, uint32_t pf) {
  return hrb::mx_act_bytes(pf, d->M, blocks_of(d->K));
}
size_t tc_weight_bytes(const hrb_gemm_desc* d, uint32_t pf) {
  return hrb::mx_weight_bytes(pf, d->N, blocks_of(d->K));
}
// (scale, bias) pairs of a GEMM with per-column scales: 8 bytes a column.
size_t tc_epv_bytes(const hrb_gemm_desc* d) {
  return d->wcol_scale != nullptr ? align_up(size_t{d->N} * 8u, 1024) : 0u;
}
size_t tc_scratch_bytes(const hrb_gemm_desc* d, uint32_t pf) {
  return align_up(tc_act_bytes(d, pf), 1024) + align_up(tc_weight_bytes(d, pf), 1024) +
         tc_epv_bytes(d);
}
size_t tc_scratch_bytes(const hrb_gemm_desc* d) { return tc_scratch_bytes(d, tc_fmt(d)); }

// The encoder job writing the tensor-core operand blocks of an M x K FP32
// activation matrix (layout of hrb_tc.cuh for path format pf).
hrb::QuantJob tc_quant_job(const float* a, uint32_t M, uint32_t K, uint32_t lda, uint32_t quant,
                           uint32_t pf, uint8_t* tiles) {
  const bool f8 = pf == HRB_WFMT_MXFP8, bf = pf == hrb::kTcW8Bf16;
  hrb::QuantJob j = make_quant_job(a, M, K, lda, quant, nullptr, nullptr);
  j.tiles = tiles;
  j.tiles_kind = bf ? 4 : f8 ? 3 : 2;
  j.tile_rows = hrb::mx_tokens_per_tile(M);
  j.k_steps = hrb::mx_steps_of(pf, blocks_of(K));
  j.cover_blocks = (f8 || bf ? 4u : 8u) * j.k_steps;
  // Encoder units: (row, 256 elements), i.e. one E2M1 step or two 128-element steps.
  j.units = static_cast<uint64_t>(j.rows) * (f8 || bf ? (j.k_steps + 1u) / 2u : j.k_steps);
  return j;
}

// Fills the encoder job and the tensor-core job of one GEMM whose prepared
// operands live at `base` (tc_scratch_bytes of them), in path format pf.
// MXFP4 codes and W8 (three E2M1 digit planes) run kind::mxf4, MXFP8 codes
// kind::mxf8f6f4, all with no decode in the kernel; W8 with at most 64
// tokens streams its int8 codes and runs kind::f16 on BF16 converted in
// shared memory.
void tc_jobs(const hrb_gemm_desc* d, uint32_t pf, uint8_t* base, hrb::QuantJob* qj,
             hrb::TcJob* tj) {
  const uint32_t kb = blocks_of(d->K);
  uint8_t* act = base;
  uint8_t* wt = base + align_up(tc_act_bytes(d, pf), 1024);
  *qj = tc_quant_job(d->a, d->M, d->K, d->lda, d->quant, pf, act);
  *tj = hrb::TcJob{};
  tj->wfmt = pf;
  tj->M = d->M;
  tj->N = d->N;
  tj->kb = kb;
  tj->k_steps = qj->k_steps;
  tj->n_tiles = (d->N + 127u) / 128u;
  tj->m_tiles = (d->M + qj->tile_rows - 1) / qj->tile_rows;
  tj->a_tiles = act;
  tj->w_tiles = wt;
  tj->bias = d->bias;
  if (d->wcol_scale != nullptr) {
    tj->epv = reinterpret_cast<const float*>(
        wt + align_up(tc_weight_bytes(d, pf), 1024));  // (scale, bias) pairs after the weights
    tj->bias = nullptr;
  }
  tj->c = d->c;
  tj->ldc = d->ldc;
  tj->accumulate = d->accumulate != 0;
  tj->cq = d->cq;
  tj->cscale = d->cscale;
  tj->cquant = d->cquant;
  tj->ldcq = d->ldcq;
}

// Translates the weights of one tensor-core GEMM into the chunk layout.
// With per-column scales, also interleaves (scale, bias) pairs (bias 0 when
// there is none) with two strided copies.
void tc_translate(const hrb_gemm_desc* d, const hrb::TcJob& tj, cudaStream_t s) {
  hrb::launch_tile_weights_mxf4(tj.wfmt, d->w, d->wscale, d->N, blocks_of(d->K),
                                const_cast<uint8_t*>(tj.w_tiles), s);
  if (tj.epv != nullptr) {
    auto* ep = const_cast<float*>(tj.epv);
    cudaMemcpy2DAsync(ep, 8, d->wcol_scale, 4, 4, d->N, cudaMemcpyDeviceToDevice, s);
    if (d->bias != nullptr) {
      cudaMemcpy2DAsync(ep + 1, 8, d->bias, 4, 4, d->N, cudaMemcpyDeviceToDevice, s);
    } else {
      cudaMemset2DAsync(ep + 1, 8, 0, 4, d->N, s);
    }
  }
}

// ---------------------------------------------------------------------------
// Convolutions: one GEMM with gathered activation rows (conv.cu).

struct ConvRun {
  hrb::ConvGeom g{};
  uint32_t M = 0, N = 0, K = 0;
  bool tc = false;       // HRB_MODE_FAST with FP32 input: the tensor cores
  bool reorder = false;  // more than one channel plane: weights reordered
  bool gather = false;   // MXFP4 with 256-channel planes: the GEMM gathers its own blocks
  uint32_t bpb = 16;     // weight bytes per K block
  uint32_t npieces = 0;  // K pieces of the exact chain (W8: one per (plane, tap) job)
  uint32_t pieces[hrb::kMaxPieces];
  // Scratch, as offsets from the run's base.
  size_t o_w = 0, o_ws = 0;      // reordered weights and scales
  size_t o_map = 0, o_maps = 0;  // exact path, FP32 input: the MXINT8 map
  size_t o_aq = 0, o_as = 0;     // exact path: the gathered MXINT8 rows
  size_t o_tc = 0;               // tensor cores: activation tiles, weight chunks
  size_t o_mt = 0;               // tensor cores: the input map's own operand blocks
  bool xtc = false;              // exact path on k_exact_tc (exact_tc): weights translated once
  size_t o_xw = 0;               // its int8 weight chunks and scales
  size_t bytes = 0;
};

// The GEMM a convolution runs: M output positions x cout x K gathered.
hrb_gemm_desc conv_gemm(const hrb_conv_desc* d, const ConvRun& r, uint8_t* base) {
  hrb_gemm_desc g{};
  g.wfmt = d->wfmt;
  g.mode = d->mode;
  g.M = r.M;
  g.N = r.N;
  g.K = r.K;
  g.quant = d->quant;
  if (r.tc) {
    g.a = d->a;
    g.lda = r.K;
  } else {
    g.aq = reinterpret_cast<const int8_t*>(base + r.o_aq);
    g.ascale = base + r.o_as;
  }
  g.w = r.reorder ? base + r.o_w : d->w;
  g.wscale = r.reorder ? base + r.o_ws : d->wscale;
  g.bias = d->bias;
  g.c = d->c;
  g.ldc = r.N;
  g.accumulate = d->accumulate;
  g.pieces = r.npieces != 0 ? r.pieces : nullptr;
  g.npieces = r.npieces;
  g.cq = d->cq;
  g.cscale = d->cscale;
  g.cquant = d->cquant;
  return g;
}

hrb_status check_conv(hrb_ctx* ctx, const hrb_conv_desc* d, ConvRun* r) {
  if (d == nullptr) return fail(ctx, HRB_EINVAL, "null conv descriptor");
  if (d->wfmt > HRB_WFMT_MXFP8) return fail(ctx, HRB_EINVAL, "unknown weight format %u", d->wfmt);
  if (d->mode > HRB_MODE_FAST) return fail(ctx, HRB_EINVAL, "unknown mode %u", d->mode);
  if (d->kh != 1 && d->kh != 3) {
    return fail(ctx, HRB_EINVAL, "conv with a %ux%u kernel (1x1 and 3x3 only)", d->kh, d->kh);
  }
  if (d->stride != 1 && d->stride != 2) {
    return fail(ctx, HRB_EINVAL, "conv with stride %u (1 and 2 only)", d->stride);
  }
  if (d->order > HRB_CONV_YMAJOR) return fail(ctx, HRB_EINVAL, "unknown position order %u", d->order);
  if (d->images == 0 || d->H / d->stride == 0 || d->W / d->stride == 0 || d->cout == 0) {
    return fail(ctx, HRB_EINVAL, "empty conv");
  }
  // MakeMap's rule (sparsedrive_common.cpp:49-51).
  if (d->cin == 0 || d->cin % 32u != 0 || (d->cin > 256u && d->cin % 256u != 0)) {
    return fail(ctx, HRB_EINVAL, "feature map of %ux%ux%u is not supported", d->H, d->W, d->cin);
  }
  if (d->a != nullptr) {
    if (d->aq != nullptr || d->ascale != nullptr) {
      return fail(ctx, HRB_EINVAL, "give either an FP32 map or an MXINT8 one, not both");
    }
    if (d->quant > HRB_QUANT_VEC) return fail(ctx, HRB_EINVAL, "unknown quantizer %u", d->quant);
    if (!aligned(d->a, 16)) return fail(ctx, HRB_EINVAL, "the FP32 map is not 16-byte aligned");
  } else {
    if (d->aq == nullptr || d->ascale == nullptr) return fail(ctx, HRB_EINVAL, "no input map");
    if (!aligned(d->aq, 16)) return fail(ctx, HRB_EINVAL, "the MXINT8 map is not 16-byte aligned");
  }
  if (d->w == nullptr || d->wscale == nullptr) {
    return fail(ctx, HRB_EINVAL, "missing weights or weight scales");
  }
  if (!aligned(d->w, 16)) return fail(ctx, HRB_EINVAL, "weights are not 16-byte aligned");
  if ((d->cq == nullptr) != (d->cscale == nullptr)) {
    return fail(ctx, HRB_EINVAL, "give both MXINT8 output codes and scales, or neither");
  }
  if (d->cq != nullptr && d->cquant > HRB_QUANT_VEC) {
    return fail(ctx, HRB_EINVAL, "unknown output quantizer %u", d->cquant);
  }
  const bool tc = d->mode == HRB_MODE_FAST && d->a != nullptr;
  if (d->c == nullptr && (d->cq == nullptr || !tc || d->accumulate)) {
    return fail(ctx, HRB_EINVAL, "missing output (an MXINT8-only output needs HRB_MODE_FAST, "
                                 "an FP32 map and no accumulate)");
  }
  ConvRun& x = *r;
  x = ConvRun{};
  const uint32_t plane = d->cin < 256u ? d->cin : 256u;
  x.g = hrb::make_conv_geom(d->images, d->H, d->W, d->cin, d->kh, d->stride, d->order);
  const uint64_t M = uint64_t{d->images} * x.g.Ho * x.g.Wo;
  const uint64_t K = uint64_t{d->kh} * d->kh * d->cin;
  if (M > (1u << 30) || K > (1u << 20) || M * (K / 32u) >= (uint64_t{1} << 32)) {
    return fail(ctx, HRB_EINVAL, "conv too large");
  }
  x.M = static_cast<uint32_t>(M);
  x.N = d->cout;
  x.K = static_cast<uint32_t>(K);
  x.tc = tc;
  x.reorder = d->cin > 256u;
  x.bpb = d->wfmt == HRB_WFMT_MXFP4 ? 16u : 32u;
  const uint32_t jobs = (d->cin / plane) * d->kh * d->kh;
  if (d->wfmt == HRB_WFMT_W8 && !tc) {
    // W8 chains HI then LO per (plane, tap) job (kernels.cpp:35-37).
    if (jobs > hrb::kMaxPieces) {
      return fail(ctx, HRB_EINVAL, "W8 conv with %u (plane, tap) jobs (at most %u)", jobs,
                  hrb::kMaxPieces);
    }
    x.npieces = jobs;
    for (uint32_t i = 0; i < jobs; ++i) x.pieces[i] = x.g.bp;
  } else {
    x.npieces = 1;  // one plane of weights: the chain is the same in any split
    x.pieces[0] = x.K / 32u;
  }
  const size_t kb = K / 32u;
  size_t off = 0;
  auto take = [&](size_t bytes) {
    const size_t o = off;
    off = align_up(off + bytes, 1024);
    return o;
  };
  if (x.reorder) {
    x.o_w = take(size_t{x.N} * kb * x.bpb);
    x.o_ws = take(size_t{x.N} * kb);
  }
  if (tc) {
    const hrb_gemm_desc g = conv_gemm(d, x, nullptr);
    // With 256-channel planes one MXFP4 K step is one (plane, tap), and the
    // GEMM assembles its activation blocks itself from the encoded map.
    x.gather = d->wfmt == HRB_WFMT_MXFP4 && x.g.bp == 8u;
    x.o_tc = take(x.gather ? hrb::mx_weight_bytes(d->wfmt, x.N, x.K / 32u)
                          : tc_scratch_bytes(&g, g.wfmt));
    x.o_mt = take(hrb::mx_act_bytes(d->wfmt, d->images * d->H * d->W, d->cin / 32u));
  } else {
    if (d->a != nullptr) {
      const size_t positions = size_t{d->images} * d->H * d->W;
      x.o_map = take(positions * d->cin);
      x.o_maps = take(positions * (d->cin / 32u));
    }
    x.o_aq = take(size_t{x.M} * kb * 32u);
    x.o_as = take(size_t{x.M} * kb);
    x.xtc = exact_tc(d->wfmt);
    if (x.xtc) x.o_xw = take(hrb::x_weight_bytes(d->wfmt, x.N, static_cast<uint32_t>(kb)));
  }
  x.bytes = off;
  return HRB_OK;
}

// Launches that depend on the weights only: the reorder and, on the tensor
// cores, the translation into chunks (plus zeroing the activation tiles,
// whose rows past M are never written).
hrb_status conv_prepare(hrb_ctx* ctx, const hrb_conv_desc* d, const ConvRun& r, uint8_t* base,
                        cudaStream_t s, uint32_t* launched) {
  if (r.reorder) {
    hrb::launch_conv_weights(d->w, d->wscale, r.N, r.g, r.bpb, base + r.o_w, base + r.o_ws, s);
    *launched += 1;
  }
  if (r.tc) {
    const hrb_gemm_desc g = conv_gemm(d, r, base);
    hrb::QuantJob qj;
    hrb::TcJob tj;
    tc_jobs(&g, g.wfmt, base + r.o_tc, &qj, &tj);
    if (r.gather) {
      tj.w_tiles = base + r.o_tc;  // no prepared activation blocks
    } else {
      HRB_CUDA(ctx, cudaMemsetAsync(base + r.o_tc, 0, align_up(tc_act_bytes(&g, g.wfmt), 1024), s));
    }
    tc_translate(&g, tj, s);
    *launched += 1;
  }
  if (r.xtc) {
    const hrb_gemm_desc g = conv_gemm(d, r, base);
    hrb::launch_x_translate(g.wfmt, g.w, g.wscale, g.N, blocks_of(g.K), base + r.o_xw, s);
    *launched += 1;
  }
  HRB_CUDA(ctx, cudaGetLastError());
  return HRB_OK;
}

// The convolution proper, once prepared.  With `only` >= 0 just that launch
// of the sequence (a profiling aid, as hrb_plan_profile's).
hrb_status conv_execute(hrb_ctx* ctx, const hrb_conv_desc* d, const ConvRun& r, uint8_t* base,
                        cudaStream_t s, uint32_t* launched, int only = -1,
                        const hrb::MxPeers* peers = nullptr) {
  const hrb_gemm_desc g = conv_gemm(d, r, base);
  int index = 0;
  auto take = [&]() { return only < 0 || index++ == only; };
  if (r.tc) {
    // The map encoded once into operand blocks, the GEMM's blocks gathered
    // from them, then the GEMM.
    hrb::QuantJob qj;
    hrb::TcJob tj;
    tc_jobs(&g, g.wfmt, base + r.o_tc, &qj, &tj);
    tj.relu = d->relu != 0;
    const hrb::QuantJob mj = tc_quant_job(d->a, d->images * d->H * d->W, d->cin, d->cin,
                                          d->quant, d->wfmt, base + r.o_mt);
    if (take()) {
      hrb::launch_quantize_planes(nullptr, 1, &mj, mj.units, ctx->d_error, ctx->sm_count, s);
      *launched += 1;
    }
    if (r.gather) {
      if (take()) {
        hrb::MxGather mg{};
        mg.map_tiles = base + r.o_mt;
        mg.map_shift = mj.tile_rows == 64u ? 6u : 7u;
        mg.map_steps = mj.k_steps;
        mg.map_block_bytes = hrb::mx_act_block_bytes(mj.tile_rows);
        mg.rows = r.M;
        mg.geom = r.g;
        tj.w_tiles = base + r.o_tc;
        tj.a_tiles = mg.map_tiles;  // not read: the kernel gathers
        const int n = hrb::launch_mxf4_gather(tj, qj.tile_rows, tj.m_tiles * tj.n_tiles,
                                              ctx->sm_count, ctx->d_error, s, mg, peers);
        if (n < 0) return fail(ctx, HRB_ECUDA, "tensor-core launch failed");
        *launched += static_cast<uint32_t>(n);
      }
      HRB_CUDA(ctx, cudaGetLastError());
      return HRB_OK;
    }
    if (take()) {
      hrb::launch_conv_gather_tiles(base + r.o_mt, mj.tile_rows, mj.k_steps, base + r.o_tc,
                                    qj.tile_rows, qj.k_steps, d->wfmt == HRB_WFMT_MXFP8, r.g, s);
      *launched += 1;
    }
    if (take()) {
      tj.tile_begin = 0;
      const int n = hrb::launch_mxf4(nullptr, &tj, qj.tile_rows, d->wfmt, tj.m_tiles * tj.n_tiles,
                                     ctx->sm_count, ctx->d_error, s, peers);
      if (n < 0) return fail(ctx, HRB_ECUDA, "tensor-core launch failed");
      *launched += static_cast<uint32_t>(n);
    }
    HRB_CUDA(ctx, cudaGetLastError());
    return HRB_OK;
  }
  const int8_t* map = d->aq;
  const uint8_t* maps = d->ascale;
  if (d->a != nullptr) {
    auto* q = reinterpret_cast<int8_t*>(base + r.o_map);
    uint8_t* sc = base + r.o_maps;
    if (take()) {
      const hrb::QuantJob j = make_quant_job(d->a, d->images * d->H * d->W, d->cin, d->cin,
                                             d->quant, q, sc);
      hrb::launch_quantize(nullptr, 1, &j, j.units, ctx->d_error, ctx->sm_count, s);
      *launched += 1;
    }
    map = q;
    maps = sc;
  }
  if (take()) {
    hrb::launch_conv_im2col(map, maps, r.g, reinterpret_cast<int8_t*>(base + r.o_aq),
                            base + r.o_as, s);
    *launched += 1;
  }
  if (take()) {
    const hrb::DenseJob job = make_dense_job(&g, g.aq, g.ascale, r.pieces, r.npieces);
    if (r.xtc) {
      // The weights were translated by conv_prepare.
      const hrb::XJob xj = x_job(job, base + r.o_xw, 0);
      const uint32_t tok = hrb::x_tok(job.M);
      const int n = hrb::launch_x_exact(nullptr, 1, &xj, hrb::x_tiles(job.M, job.N, tok), tok,
                                        ctx->sm_count, ctx->d_error, s);
      if (n < 0) return fail(ctx, HRB_ECUDA, "k_exact_tc launch failed");
      *launched += static_cast<uint32_t>(n);
    } else {
      const uint64_t before = ctx->launches;
      const hrb_status st = run_dense(ctx, job, s);
      *launched += static_cast<uint32_t>(ctx->launches - before);
      ctx->launches = before;
      if (st != HRB_OK) return st;
    }
  }
  if (d->relu && take()) {
    hrb::launch_relu_exact(d->c, r.M, r.N, r.N, s);
    *launched += 1;
  }
  if (d->cq != nullptr && take()) {
    const hrb::QuantJob pq = post_quant_job(&g);
    hrb::launch_quantize(nullptr, 1, &pq, pq.units, ctx->d_error, ctx->sm_count, s);
    *launched += 1;
  }
  HRB_CUDA(ctx, cudaGetLastError());
  return HRB_OK;
}

// Launches of one conv run (the sequence conv_execute walks).
uint32_t conv_launches(const hrb_conv_desc* d, const ConvRun& r) {
  if (r.tc) return r.gather ? 2u : 3u;
  return (d->a != nullptr ? 1u : 0u) + 2u + (d->relu ? 1u : 0u) + (d->cq != nullptr ? 1u : 0u);
}

// ABUF/WBUF/FBUF words a command touches: the circular span from `base` of
// `length` words in a memory of `depth` words, as one or two segments.
struct Span {
  uint32_t first[2], count[2];
  int parts;
};

Span circular(uint64_t base, uint64_t length, uint32_t depth) {
  Span s{};
  if (length >= depth) {
    s.first[0] = 0;
    s.count[0] = depth;
    s.parts = 1;
    return s;
  }
  const uint32_t start = static_cast<uint32_t>(base % depth);
  const uint32_t len = static_cast<uint32_t>(length);
  if (start + len <= depth) {
    s.first[0] = start;
    s.count[0] = len;
    s.parts = 1;
  } else {
    s.first[0] = start;
    s.count[0] = depth - start;
    s.first[1] = 0;
    s.count[1] = len - (depth - start);
    s.parts = 2;
  }
  return s;
}

}  // namespace

namespace hrb {

hrb_status check_desc_for_noalloc(const hrb_gemm_desc* desc, uint32_t* pieces,
                                  uint32_t* npieces) {
  return check_desc(nullptr, desc, pieces, npieces);
}

QuantJob make_quant_job_for_noalloc(const hrb_gemm_desc* d, int8_t* q, uint8_t* scale) {
  return make_quant_job(d->a, d->M, d->K, d->lda, d->quant, q, scale);
}

QuantJob make_post_quant_job_for_noalloc(const hrb_gemm_desc* d) { return post_quant_job(d); }

int ctx_device(const hrb_ctx* ctx) { return ctx->device; }

hrb_status ctx_fail(hrb_ctx* ctx, hrb_status status, const char* message) {
  return fail(ctx, status, "%s", message);
}

hrb_status noalloc_fail(hrb_status status, const char* message) {
  return fail(nullptr, status, "%s", message);
}

hrb_status noalloc_cuda_fail(cudaError_t err, const char* what) {
  return cuda_fail(nullptr, err, what);
}

DenseJob make_dense_job_for_noalloc(const hrb_gemm_desc* d, const int8_t* aq,
                                    const uint8_t* ascale, const uint32_t* pieces,
                                    uint32_t npieces) {
  return make_dense_job(d, aq, ascale, pieces, npieces);
}

}  // namespace hrb

extern "C" {

const char* hrb_status_string(hrb_status status) {
  switch (status) {
    case HRB_OK: return "ok";
    case HRB_EINVAL: return "invalid argument";
    case HRB_ECUDA: return "CUDA error";
    case HRB_ENOMEM: return "out of memory";
    case HRB_ENOTSUP: return "not supported";
    case HRB_EDATA: return "non-finite activation";
  }
  return "unknown status";
}

hrb_status hrb_create(int device, hrb_ctx** out) {
  if (out == nullptr) return HRB_EINVAL;
  *out = nullptr;
  int count = 0;
  if (cudaGetDeviceCount(&count) != cudaSuccess || device < 0 || device >= count) {
    return HRB_EINVAL;
  }
  auto* ctx = new (std::nothrow) hrb_ctx();
  if (ctx == nullptr) return HRB_ENOMEM;
  ctx->device = device;
  cudaError_t err = cudaSetDevice(device);
  if (err == cudaSuccess) err = cudaDeviceGetAttribute(&ctx->sm_count, cudaDevAttrMultiProcessorCount, device);
  if (err == cudaSuccess) err = cudaStreamCreateWithFlags(&ctx->stream, cudaStreamNonBlocking);
  ctx->own_stream = err == cudaSuccess;
  if (err == cudaSuccess) err = cudaMalloc(&ctx->d_error, sizeof(uint32_t));
  if (err == cudaSuccess) err = cudaMemset(ctx->d_error, 0, sizeof(uint32_t));
  if (err != cudaSuccess) {
    hrb_destroy(ctx);
    return err == cudaErrorMemoryAllocation ? HRB_ENOMEM : HRB_ECUDA;
  }
  *out = ctx;
  return HRB_OK;
}

hrb_status hrb_destroy(hrb_ctx* ctx) {
  if (ctx == nullptr) return HRB_OK;
  cudaSetDevice(ctx->device);
  if (ctx->stream != nullptr) cudaStreamSynchronize(ctx->stream);
  cudaFree(ctx->d_abuf);
  cudaFree(ctx->d_wbuf);
  cudaFree(ctx->d_fbuf);
  cudaFree(ctx->scratch);
  cudaFree(ctx->staging);
  cudaFree(ctx->xscratch);
  cudaFree(ctx->d_error);
  if (ctx->own_stream) cudaStreamDestroy(ctx->stream);
  delete ctx;
  return HRB_OK;
}

hrb_status hrb_sync(hrb_ctx* ctx) {
  if (ctx == nullptr) return HRB_EINVAL;
  HRB_CUDA(ctx, cudaSetDevice(ctx->device));
  HRB_CUDA(ctx, cudaStreamSynchronize(ctx->stream));
  uint32_t flag = 0;
  HRB_CUDA(ctx, cudaMemcpy(&flag, ctx->d_error, sizeof flag, cudaMemcpyDeviceToHost));
  if (flag != 0) {
    HRB_CUDA(ctx, cudaMemset(ctx->d_error, 0, sizeof(uint32_t)));
    if (flag & 2u) return fail(ctx, HRB_ECUDA, "a tensor-core GEMM timed out waiting");
    if (flag & 4u) return fail(ctx, HRB_EDATA, "a GACC entry names a row outside the feature rows");
    if (flag & hrb::kErrRowOutside) {
      return fail(ctx, HRB_EDATA, "a ROW_INDEXED entry names a unit outside the DDR window");
    }
    if (flag & hrb::kErrScaleRange) {
      return fail(ctx, HRB_EDATA, "an activation scale byte of 255 has no tensor-core encoding "
                                  "(use HRB_MODE_EXACT)");
    }
    return fail(ctx, HRB_EDATA, "MXINT8 input is infinite or NaN");
  }
  return HRB_OK;
}

const char* hrb_last_error(const hrb_ctx* ctx) {
  return ctx == nullptr ? t_last_error.c_str() : ctx->last_error.c_str();
}

void* hrb_get_stream(const hrb_ctx* ctx) { return ctx == nullptr ? nullptr : ctx->stream; }

hrb_status hrb_set_stream(hrb_ctx* ctx, void* stream) {
  if (ctx == nullptr) return HRB_EINVAL;
  if (ctx->own_stream) {
    cudaStreamSynchronize(ctx->stream);
    cudaStreamDestroy(ctx->stream);
    ctx->own_stream = false;
  }
  ctx->stream = static_cast<cudaStream_t>(stream);
  return HRB_OK;
}

uint64_t hrb_launch_count(const hrb_ctx* ctx) { return ctx == nullptr ? 0 : ctx->launches; }

// ---------------------------------------------------------------------------
// ISS drop-in

hrb_status hrb_gemm_decode(const uint8_t instruction[16], hrb_gemm_cmd* out) {
  if (instruction == nullptr || out == nullptr) return HRB_EINVAL;
  // Little-endian 128-bit word; field (lsb, width) per isa.hpp:75-86.
  auto field = [&](uint32_t lsb, uint32_t width) {
    uint32_t v = 0;
    for (uint32_t i = 0; i < width; ++i) {
      const uint32_t bit = lsb + i;
      v |= static_cast<uint32_t>((instruction[bit / 8] >> (bit % 8)) & 1u) << i;
    }
    return v;
  };
  out->a_base = field(92, 20);
  out->a_stride = field(82, 10);
  out->kb = field(72, 10);
  out->m = field(62, 10);
  out->w_base = field(42, 20);
  out->w_stride = field(32, 10);
  out->n8 = field(24, 8);
  out->c_base = field(4, 20);
  out->wmode = field(2, 2);
  out->acc = field(1, 1);
  return HRB_OK;
}

hrb_status hrb_gemm_check(hrb_ctx* ctx, const hrb_gemm_cmd* c) {
  if (c == nullptr) return fail(ctx, HRB_EINVAL, "null GEMM command");
  if (!(c->m >= 32 && c->m <= 992 && c->m % 32 == 0)) {
    return fail(ctx, HRB_EINVAL, "GEMM m = %u is not a multiple of 32 from 32 to 992", c->m);
  }
  if (!(c->kb >= 1 && c->kb <= c->a_stride)) {
    return fail(ctx, HRB_EINVAL, "GEMM kb = %u is not in [1, a_stride = %u]", c->kb, c->a_stride);
  }
  if (c->n8 < 1) return fail(ctx, HRB_EINVAL, "GEMM n8 = 0");
  return HRB_OK;
}

hrb_status hrb_gemm_accesses(const hrb_gemm_cmd* c, uint8_t* abuf_reads, uint8_t* wbuf_reads,
                             uint8_t* fbuf_reads, uint8_t* fbuf_writes) {
  if (hrb_gemm_check(nullptr, c) != HRB_OK) return HRB_EINVAL;
  if (abuf_reads) std::memset(abuf_reads, 0, HRB_ABUF_WORDS);
  if (wbuf_reads) std::memset(wbuf_reads, 0, HRB_WBUF_WORDS);
  if (fbuf_reads) std::memset(fbuf_reads, 0, HRB_FBUF_WORDS);
  if (fbuf_writes) std::memset(fbuf_writes, 0, HRB_FBUF_WORDS);
  const uint32_t mask = (1u << 20) - 1u;
  for (uint32_t g = 0; g < c->n8; ++g) {
    for (uint32_t b = 0; b < c->kb; ++b) {
      if (wbuf_reads) wbuf_reads[((c->w_base + g * c->w_stride + b) & mask) % HRB_WBUF_WORDS] = 1;
    }
    for (uint32_t q = 0; q < c->m / 4; ++q) {
      const uint32_t word = ((c->c_base + q * c->n8 + g) & mask) % HRB_FBUF_WORDS;
      if (c->acc && fbuf_reads) fbuf_reads[word] = 1;
      if (fbuf_writes) fbuf_writes[word] = 1;
      for (uint32_t b = 0; b < c->kb; ++b) {
        if (abuf_reads) abuf_reads[((c->a_base + q * c->a_stride + b) & mask) % HRB_ABUF_WORDS] = 1;
      }
    }
  }
  return HRB_OK;
}

uint64_t hrb_gemm_npu_cycles(const hrb_gemm_cmd* c) {
  if (c == nullptr) return 0;
  // GemmArrayCycles (timing.cpp:65-67) + gemm_fixed_cycles (timing.hpp:21).
  return uint64_t{c->n8} * (c->m / 32u) * c->kb * 8u + 51u;
}

uint64_t hrb_dense_npu_cycles(uint32_t wfmt, uint32_t M, uint32_t N, uint32_t K) {
  const uint32_t kb = blocks_of(K);
  if (wfmt > HRB_WFMT_W8 || kb == 0 || kb > HRB_WBUF_WORDS || N % 8u != 0 || M == 0) return 0;
  const uint32_t planes = wfmt == HRB_WFMT_W8 ? 2u : 1u;
  // Row chunks and column tiles that fit ABUF, WBUF and FBUF at once.
  uint32_t tile_groups = std::min<uint32_t>(255u, HRB_WBUF_WORDS / kb);
  uint32_t chunk_quads = std::min<uint32_t>(248u, HRB_ABUF_WORDS / kb);
  chunk_quads -= chunk_quads % 8u;
  if (chunk_quads == 0) return 0;
  while (chunk_quads * tile_groups > HRB_FBUF_WORDS) {
    if (tile_groups > 8u) {
      tile_groups /= 2u;
    } else {
      chunk_quads -= 8u;
    }
  }
  const uint32_t quads = (M + 3u) / 4u, groups = N / 8u;
  uint64_t cycles = 0;
  for (uint32_t q0 = 0; q0 < quads; q0 += chunk_quads) {
    const uint32_t m = ((std::min(chunk_quads, quads - q0) * 4u) + 31u) / 32u * 32u;
    for (uint32_t g0 = 0; g0 < groups; g0 += tile_groups) {
      hrb_gemm_cmd c{};
      c.kb = kb;
      c.m = m;
      c.n8 = std::min(tile_groups, groups - g0);
      cycles += planes * hrb_gemm_npu_cycles(&c);
    }
  }
  return cycles;
}

hrb_status hrb_gemm_exec_device(hrb_ctx* ctx, const hrb_gemm_cmd* cmd, const void* abuf,
                                const void* wbuf, void* fbuf, void* stream) {
  if (ctx == nullptr) return HRB_EINVAL;
  const hrb_status st = hrb_gemm_check(ctx, cmd);
  if (st != HRB_OK) return st;
  if (abuf == nullptr || wbuf == nullptr || fbuf == nullptr) {
    return fail(ctx, HRB_EINVAL, "missing GEMM memories");
  }
  HRB_CUDA(ctx, cudaSetDevice(ctx->device));
  const hrb::ExecCmd e{cmd->a_base, cmd->a_stride, cmd->kb, cmd->m, cmd->w_base,
                       cmd->w_stride, cmd->n8, cmd->c_base, cmd->wmode, cmd->acc ? 1u : 0u};
  ctx->launches += static_cast<uint64_t>(hrb::launch_exec(
      e, static_cast<const uint8_t*>(abuf), static_cast<const uint8_t*>(wbuf),
      static_cast<float*>(fbuf), pick(ctx, stream)));
  HRB_CUDA(ctx, cudaGetLastError());
  return HRB_OK;
}

hrb_status hrb_gemm_exec(hrb_ctx* ctx, const hrb_gemm_cmd* cmd, const uint8_t* abuf,
                         const uint8_t* wbuf, uint32_t* fbuf) {
  if (ctx == nullptr) return HRB_EINVAL;
  hrb_status st = hrb_gemm_check(ctx, cmd);
  if (st != HRB_OK) return st;
  if (abuf == nullptr || wbuf == nullptr || fbuf == nullptr) {
    return fail(ctx, HRB_EINVAL, "missing GEMM memories");
  }
  HRB_CUDA(ctx, cudaSetDevice(ctx->device));
  if (ctx->d_abuf == nullptr) {
    HRB_CUDA(ctx, cudaMalloc(&ctx->d_abuf, size_t{HRB_ABUF_WORDS} * HRB_ABUF_WORD_BYTES));
    HRB_CUDA(ctx, cudaMalloc(&ctx->d_wbuf, size_t{HRB_WBUF_WORDS} * HRB_WBUF_WORD_BYTES));
    HRB_CUDA(ctx, cudaMalloc(&ctx->d_fbuf, size_t{HRB_FBUF_WORDS} * 128u));
  }
  const uint64_t quads = cmd->m / 4u;
  // Only the words the command can touch travel.
  const Span a = circular(cmd->a_base, (quads - 1) * cmd->a_stride + cmd->kb, HRB_ABUF_WORDS);
  const Span w = circular(cmd->w_base, uint64_t{cmd->n8 - 1} * cmd->w_stride + cmd->kb,
                          HRB_WBUF_WORDS);
  const Span c = circular(cmd->c_base, quads * cmd->n8, HRB_FBUF_WORDS);
  cudaStream_t s = ctx->stream;
  for (int i = 0; i < a.parts; ++i) {
    const size_t off = size_t{a.first[i]} * HRB_ABUF_WORD_BYTES;
    HRB_CUDA(ctx, cudaMemcpyAsync(ctx->d_abuf + off, abuf + off,
                                  size_t{a.count[i]} * HRB_ABUF_WORD_BYTES,
                                  cudaMemcpyHostToDevice, s));
  }
  for (int i = 0; i < w.parts; ++i) {
    const size_t off = size_t{w.first[i]} * HRB_WBUF_WORD_BYTES;
    HRB_CUDA(ctx, cudaMemcpyAsync(ctx->d_wbuf + off, wbuf + off,
                                  size_t{w.count[i]} * HRB_WBUF_WORD_BYTES,
                                  cudaMemcpyHostToDevice, s));
  }
  for (int i = 0; i < c.parts; ++i) {
    const size_t off = size_t{c.first[i]} * 32u;
    HRB_CUDA(ctx, cudaMemcpyAsync(ctx->d_fbuf + off, fbuf + off, size_t{c.count[i]} * 128u,
                                  cudaMemcpyHostToDevice, s));
  }
  st = hrb_gemm_exec_device(ctx, cmd, ctx->d_abuf, ctx->d_wbuf, ctx->d_fbuf, s);
  if (st != HRB_OK) return st;
  for (int i = 0; i < c.parts; ++i) {
    const size_t off = size_t{c.first[i]} * 32u;
    HRB_CUDA(ctx, cudaMemcpyAsync(fbuf + off, ctx->d_fbuf + off, size_t{c.count[i]} * 128u,
                                  cudaMemcpyDeviceToHost, s));
  }
  HRB_CUDA(ctx, cudaStreamSynchronize(s));
  return HRB_OK;
}

// ---------------------------------------------------------------------------
// Dense

hrb_status hrb_quantize_mxint8(hrb_ctx* ctx, const float* x, uint32_t rows, uint32_t cols,
                               uint32_t ldx, uint32_t quant, int8_t* q, uint8_t* scale,
                               void* stream) {
  if (ctx == nullptr) return HRB_EINVAL;
  if (x == nullptr || q == nullptr || scale == nullptr) return fail(ctx, HRB_EINVAL, "null buffer");
  if (rows == 0 || cols == 0) return fail(ctx, HRB_EINVAL, "empty matrix %u x %u", rows, cols);
  if (ldx < cols) return fail(ctx, HRB_EINVAL, "ldx %u < cols %u", ldx, cols);
  if (quant > HRB_QUANT_VEC) return fail(ctx, HRB_EINVAL, "unknown quantizer %u", quant);
  if (!aligned(x, 4) || !aligned(q, 4)) return fail(ctx, HRB_EINVAL, "misaligned buffer");
  HRB_CUDA(ctx, cudaSetDevice(ctx->device));
  const hrb::QuantJob j = make_quant_job(x, rows, cols, ldx, quant, q, scale);
  hrb::launch_quantize(nullptr, 1, &j, j.units, ctx->d_error, ctx->sm_count, pick(ctx, stream));
  ctx->launches += 1;
  HRB_CUDA(ctx, cudaGetLastError());
  return HRB_OK;
}

hrb_status hrb_gemm_dense(hrb_ctx* ctx, const hrb_gemm_desc* d, void* stream) {
  if (ctx == nullptr) return HRB_EINVAL;
  uint32_t pieces[hrb::kMaxPieces];
  uint32_t npieces = 0;
  hrb_status st = check_desc(ctx, d, pieces, &npieces);
  if (st != HRB_OK) return st;
  HRB_CUDA(ctx, cudaSetDevice(ctx->device));
  cudaStream_t s = pick(ctx, stream);
  if (use_tc(d)) {
    st = grow(ctx, &ctx->scratch, &ctx->scratch_bytes, tc_scratch_bytes(d));
    if (st != HRB_OK) return st;
    hrb::QuantJob qj;
    hrb::TcJob tj;
    tc_jobs(d, tc_fmt(d), static_cast<uint8_t*>(ctx->scratch), &qj, &tj);
    // Rows of the last activation tile past M stay zero.
    HRB_CUDA(ctx, cudaMemsetAsync(ctx->scratch, 0, align_up(tc_act_bytes(d, tj.wfmt), 1024), s));
    tc_translate(d, tj, s);
    hrb::launch_quantize_planes(nullptr, 1, &qj, qj.units, ctx->d_error, ctx->sm_count, s);
    tj.tile_begin = 0;
    const int n = hrb::launch_mxf4(nullptr, &tj, qj.tile_rows, tj.wfmt, tj.m_tiles * tj.n_tiles,
                                   ctx->sm_count, ctx->d_error, s);
    if (n < 0) return fail(ctx, HRB_ECUDA, "tensor-core launch failed");
    ctx->launches += 2u + static_cast<uint64_t>(n);
    HRB_CUDA(ctx, cudaGetLastError());
    return HRB_OK;
  }
  const int8_t* aq = d->aq;
  const uint8_t* ascale = d->ascale;
  if (d->a != nullptr) {
    st = grow(ctx, &ctx->scratch, &ctx->scratch_bytes, act_scratch_bytes(d->M, d->K));
    if (st != HRB_OK) return st;
    const uint32_t kb = blocks_of(d->K);
    auto* q = static_cast<int8_t*>(ctx->scratch);
    auto* sc = reinterpret_cast<uint8_t*>(ctx->scratch) + align_up(size_t{d->M} * kb * 32u, 256);
    const hrb::QuantJob j = make_quant_job(d->a, d->M, d->K, d->lda, d->quant, q, sc);
    hrb::launch_quantize(nullptr, 1, &j, j.units, ctx->d_error, ctx->sm_count, s);
    ctx->launches += 1;
    aq = q;
    ascale = sc;
  }
  st = run_dense(ctx, make_dense_job(d, aq, ascale, pieces, npieces), s);
  if (st != HRB_OK || d->cq == nullptr) return st;
  const hrb::QuantJob pq = post_quant_job(d);
  hrb::launch_quantize(nullptr, 1, &pq, pq.units, ctx->d_error, ctx->sm_count, s);
  ctx->launches += 1;
  HRB_CUDA(ctx, cudaGetLastError());
  return HRB_OK;
}

namespace {

// The row-format source of hrb_gemm_rows, checked against M and K.
hrb_status make_rows_src(hrb_ctx* ctx, const hrb_gemm_desc* d, const hrb_rows* r,
                         hrb::RowsSrc* out) {
  if (r->window == nullptr || !aligned(r->window, 16)) {
    return fail(ctx, HRB_EINVAL, "the DDR window is null or not 16-byte aligned");
  }
  if (r->ddr_base % 16u != 0) return fail(ctx, HRB_EINVAL, "ddr_base is not a multiple of 16");
  if (r->tok == 0 || r->tok > 32) return fail(ctx, HRB_EINVAL, "row format with tok = %u", r->tok);
  if (r->plane_stride % 16u != 0) {
    return fail(ctx, HRB_EINVAL, "plane_stride is not a multiple of 16");
  }
  const uint32_t kb = blocks_of(d->K);
  if (r->planes == 0 || (kb + r->tok - 1) / r->tok != r->planes) {
    return fail(ctx, HRB_EINVAL, "%u planes of %u blocks do not hold K = %u", r->planes, r->tok,
                d->K);
  }
  hrb::RowsSrc& s = *out;
  s = hrb::RowsSrc{};
  s.window = static_cast<const uint8_t*>(r->window);
  s.ddr_base = r->ddr_base;
  s.window_bytes = r->window_bytes;
  s.index = r->index;
  s.plane_stride = r->plane_stride;
  s.row_stride = r->row_stride;
  s.tok = r->tok;
  s.planes = r->planes;
  s.row_tokens = r->row_tokens;
  s.unit_bytes = r->tok * 32u + (r->tok > 16 ? 32u : 16u);
  s.kb = kb;
  s.kp = kb * 32u;
  if (r->index != nullptr) {
    if (!aligned(r->index, 4)) return fail(ctx, HRB_EINVAL, "the index list is not 4-byte aligned");
    return HRB_OK;
  }
  if (r->row_tokens == 0 || r->row_tokens % 4u != 0) {
    return fail(ctx, HRB_EINVAL, "row format with %u tokens a row, not a multiple of 4",
                r->row_tokens);
  }
  if (r->row_stride % 16u != 0) return fail(ctx, HRB_EINVAL, "row_stride is not a multiple of 16");
  const uint64_t first = uint64_t{r->ddr_addr} * 16u;
  if (first < r->ddr_base) return fail(ctx, HRB_EINVAL, "ddr_addr lies before the window");
  s.first = first - r->ddr_base;
  // The farthest unit: the last row's last token, or the full row before it.
  const uint64_t rt = r->row_tokens, q = (d->M - 1u) / rt;
  uint64_t far = q * r->row_stride + ((d->M - 1u) % rt) * s.unit_bytes;
  if (q > 0) far = std::max<uint64_t>(far, (q - 1) * r->row_stride + (rt - 1) * s.unit_bytes);
  far += s.first + uint64_t{r->planes - 1u} * r->plane_stride + s.unit_bytes;
  if (far > r->window_bytes) {
    return fail(ctx, HRB_EINVAL, "row-format units reach byte %llu of a %llu-byte window",
                static_cast<unsigned long long>(far),
                static_cast<unsigned long long>(r->window_bytes));
  }
  return HRB_OK;
}

}  // namespace

hrb_status hrb_gemm_rows(hrb_ctx* ctx, const hrb_gemm_desc* desc, const hrb_rows* rows,
                         void* stream) {
  if (ctx == nullptr) return HRB_EINVAL;
  if (desc == nullptr || rows == nullptr) return fail(ctx, HRB_EINVAL, "null descriptor");
  if (desc->a != nullptr || desc->aq != nullptr || desc->ascale != nullptr) {
    return fail(ctx, HRB_EINVAL, "row-format activations replace a, aq and ascale");
  }
  if (desc->c == nullptr) return fail(ctx, HRB_EINVAL, "row-format activations need the output c");
  if (desc->M == 0 || desc->K == 0) return fail(ctx, HRB_EINVAL, "empty GEMM");
  hrb::RowsSrc src;
  hrb_status st = make_rows_src(ctx, desc, rows, &src);
  if (st != HRB_OK) return st;
  // The descriptor's own checks, with the window standing in for the codes.
  hrb_gemm_desc d = *desc;
  d.aq = static_cast<const int8_t*>(rows->window);
  d.ascale = static_cast<const uint8_t*>(rows->window);
  uint32_t plane_pieces[hrb::kMaxPieces];
  if (d.pieces == nullptr || d.npieces == 0) {
    if (rows->planes > hrb::kMaxPieces) {
      return fail(ctx, HRB_EINVAL, "%u planes (at most %u K pieces)", rows->planes,
                  hrb::kMaxPieces);
    }
    for (uint32_t p = 0; p < rows->planes; ++p) {
      plane_pieces[p] = std::min(rows->tok, src.kb - p * rows->tok);
    }
    d.pieces = plane_pieces;
    d.npieces = rows->planes;
  }
  uint32_t pieces[hrb::kMaxPieces];
  uint32_t npieces = 0;
  st = check_desc(ctx, &d, pieces, &npieces);
  if (st != HRB_OK) return st;
  HRB_CUDA(ctx, cudaSetDevice(ctx->device));
  cudaStream_t s = pick(ctx, stream);
  if (d.mode == HRB_MODE_FAST) {
    const uint32_t pf = tc_fmt(&d);
    st = grow(ctx, &ctx->scratch, &ctx->scratch_bytes, tc_scratch_bytes(&d, pf));
    if (st != HRB_OK) return st;
    hrb::QuantJob qj;
    hrb::TcJob tj;
    tc_jobs(&d, pf, static_cast<uint8_t*>(ctx->scratch), &qj, &tj);
    HRB_CUDA(ctx, cudaMemsetAsync(ctx->scratch, 0, align_up(tc_act_bytes(&d, pf), 1024), s));
    tc_translate(&d, tj, s);
    hrb::launch_rows_planes(src, qj, ctx->d_error, ctx->sm_count, s);
    tj.tile_begin = 0;
    const int n = hrb::launch_mxf4(nullptr, &tj, qj.tile_rows, tj.wfmt, tj.m_tiles * tj.n_tiles,
                                   ctx->sm_count, ctx->d_error, s);
    if (n < 0) return fail(ctx, HRB_ECUDA, "tensor-core launch failed");
    ctx->launches += 2u + static_cast<uint64_t>(n);
    HRB_CUDA(ctx, cudaGetLastError());
    return HRB_OK;
  }
  st = grow(ctx, &ctx->scratch, &ctx->scratch_bytes, act_scratch_bytes(d.M, d.K));
  if (st != HRB_OK) return st;
  auto* q = static_cast<int8_t*>(ctx->scratch);
  auto* sc = reinterpret_cast<uint8_t*>(ctx->scratch) + align_up(size_t{d.M} * src.kb * 32u, 256);
  hrb::launch_rows_dense(src, d.M, q, sc, ctx->d_error, ctx->sm_count, s);
  ctx->launches += 1;
  st = run_dense(ctx, make_dense_job(&d, q, sc, pieces, npieces), s);
  if (st != HRB_OK || d.cq == nullptr) return st;
  const hrb::QuantJob pq = post_quant_job(&d);
  hrb::launch_quantize(nullptr, 1, &pq, pq.units, ctx->d_error, ctx->sm_count, s);
  ctx->launches += 1;
  HRB_CUDA(ctx, cudaGetLastError());
  return HRB_OK;
}

hrb_status hrb_gemm_dense_host(hrb_ctx* ctx, const hrb_gemm_desc* d) {
  if (ctx == nullptr) return HRB_EINVAL;
  uint32_t pieces[hrb::kMaxPieces];
  uint32_t npieces = 0;
  hrb_status st = check_desc(ctx, d, pieces, &npieces);
  if (st != HRB_OK) return st;
  HRB_CUDA(ctx, cudaSetDevice(ctx->device));
  const uint32_t kb = blocks_of(d->K);
  const size_t kp = size_t{kb} * 32u;
  // Staging layout: activations (FP32 packed, or MXINT8), weights, scales,
  // bias, output; every part 256-byte aligned.
  const size_t a_bytes = d->a ? size_t{d->M} * d->K * 4u : size_t{d->M} * kp;
  const size_t as_bytes = d->a ? 0 : size_t{d->M} * kb;
  const size_t w_bytes = size_t{d->N} * weight_row_bytes(d->wfmt, kb);
  const size_t ws_bytes = size_t{d->N} * kb;
  const size_t b_bytes = d->bias ? size_t{d->N} * 4u : 0;
  const size_t cs_bytes = d->wcol_scale ? size_t{d->N} * 4u : 0;
  const size_t c_bytes = d->c ? size_t{d->M} * d->N * 4u : 0;
  const uint32_t kbq = d->ldcq != 0 ? d->ldcq / 32u : blocks_of(d->N);  // row blocks of the copy
  const size_t q_bytes = d->cq ? size_t{d->M} * kbq * 32u : 0;
  const size_t qs_bytes = d->cq ? size_t{d->M} * kbq : 0;
  size_t off = 0;
  const size_t o_a = off; off = align_up(off + a_bytes, 256);
  const size_t o_as = off; off = align_up(off + as_bytes, 256);
  const size_t o_w = off; off = align_up(off + w_bytes, 256);
  const size_t o_ws = off; off = align_up(off + ws_bytes, 256);
  const size_t o_b = off; off = align_up(off + b_bytes, 256);
  const size_t o_cs = off; off = align_up(off + cs_bytes, 256);
  const size_t o_c = off; off = align_up(off + c_bytes, 256);
  const size_t o_q = off; off = align_up(off + q_bytes, 256);
  const size_t o_qs = off; off = align_up(off + qs_bytes, 256);
  st = grow(ctx, &ctx->staging, &ctx->staging_bytes, off);
  if (st != HRB_OK) return st;
  auto* base = static_cast<uint8_t*>(ctx->staging);
  cudaStream_t s = ctx->stream;
  hrb_gemm_desc dd = *d;
  if (d->a) {
    HRB_CUDA(ctx, cudaMemcpy2DAsync(base + o_a, size_t{d->K} * 4u, d->a, size_t{d->lda} * 4u,
                                    size_t{d->K} * 4u, d->M, cudaMemcpyHostToDevice, s));
    dd.a = reinterpret_cast<const float*>(base + o_a);
    dd.lda = d->K;
  } else {
    HRB_CUDA(ctx, cudaMemcpyAsync(base + o_a, d->aq, a_bytes, cudaMemcpyHostToDevice, s));
    HRB_CUDA(ctx, cudaMemcpyAsync(base + o_as, d->ascale, as_bytes, cudaMemcpyHostToDevice, s));
    dd.aq = reinterpret_cast<const int8_t*>(base + o_a);
    dd.ascale = base + o_as;
  }
  HRB_CUDA(ctx, cudaMemcpyAsync(base + o_w, d->w, w_bytes, cudaMemcpyHostToDevice, s));
  HRB_CUDA(ctx, cudaMemcpyAsync(base + o_ws, d->wscale, ws_bytes, cudaMemcpyHostToDevice, s));
  dd.w = base + o_w;
  dd.wscale = base + o_ws;
  if (d->bias) {
    HRB_CUDA(ctx, cudaMemcpyAsync(base + o_b, d->bias, b_bytes, cudaMemcpyHostToDevice, s));
    dd.bias = reinterpret_cast<const float*>(base + o_b);
  }
  if (d->wcol_scale) {
    HRB_CUDA(ctx, cudaMemcpyAsync(base + o_cs, d->wcol_scale, cs_bytes, cudaMemcpyHostToDevice, s));
    dd.wcol_scale = reinterpret_cast<const float*>(base + o_cs);
  }
  dd.c = d->c ? reinterpret_cast<float*>(base + o_c) : nullptr;
  dd.ldc = d->N;
  if (d->accumulate) {
    HRB_CUDA(ctx, cudaMemcpy2DAsync(dd.c, size_t{d->N} * 4u, d->c, size_t{d->ldc} * 4u,
                                    size_t{d->N} * 4u, d->M, cudaMemcpyHostToDevice, s));
  }
  if (d->cq) {
    dd.cq = reinterpret_cast<int8_t*>(base + o_q);
    dd.cscale = base + o_qs;
  }
  st = hrb_gemm_dense(ctx, &dd, s);
  if (st != HRB_OK) return st;
  if (d->c) {
    HRB_CUDA(ctx, cudaMemcpy2DAsync(d->c, size_t{d->ldc} * 4u, dd.c, size_t{d->N} * 4u,
                                    size_t{d->N} * 4u, d->M, cudaMemcpyDeviceToHost, s));
  }
  if (d->cq) {
    if (d->ldcq == 0) {
      HRB_CUDA(ctx, cudaMemcpyAsync(d->cq, dd.cq, q_bytes, cudaMemcpyDeviceToHost, s));
      HRB_CUDA(ctx, cudaMemcpyAsync(d->cscale, dd.cscale, qs_bytes, cudaMemcpyDeviceToHost, s));
    } else {
      // Only this GEMM's columns of each row: the rest of the wider rows is
      // the caller's.
      const size_t kpn = size_t{blocks_of(d->N)} * 32u;
      HRB_CUDA(ctx, cudaMemcpy2DAsync(d->cq, d->ldcq, dd.cq, d->ldcq, kpn, d->M,
                                      cudaMemcpyDeviceToHost, s));
      HRB_CUDA(ctx, cudaMemcpy2DAsync(d->cscale, d->ldcq / 32u, dd.cscale, d->ldcq / 32u,
                                      kpn / 32u, d->M, cudaMemcpyDeviceToHost, s));
    }
  }
  return hrb_sync(ctx);
}

// ---------------------------------------------------------------------------
// Plans

hrb_status hrb_plan_create(hrb_ctx* ctx, const hrb_gemm_desc* descs, uint32_t count,
                           hrb_plan** out) {
  if (ctx == nullptr || out == nullptr) return HRB_EINVAL;
  *out = nullptr;
  if (descs == nullptr || count == 0) return fail(ctx, HRB_EINVAL, "empty plan");
  std::vector<std::vector<uint32_t>> pieces(count, std::vector<uint32_t>(hrb::kMaxPieces));
  std::vector<uint32_t> npieces(count);
  size_t scratch = 0;
  for (uint32_t i = 0; i < count; ++i) {
    const hrb_status st = check_desc(ctx, &descs[i], pieces[i].data(), &npieces[i]);
    if (st != HRB_OK) return st;
    if (use_tc(&descs[i])) {
      scratch += tc_scratch_bytes(&descs[i]);
    } else {
      if (descs[i].a != nullptr) scratch += align_up(act_scratch_bytes(descs[i].M, descs[i].K), 1024);
      if (exact_tc(descs[i].wfmt)) {
        scratch += align_up(hrb::x_weight_bytes(descs[i].wfmt, descs[i].N, blocks_of(descs[i].K)),
                            1024);
      }
    }
  }
  HRB_CUDA(ctx, cudaSetDevice(ctx->device));
  auto plan = new (std::nothrow) hrb_plan();
  if (plan == nullptr) return HRB_ENOMEM;
  plan->ctx = ctx;
  for (uint32_t i = 0; i < count; ++i) {
    const hrb_gemm_desc& d = descs[i];
    const size_t kb = blocks_of(d.K);
    hrb_plan::Io io{};
    if (d.a != nullptr) {
      io.a = const_cast<float*>(d.a);
      io.a_bytes = (static_cast<size_t>(d.M - 1) * d.lda + d.K) * sizeof(float);
    } else {
      io.a = const_cast<int8_t*>(d.aq);
      io.a_bytes = static_cast<size_t>(d.M) * kb * 32u;
      io.ascale = const_cast<uint8_t*>(d.ascale);
      io.ascale_bytes = static_cast<size_t>(d.M) * kb;
    }
    io.c = d.c;
    io.c_bytes = (static_cast<size_t>(d.M - 1) * d.ldc + d.N) * sizeof(float);
    plan->io.push_back(io);
  }
  if (scratch > 0) {
    cudaError_t err = cudaMalloc(&plan->d_scratch, scratch);
    // Zero once: padding rows of the last activation tile are never written.
    if (err == cudaSuccess) err = cudaMemset(plan->d_scratch, 0, scratch);
    if (err != cudaSuccess) {
      hrb_plan_destroy(plan);
      return cuda_fail(ctx, err, "plan scratch");
    }
  }
  // Encoder jobs, exact-kernel jobs per format, tensor-core jobs per
  // (tokens per tile, format).  Tensor-core weights are translated now, once.
  std::vector<hrb::QuantJob> quant, planes, post;
  std::vector<std::vector<hrb::DenseJob>> exact(3);
  uint32_t exact_tiles[3] = {0, 0, 0};
  // Exact GEMMs on the tensor cores (exact_tc), per format, weights translated now.
  // Groups: format (MXFP4, W8) x token tile (64, 16): index 2 wfmt + (tok == 16).
  std::vector<std::vector<hrb::XJob>> xexact(4);
  uint32_t xexact_tiles[4] = {0, 0, 0, 0};
  struct TcKey { uint32_t nt, wfmt, kind; bool pairs; };
  std::vector<TcKey> tc_keys;
  std::vector<std::vector<hrb::TcJob>> tc_groups;
  std::vector<uint32_t> tc_tiles;
  auto* sbase = static_cast<uint8_t*>(plan->d_scratch);
  size_t soff = 0;
  for (uint32_t i = 0; i < count; ++i) {
    const hrb_gemm_desc& d = descs[i];
    if (use_tc(&d)) {
      hrb::QuantJob qj;
      hrb::TcJob tj;
      tc_jobs(&d, tc_fmt(&d), sbase + soff, &qj, &tj);
      soff += tc_scratch_bytes(&d);
      tc_translate(&d, tj, ctx->stream);
      qj.unit_begin = plan->plane_units;
      plan->plane_units += qj.units;
      qj.group_begin = plan->plane_groups;
      plan->plane_groups += static_cast<uint64_t>(qj.rows) * ((qj.k_steps + 3u) / 4u);
      planes.push_back(qj);
      size_t g = 0;
      const uint32_t kind = 2u;
      const bool pairs = hrb::mx_pairs(tj.wfmt, tj.n_tiles);
      while (g < tc_keys.size() && !(tc_keys[g].nt == qj.tile_rows && tc_keys[g].wfmt == tj.wfmt &&
                                     tc_keys[g].kind == kind && tc_keys[g].pairs == pairs)) {
        ++g;
      }
      if (g == tc_keys.size()) {
        tc_keys.push_back({qj.tile_rows, tj.wfmt, kind, pairs});
        tc_groups.emplace_back();
        tc_tiles.push_back(0);
      }
      const uint32_t job_tiles = hrb::mx_job_tiles(tj, pairs);
      tj.tile_begin = tc_tiles[g];
      tc_tiles[g] += job_tiles;
      tc_groups[g].push_back(tj);
      plan->io[i].tile_begin = tj.tile_begin;
      plan->io[i].tiles = job_tiles;
      continue;
    }
    const int8_t* aq = d.aq;
    const uint8_t* as = d.ascale;
    if (d.a != nullptr) {
      const uint32_t kb = blocks_of(d.K);
      auto* q = reinterpret_cast<int8_t*>(sbase + soff);
      auto* sc = reinterpret_cast<uint8_t*>(q) + align_up(size_t{d.M} * kb * 32u, 256);
      soff += align_up(act_scratch_bytes(d.M, d.K), 1024);
      hrb::QuantJob j = make_quant_job(d.a, d.M, d.K, d.lda, d.quant, q, sc);
      j.unit_begin = plan->quant_units;
      plan->quant_units += j.units;
      quant.push_back(j);
      aq = q;
      as = sc;
    }
    if (d.cq != nullptr) {
      hrb::QuantJob pq = post_quant_job(&d);
      pq.unit_begin = plan->post_units;
      plan->post_units += pq.units;
      post.push_back(pq);
    }
    hrb::DenseJob j = make_dense_job(&d, aq, as, pieces[i].data(), npieces[i]);
    if (exact_tc(j.wfmt)) {
      uint8_t* xw = sbase + soff;
      soff += align_up(hrb::x_weight_bytes(j.wfmt, j.N, j.kb), 1024);
      hrb::launch_x_translate(j.wfmt, j.w, j.wscale, j.N, j.kb, xw, ctx->stream);
      const uint32_t tok = hrb::x_tok(j.M), xg = 2u * j.wfmt + (tok == 16u ? 1u : 0u);
      xexact[xg].push_back(x_job(j, xw, xexact_tiles[xg]));
      xexact_tiles[xg] += hrb::x_tiles(j.M, j.N, tok);
      plan->io[i].tile_begin = xexact[xg].back().tile_begin;
      plan->io[i].tiles = hrb::x_tiles(j.M, j.N, tok);
      continue;
    }
    uint32_t tiles_n = 0;
    const uint32_t tiles = hrb::dense_exact_tiles(j.M, j.N, tiles_n);
    j.tiles_n = tiles_n;
    j.tile_begin = exact_tiles[j.wfmt];
    exact_tiles[j.wfmt] += tiles;
    exact[j.wfmt].push_back(j);
  }
  size_t bytes = (quant.size() + planes.size() + post.size()) * sizeof(hrb::QuantJob);
  for (auto& g : exact) bytes += g.size() * sizeof(hrb::DenseJob);
  for (auto& g : xexact) bytes += g.size() * sizeof(hrb::XJob);
  for (auto& g : tc_groups) bytes += g.size() * sizeof(hrb::TcJob);
  // kind::mxf4 groups also get their output tiles located on the host.
  std::vector<std::vector<hrb::MxTile>> mx_tiles(tc_groups.size());
  for (size_t g = 0; g < tc_groups.size(); ++g) {
    if (tc_keys[g].kind != 2) continue;
    mx_tiles[g].resize(tc_tiles[g]);
    for (const hrb::TcJob& tj : tc_groups[g]) {
      hrb::mx_fill_tiles(tj, tc_keys[g].nt, mx_tiles[g].data() + tj.tile_begin, tc_keys[g].pairs);
    }
    bytes += 16 + mx_tiles[g].size() * sizeof(hrb::MxTile);  // 16: alignment slack
  }
  if (bytes > 0) {
    const cudaError_t err = cudaMalloc(&plan->d_jobs, bytes);
    if (err != cudaSuccess) {
      hrb_plan_destroy(plan);
      return cuda_fail(ctx, err, "plan jobs");
    }
  }
  auto* dst = static_cast<uint8_t*>(plan->d_jobs);
  if (!quant.empty()) {
    HRB_CUDA(ctx, cudaMemcpy(dst, quant.data(), quant.size() * sizeof(hrb::QuantJob),
                             cudaMemcpyHostToDevice));
    plan->d_quant = reinterpret_cast<const hrb::QuantJob*>(dst);
    plan->nquant = static_cast<uint32_t>(quant.size());
    dst += quant.size() * sizeof(hrb::QuantJob);
  }
  if (!planes.empty()) {
    HRB_CUDA(ctx, cudaMemcpy(dst, planes.data(), planes.size() * sizeof(hrb::QuantJob),
                             cudaMemcpyHostToDevice));
    plan->d_planes = reinterpret_cast<const hrb::QuantJob*>(dst);
    plan->nplanes = static_cast<uint32_t>(planes.size());
    plan->d_planes_host = planes;
    dst += planes.size() * sizeof(hrb::QuantJob);
  }
  if (!post.empty()) {
    HRB_CUDA(ctx, cudaMemcpy(dst, post.data(), post.size() * sizeof(hrb::QuantJob),
                             cudaMemcpyHostToDevice));
    plan->d_post = reinterpret_cast<const hrb::QuantJob*>(dst);
    plan->npost = static_cast<uint32_t>(post.size());
    dst += post.size() * sizeof(hrb::QuantJob);
  }
  for (uint32_t f = 0; f < 3; ++f) {
    auto& g = exact[f];
    if (g.empty()) continue;
    HRB_CUDA(ctx, cudaMemcpy(dst, g.data(), g.size() * sizeof(hrb::DenseJob),
                             cudaMemcpyHostToDevice));
    plan->groups.push_back({f, 0u, 0, static_cast<uint32_t>(g.size()), exact_tiles[f], dst,
                            nullptr});
    dst += g.size() * sizeof(hrb::DenseJob);
  }
  for (uint32_t xg = 0; xg < 4; ++xg) {
    auto& g = xexact[xg];
    if (g.empty()) continue;
    HRB_CUDA(ctx, cudaMemcpy(dst, g.data(), g.size() * sizeof(hrb::XJob), cudaMemcpyHostToDevice));
    // nt: the group's token tile.
    plan->groups.push_back({xg / 2u, 1u, xg % 2u != 0 ? 16u : 64u,
                            static_cast<uint32_t>(g.size()), xexact_tiles[xg], dst, nullptr});
    dst += g.size() * sizeof(hrb::XJob);
  }
  for (size_t g = 0; g < tc_groups.size(); ++g) {
    HRB_CUDA(ctx, cudaMemcpy(dst, tc_groups[g].data(), tc_groups[g].size() * sizeof(hrb::TcJob),
                             cudaMemcpyHostToDevice));
    plan->groups.push_back({tc_keys[g].wfmt, tc_keys[g].kind, tc_keys[g].nt,
                            static_cast<uint32_t>(tc_groups[g].size()), tc_tiles[g], dst,
                            nullptr, tc_keys[g].pairs});
    dst += tc_groups[g].size() * sizeof(hrb::TcJob);
    if (!mx_tiles[g].empty()) {
      auto* base = static_cast<uint8_t*>(plan->d_jobs);
      dst = base + align_up(static_cast<size_t>(dst - base), 16);
      HRB_CUDA(ctx, cudaMemcpy(dst, mx_tiles[g].data(), mx_tiles[g].size() * sizeof(hrb::MxTile),
                               cudaMemcpyHostToDevice));
      plan->groups.back().d_tiles = reinterpret_cast<const hrb::MxTile*>(dst);
      dst += mx_tiles[g].size() * sizeof(hrb::MxTile);
    }
  }
  HRB_CUDA(ctx, cudaGetLastError());
  HRB_CUDA(ctx, cudaStreamSynchronize(ctx->stream));   // weight translation done
  *out = plan;
  return HRB_OK;
}

}  // extern "C"

namespace {

// Launches every kernel of a plan on s; when `events` is given, records
// events[i] before launch i and events[n] after the last.
// Launch steps of a plan: the encoders (FP32 -> MXINT8 codes, then
// FP32 -> digit planes), then one GEMM launch per group.
uint32_t plan_steps(const hrb_plan* plan) {
  return (plan->nquant > 0 ? 1u : 0u) + (plan->nplanes > 0 ? 1u : 0u) +
         static_cast<uint32_t>(plan->groups.size()) + (plan->npost > 0 ? 1u : 0u);
}

// Launches step `only` of a plan on s, or every step in order when `only`
// is negative; adds the number of kernels launched to *launched.
hrb_status plan_launch(hrb_plan* plan, cudaStream_t s, int64_t only, uint32_t* launched) {
  hrb_ctx* ctx = plan->ctx;
  uint32_t n = 0;
  int64_t step = 0;
  auto take = [&]() { return only < 0 || only == step++; };
  if (plan->nquant > 0 && take()) {
    hrb::launch_quantize(plan->d_quant, plan->nquant, nullptr, plan->quant_units, ctx->d_error,
                         ctx->sm_count, s);
    ++n;
  }
  if (plan->nplanes > 0 && take()) {
    hrb::launch_quantize_planes(plan->d_planes, plan->nplanes, nullptr, plan->plane_units,
                                ctx->d_error, ctx->sm_count, s, plan->d_planes_host.data());
    ++n;
  }
  for (auto& g : plan->groups) {
    if (!take()) continue;
    if (g.kind == 0) {
      n += static_cast<uint32_t>(hrb::launch_dense_exact(
          static_cast<const hrb::DenseJob*>(g.d_jobs), g.njobs, nullptr, g.tiles, g.wfmt, s));
    } else if (g.kind == 1) {
      const int k = hrb::launch_x_exact(static_cast<const hrb::XJob*>(g.d_jobs), g.njobs, nullptr,
                                        g.tiles, g.nt, ctx->sm_count, ctx->d_error, s);
      if (k < 0) return fail(ctx, HRB_ECUDA, "k_exact_tc launch failed");
      n += static_cast<uint32_t>(k);
    } else {
      const int k = hrb::launch_mxf4(g.d_tiles, nullptr, g.nt, g.wfmt, g.tiles, ctx->sm_count,
                                     ctx->d_error, s, &plan->peers, true, g.pairs ? 1 : 0);
      if (k < 0) return fail(ctx, HRB_ECUDA, "tensor-core launch failed");
      n += static_cast<uint32_t>(k);
    }
  }
  if (plan->npost > 0 && take()) {
    hrb::launch_quantize(plan->d_post, plan->npost, nullptr, plan->post_units, ctx->d_error,
                         ctx->sm_count, s);
    ++n;
  }
  ctx->launches += n;
  *launched += n;
  HRB_CUDA(ctx, cudaGetLastError());
  return HRB_OK;
}

}  // namespace

extern "C" {

hrb_status hrb_plan_run(hrb_plan* plan, void* stream, uint32_t* launches) {
  if (plan == nullptr) return HRB_EINVAL;
  HRB_CUDA(plan->ctx, cudaSetDevice(plan->ctx->device));
  uint32_t n = 0;
  const hrb_status st = plan_launch(plan, pick(plan->ctx, stream), -1, &n);
  if (launches != nullptr) *launches = n;
  return st;
}

hrb_status hrb_plan_run_host(hrb_plan* plan, void* stream, const void* const* a_host,
                             const void* const* ascale_host, void* const* c_host) {
  if (plan == nullptr) return HRB_EINVAL;
  hrb_ctx* ctx = plan->ctx;
  HRB_CUDA(ctx, cudaSetDevice(ctx->device));
  cudaStream_t s = pick(ctx, stream);
  const uint32_t n = static_cast<uint32_t>(plan->io.size());
  // Copies of GEMMs [g0, g1) in one direction, adjacent ranges merged.
  auto copy_in = [&](uint32_t g0, uint32_t g1, cudaStream_t cs) -> hrb_status {
    for (int part = 0; part < 2; ++part) {
      const void* const* host = part == 0 ? a_host : ascale_host;
      if (host == nullptr) continue;
      char* dst = nullptr;
      const char* src = nullptr;
      size_t len = 0;
      for (uint32_t i = g0; i <= g1; ++i) {
        char* d = nullptr;
        const char* h = nullptr;
        size_t b = 0;
        if (i < g1 && host[i] != nullptr) {
          d = static_cast<char*>(part == 0 ? plan->io[i].a : plan->io[i].ascale);
          h = static_cast<const char*>(host[i]);
          b = part == 0 ? plan->io[i].a_bytes : plan->io[i].ascale_bytes;
          if (d == nullptr) b = 0;
        }
        if (len > 0 && b > 0 && d == dst + len && h == src + len) {
          len += b;
          continue;
        }
        if (len > 0) HRB_CUDA(ctx, cudaMemcpyAsync(dst, src, len, cudaMemcpyHostToDevice, cs));
        dst = d;
        src = h;
        len = b;
      }
    }
    return HRB_OK;
  };
  auto copy_out = [&](uint32_t g0, uint32_t g1, cudaStream_t cs) -> hrb_status {
    if (c_host == nullptr) return HRB_OK;
    char* dst = nullptr;
    const char* src = nullptr;
    size_t len = 0;
    for (uint32_t i = g0; i <= g1; ++i) {
      char* h = nullptr;
      const char* d = nullptr;
      size_t b = 0;
      if (i < g1 && c_host[i] != nullptr) {
        h = static_cast<char*>(c_host[i]);
        d = static_cast<const char*>(plan->io[i].c);
        b = plan->io[i].c_bytes;
      }
      if (len > 0 && b > 0 && h == dst + len && d == src + len) {
        len += b;
        continue;
      }
      if (len > 0) HRB_CUDA(ctx, cudaMemcpyAsync(dst, src, len, cudaMemcpyDeviceToHost, cs));
      dst = h;
      src = d;
      len = b;
    }
    return HRB_OK;
  };
  const bool pipelined = plan->nquant == 0 && plan->nplanes == n && plan->groups.size() == 1 &&
                         plan->groups[0].kind == 2 && plan->npost == 0 && n >= 8;
  if (!pipelined) {
    hrb_status st = copy_in(0, n, s);
    if (st != HRB_OK) return st;
    uint32_t launched = 0;
    st = plan_launch(plan, s, -1, &launched);
    if (st != HRB_OK) return st;
    return copy_out(0, n, s);
  }
  // Chunks of GEMMs: copy-in of chunk c+1 and copy-out of chunk c-1 overlap
  // the encoder and GEMM of chunk c.
  constexpr uint32_t kChunks = 8;
  const uint32_t chunks = std::min(kChunks, n / 2);
  if (plan->s_in == nullptr) {
    HRB_CUDA(ctx, cudaStreamCreateWithFlags(&plan->s_in, cudaStreamNonBlocking));
    HRB_CUDA(ctx, cudaStreamCreateWithFlags(&plan->s_out, cudaStreamNonBlocking));
    plan->events.resize(3 * kChunks + 1);
    for (auto& e : plan->events) {
      HRB_CUDA(ctx, cudaEventCreateWithFlags(&e, cudaEventDisableTiming));
    }
  }
  cudaEvent_t* ev = plan->events.data();
  cudaEvent_t entry = ev[3 * kChunks];
  // Nothing of this run starts before the work already queued on s.
  HRB_CUDA(ctx, cudaEventRecord(entry, s));
  HRB_CUDA(ctx, cudaStreamWaitEvent(plan->s_in, entry, 0));
  HRB_CUDA(ctx, cudaStreamWaitEvent(plan->s_out, entry, 0));
  const auto& g = plan->groups[0];
  for (uint32_t c = 0; c < chunks; ++c) {
    const uint32_t g0 = static_cast<uint32_t>(static_cast<uint64_t>(n) * c / chunks);
    const uint32_t g1 = static_cast<uint32_t>(static_cast<uint64_t>(n) * (c + 1) / chunks);
    hrb_status st = copy_in(g0, g1, plan->s_in);
    if (st != HRB_OK) return st;
    HRB_CUDA(ctx, cudaEventRecord(ev[c], plan->s_in));
    HRB_CUDA(ctx, cudaStreamWaitEvent(s, ev[c], 0));
    uint64_t units = 0;
    for (uint32_t i = g0; i < g1; ++i) units += plan->d_planes_host[i].units;
    hrb::launch_quantize_planes(plan->d_planes + g0, g1 - g0, nullptr, units, ctx->d_error,
                                ctx->sm_count, s, plan->d_planes_host.data() + g0);
    const uint32_t t0 = plan->io[g0].tile_begin;
    const uint32_t t1 = plan->io[g1 - 1].tile_begin + plan->io[g1 - 1].tiles;
    const int k = hrb::launch_mxf4(g.d_tiles + t0, nullptr, g.nt, g.wfmt, t1 - t0,
                                   ctx->sm_count, ctx->d_error, s, &plan->peers, true,
                                   g.pairs ? 1 : 0);
    if (k < 0) return fail(ctx, HRB_ECUDA, "tensor-core launch failed");
    ctx->launches += 1u + static_cast<uint64_t>(k);
    HRB_CUDA(ctx, cudaEventRecord(ev[kChunks + c], s));
    HRB_CUDA(ctx, cudaStreamWaitEvent(plan->s_out, ev[kChunks + c], 0));
    st = copy_out(g0, g1, plan->s_out);
    if (st != HRB_OK) return st;
  }
  // The caller's stream covers every copy: its next work follows them.
  HRB_CUDA(ctx, cudaEventRecord(ev[2 * kChunks], plan->s_out));
  HRB_CUDA(ctx, cudaStreamWaitEvent(s, ev[2 * kChunks], 0));
  HRB_CUDA(ctx, cudaGetLastError());
  return HRB_OK;
}

hrb_status hrb_plan_profile(hrb_plan* plan, void* stream, uint32_t reps, float* ms, uint32_t cap,
                            uint32_t* nkernels) {
  if (plan == nullptr || ms == nullptr || nkernels == nullptr || reps == 0 || cap == 0) {
    return HRB_EINVAL;
  }
  hrb_ctx* ctx = plan->ctx;
  HRB_CUDA(ctx, cudaSetDevice(ctx->device));
  cudaStream_t s = pick(ctx, stream);
  const uint32_t steps = std::min(plan_steps(plan), cap);
  cudaEvent_t ev[2];
  HRB_CUDA(ctx, cudaEventCreate(&ev[0]));
  HRB_CUDA(ctx, cudaEventCreate(&ev[1]));
  hrb_status st = HRB_OK;
  uint32_t n = 0;
  // A whole run first, so every step's inputs exist; then each step alone,
  // `reps` launches back to back between two events (a step launched again
  // recomputes the same outputs; GEMMs that accumulate onto C add again).
  st = plan_launch(plan, s, -1, &n);
  for (uint32_t i = 0; i < steps && st == HRB_OK; ++i) {
    st = plan_launch(plan, s, i, &n);  // warm
    if (st == HRB_OK && cudaEventRecord(ev[0], s) != cudaSuccess) st = HRB_ECUDA;
    for (uint32_t r = 0; r < reps && st == HRB_OK; ++r) st = plan_launch(plan, s, i, &n);
    if (st == HRB_OK && cudaEventRecord(ev[1], s) != cudaSuccess) st = HRB_ECUDA;
    float t = 0;
    if (st == HRB_OK && (cudaEventSynchronize(ev[1]) != cudaSuccess ||
                         cudaEventElapsedTime(&t, ev[0], ev[1]) != cudaSuccess)) {
      st = HRB_ECUDA;
    }
    ms[i] = t / static_cast<float>(reps);
  }
  cudaEventDestroy(ev[0]);
  cudaEventDestroy(ev[1]);
  if (st != HRB_OK) return st == HRB_ECUDA ? fail(ctx, st, "profiling run failed") : st;
  *nkernels = steps;
  return HRB_OK;
}

hrb_status hrb_plan_set_peers(hrb_plan* plan, const void* local_base, void* const* peer_bases,
                              uint32_t npeers) {
  if (plan == nullptr) return HRB_EINVAL;
  hrb_ctx* ctx = plan->ctx;
  if (npeers > hrb::kMaxPeers || (npeers > 0 && (local_base == nullptr || peer_bases == nullptr))) {
    return fail(ctx, HRB_EINVAL, "at most %u peers, with a local base", hrb::kMaxPeers);
  }
  if (npeers > 0 && (plan->nquant > 0 || std::any_of(plan->groups.begin(), plan->groups.end(),
                                                      [](const auto& g) { return g.kind != 2; }))) {
    return fail(ctx, HRB_ENOTSUP,
                "peer outputs need every GEMM on the MXFP4/W8 tensor-core path");
  }
  hrb::MxPeers peers{};
  peers.count = npeers;
  for (uint32_t i = 0; i < npeers; ++i) {
    if (peer_bases[i] == nullptr) return fail(ctx, HRB_EINVAL, "null peer base");
    peers.delta[i] = static_cast<const char*>(peer_bases[i]) - static_cast<const char*>(local_base);
  }
  HRB_CUDA(ctx, cudaStreamSynchronize(ctx->stream));  // no run in flight sees half a change
  plan->peers = peers;
  return HRB_OK;
}

hrb_status hrb_shared_alloc(hrb_ctx* ctx, size_t bytes, void** ptr, hrb_ipc_handle* handle) {
  if (ctx == nullptr || ptr == nullptr || handle == nullptr || bytes == 0) return HRB_EINVAL;
  static_assert(sizeof(cudaIpcMemHandle_t) <= sizeof(hrb_ipc_handle), "IPC handle size");
  *ptr = nullptr;
  HRB_CUDA(ctx, cudaSetDevice(ctx->device));
  HRB_CUDA(ctx, cudaMalloc(ptr, bytes));
  cudaIpcMemHandle_t h;
  const cudaError_t err = cudaIpcGetMemHandle(&h, *ptr);
  if (err != cudaSuccess) {
    cudaFree(*ptr);
    *ptr = nullptr;
    return cuda_fail(ctx, err, "cudaIpcGetMemHandle");
  }
  std::memset(handle, 0, sizeof(*handle));
  std::memcpy(handle->bytes, &h, sizeof(h));
  return HRB_OK;
}

hrb_status hrb_shared_free(hrb_ctx* ctx, void* ptr) {
  if (ctx == nullptr) return HRB_EINVAL;
  HRB_CUDA(ctx, cudaSetDevice(ctx->device));
  HRB_CUDA(ctx, cudaFree(ptr));
  return HRB_OK;
}

hrb_status hrb_peer_open(hrb_ctx* ctx, const hrb_ipc_handle* handle, void** peer_ptr) {
  if (ctx == nullptr || handle == nullptr || peer_ptr == nullptr) return HRB_EINVAL;
  *peer_ptr = nullptr;
  HRB_CUDA(ctx, cudaSetDevice(ctx->device));
  cudaIpcMemHandle_t h;
  std::memcpy(&h, handle->bytes, sizeof(h));
  HRB_CUDA(ctx, cudaIpcOpenMemHandle(peer_ptr, h, cudaIpcMemLazyEnablePeerAccess));
  return HRB_OK;
}

hrb_status hrb_peer_close(hrb_ctx* ctx, void* peer_ptr) {
  if (ctx == nullptr) return HRB_EINVAL;
  HRB_CUDA(ctx, cudaSetDevice(ctx->device));
  HRB_CUDA(ctx, cudaIpcCloseMemHandle(peer_ptr));
  return HRB_OK;
}

void hrb_shard_columns(uint32_t N, uint32_t rank, uint32_t ranks, uint32_t* n0, uint32_t* n1) {
  if (n0 == nullptr || n1 == nullptr) return;
  if (ranks == 0 || rank >= ranks) {
    *n0 = *n1 = 0;
    return;
  }
  const uint32_t tiles = (N + 127u) / 128u;
  const uint32_t t0 = static_cast<uint32_t>(static_cast<uint64_t>(tiles) * rank / ranks);
  const uint32_t t1 = static_cast<uint32_t>(static_cast<uint64_t>(tiles) * (rank + 1) / ranks);
  *n0 = std::min(N, t0 * 128u);
  *n1 = std::min(N, t1 * 128u);
}

hrb_status hrb_plan_destroy(hrb_plan* plan) {
  if (plan == nullptr) return HRB_OK;
  cudaSetDevice(plan->ctx->device);
  cudaStreamSynchronize(plan->ctx->stream);
  if (plan->s_in != nullptr) {
    cudaStreamSynchronize(plan->s_in);
    cudaStreamSynchronize(plan->s_out);
    for (auto& e : plan->events) cudaEventDestroy(e);
    cudaStreamDestroy(plan->s_in);
    cudaStreamDestroy(plan->s_out);
  }
  cudaFree(plan->d_jobs);
  cudaFree(plan->d_scratch);
  delete plan;
  return HRB_OK;
}

// ---------------------------------------------------------------------------
// Layout translation

hrb_status hrb_wbuf_to_dense(hrb_ctx* ctx, const uint8_t* words, uint32_t groups, uint32_t kb,
                             uint8_t* codes, uint8_t* scales, void* stream) {
  if (ctx == nullptr) return HRB_EINVAL;
  if (!words || !codes || !scales || groups == 0 || kb == 0) return fail(ctx, HRB_EINVAL, "bad WBUF translation");
  HRB_CUDA(ctx, cudaSetDevice(ctx->device));
  hrb::launch_wbuf_to_dense(words, groups, kb, codes, scales, pick(ctx, stream));
  ctx->launches += 1;
  HRB_CUDA(ctx, cudaGetLastError());
  return HRB_OK;
}

hrb_status hrb_w8_planes_to_dense(hrb_ctx* ctx, const uint8_t* hi, const uint8_t* lo,
                                  uint32_t groups, uint32_t kb, int8_t* q, uint8_t* scales,
                                  void* stream) {
  if (ctx == nullptr) return HRB_EINVAL;
  if (!hi || !lo || !q || !scales || groups == 0 || kb == 0) return fail(ctx, HRB_EINVAL, "bad W8 translation");
  HRB_CUDA(ctx, cudaSetDevice(ctx->device));
  hrb::launch_w8_planes_to_dense(hi, lo, groups, kb, q, scales, pick(ctx, stream));
  ctx->launches += 1;
  HRB_CUDA(ctx, cudaGetLastError());
  return HRB_OK;
}

hrb_status hrb_abuf_to_dense(hrb_ctx* ctx, const uint8_t* words, uint32_t quads, uint32_t kb,
                             int8_t* q, uint8_t* scales, void* stream) {
  if (ctx == nullptr) return HRB_EINVAL;
  if (!words || !q || !scales || quads == 0 || kb == 0) return fail(ctx, HRB_EINVAL, "bad ABUF translation");
  HRB_CUDA(ctx, cudaSetDevice(ctx->device));
  hrb::launch_abuf_to_dense(words, quads, kb, q, scales, pick(ctx, stream));
  ctx->launches += 1;
  HRB_CUDA(ctx, cudaGetLastError());
  return HRB_OK;
}

hrb_status hrb_t32_split8_dense(hrb_ctx* ctx, const int8_t* vq, const uint8_t* vscale,
                                uint32_t tokens, uint32_t hd, uint32_t ldv, int8_t* wq,
                                uint8_t* wscale, void* stream) {
  if (ctx == nullptr) return HRB_EINVAL;
  if (!vq || !vscale || !wq || !wscale) return fail(ctx, HRB_EINVAL, "null buffer");
  if (tokens == 0 || hd == 0) return fail(ctx, HRB_EINVAL, "empty V cache %u x %u", tokens, hd);
  if (tokens % 4u != 0) {
    return fail(ctx, HRB_EINVAL, "%u tokens do not fill DMA rows of 4 tokens", tokens);
  }
  // LoadT32's own check (dma_engine.cpp:380-382), on DMA rows of 4 tokens.
  if (tokens % 32u != 0) {
    return fail(ctx, HRB_EINVAL, "T32_SPLIT8 with %u rows, not a multiple of 8", tokens / 4u);
  }
  if (hd % 32u != 0 || ldv % 32u != 0 || ldv < hd) {
    return fail(ctx, HRB_EINVAL, "head dim %u / row stride %u are not whole blocks of 32", hd, ldv);
  }
  if (!aligned(vq, 16) || !aligned(wq, 16)) return fail(ctx, HRB_EINVAL, "misaligned buffer");
  HRB_CUDA(ctx, cudaSetDevice(ctx->device));
  hrb::launch_t32_split8(vq, vscale, tokens, hd, ldv, wq, wscale, ctx->sm_count,
                         pick(ctx, stream));
  ctx->launches += 1;
  HRB_CUDA(ctx, cudaGetLastError());
  return HRB_OK;
}

// ---------------------------------------------------------------------------
// Gather-accumulate

hrb_status hrb_gacc_dense(hrb_ctx* ctx, const hrb_gacc_desc* d, void* stream) {
  if (ctx == nullptr) return HRB_EINVAL;
  if (d == nullptr) return fail(ctx, HRB_EINVAL, "null GACC descriptor");
  if (d->tokens == 0 || d->slots == 0 || d->corners == 0) return HRB_OK;
  if (d->blocks == 0) return fail(ctx, HRB_EINVAL, "GACC with 0 blocks per token");
  if (!d->entries || !d->w || !d->rows || !d->out) return fail(ctx, HRB_EINVAL, "null buffer");
  if (d->row_stride % 8u != 0 || d->row_stride < uint64_t{d->blocks} * 33u ||
      !aligned(d->rows, 8) || !aligned(d->entries, 8) || !aligned(d->w, 4) || !aligned(d->out, 4)) {
    return fail(ctx, HRB_EINVAL, "GACC rows of %llu bytes for %u blocks, or a misaligned buffer",
                static_cast<unsigned long long>(d->row_stride), d->blocks);
  }
  HRB_CUDA(ctx, cudaSetDevice(ctx->device));
  hrb::GaccJob j{};
  j.entries = d->entries;
  j.w = reinterpret_cast<const uint32_t*>(d->w);
  j.rows = d->rows;
  j.row_stride = d->row_stride;
  j.nrows = d->nrows;
  j.out = d->out;
  j.tokens = d->tokens;
  j.slots = d->slots;
  j.corners = d->corners;
  j.blocks = d->blocks;
  j.accumulate = d->accumulate != 0;
  hrb::launch_gacc(j, ctx->d_error, ctx->sm_count, pick(ctx, stream));
  ctx->launches += 1;
  HRB_CUDA(ctx, cudaGetLastError());
  return HRB_OK;
}

// ---------------------------------------------------------------------------
// Convolutions

hrb_status hrb_conv_dense(hrb_ctx* ctx, const hrb_conv_desc* d, void* stream) {
  if (ctx == nullptr) return HRB_EINVAL;
  ConvRun r;
  hrb_status st = check_conv(ctx, d, &r);
  if (st != HRB_OK) return st;
  HRB_CUDA(ctx, cudaSetDevice(ctx->device));
  cudaStream_t s = pick(ctx, stream);
  st = grow(ctx, &ctx->scratch, &ctx->scratch_bytes, r.bytes);
  if (st != HRB_OK) return st;
  auto* base = static_cast<uint8_t*>(ctx->scratch);
  uint32_t launched = 0;
  st = conv_prepare(ctx, d, r, base, s, &launched);
  if (st == HRB_OK) st = conv_execute(ctx, d, r, base, s, &launched);
  ctx->launches += launched;
  return st;
}

hrb_status hrb_conv_plan_create(hrb_ctx* ctx, const hrb_conv_desc* d, hrb_conv_plan** out) {
  if (ctx == nullptr || out == nullptr) return HRB_EINVAL;
  *out = nullptr;
  ConvRun r;
  hrb_status st = check_conv(ctx, d, &r);
  if (st != HRB_OK) return st;
  HRB_CUDA(ctx, cudaSetDevice(ctx->device));
  auto* plan = new hrb_conv_plan;
  plan->ctx = ctx;
  plan->desc = *d;
  if (r.bytes != 0) {
    const cudaError_t e = cudaMalloc(&plan->d_scratch, r.bytes);
    if (e != cudaSuccess) {
      delete plan;
      return cuda_fail(ctx, e, "cudaMalloc");
    }
  }
  uint32_t launched = 0;
  st = conv_prepare(ctx, d, r, static_cast<uint8_t*>(plan->d_scratch), ctx->stream, &launched);
  if (st == HRB_OK) {
    const cudaError_t e = cudaStreamSynchronize(ctx->stream);
    if (e != cudaSuccess) st = cuda_fail(ctx, e, "conv plan preparation");
  }
  ctx->launches += launched;
  if (st != HRB_OK) {
    cudaFree(plan->d_scratch);
    delete plan;
    return st;
  }
  *out = plan;
  return HRB_OK;
}

hrb_status hrb_conv_plan_run(hrb_conv_plan* plan, void* stream, uint32_t* launched) {
  if (plan == nullptr) return HRB_EINVAL;
  hrb_ctx* ctx = plan->ctx;
  ConvRun r;
  hrb_status st = check_conv(ctx, &plan->desc, &r);
  if (st != HRB_OK) return st;
  HRB_CUDA(ctx, cudaSetDevice(ctx->device));
  uint32_t n = 0;
  st = conv_execute(ctx, &plan->desc, r, static_cast<uint8_t*>(plan->d_scratch),
                    pick(ctx, stream), &n, -1, &plan->peers);
  ctx->launches += n;
  if (launched != nullptr) *launched = n;
  return st;
}

hrb_status hrb_conv_plan_set_peers(hrb_conv_plan* plan, const void* local_base,
                                   void* const* peer_bases, uint32_t npeers) {
  if (plan == nullptr) return HRB_EINVAL;
  hrb_ctx* ctx = plan->ctx;
  if (npeers > hrb::kMaxPeers || (npeers > 0 && (local_base == nullptr || peer_bases == nullptr))) {
    return fail(ctx, HRB_EINVAL, "at most %u peers, with a local base", hrb::kMaxPeers);
  }
  ConvRun r;
  const hrb_status st = check_conv(ctx, &plan->desc, &r);
  if (st != HRB_OK) return st;
  if (npeers > 0 && !r.tc) {
    return fail(ctx, HRB_ENOTSUP, "peer outputs need the tensor-core convolution");
  }
  hrb::MxPeers peers{};
  peers.count = npeers;
  for (uint32_t i = 0; i < npeers; ++i) {
    if (peer_bases[i] == nullptr) return fail(ctx, HRB_EINVAL, "null peer base");
    peers.delta[i] = static_cast<const char*>(peer_bases[i]) - static_cast<const char*>(local_base);
  }
  HRB_CUDA(ctx, cudaStreamSynchronize(ctx->stream));  // no run in flight sees half a change
  plan->peers = peers;
  return HRB_OK;
}

hrb_status hrb_conv_plan_profile(hrb_conv_plan* plan, void* stream, uint32_t reps, float* ms,
                                 uint32_t cap, uint32_t* nkernels) {
  if (plan == nullptr || ms == nullptr || nkernels == nullptr || reps == 0 || cap == 0) {
    return HRB_EINVAL;
  }
  hrb_ctx* ctx = plan->ctx;
  ConvRun r;
  hrb_status st = check_conv(ctx, &plan->desc, &r);
  if (st != HRB_OK) return st;
  HRB_CUDA(ctx, cudaSetDevice(ctx->device));
  cudaStream_t s = pick(ctx, stream);
  auto* base = static_cast<uint8_t*>(plan->d_scratch);
  const uint32_t steps = std::min(conv_launches(&plan->desc, r), cap);
  cudaEvent_t ev[2];
  HRB_CUDA(ctx, cudaEventCreate(&ev[0]));
  HRB_CUDA(ctx, cudaEventCreate(&ev[1]));
  uint32_t n = 0;
  st = conv_execute(ctx, &plan->desc, r, base, s, &n);
  for (uint32_t i = 0; i < steps && st == HRB_OK; ++i) {
    st = conv_execute(ctx, &plan->desc, r, base, s, &n, static_cast<int>(i));  // warm
    if (st == HRB_OK && cudaEventRecord(ev[0], s) != cudaSuccess) st = HRB_ECUDA;
    for (uint32_t k = 0; k < reps && st == HRB_OK; ++k) {
      st = conv_execute(ctx, &plan->desc, r, base, s, &n, static_cast<int>(i));
    }
    if (st == HRB_OK && cudaEventRecord(ev[1], s) != cudaSuccess) st = HRB_ECUDA;
    float t = 0;
    if (st == HRB_OK && (cudaEventSynchronize(ev[1]) != cudaSuccess ||
                         cudaEventElapsedTime(&t, ev[0], ev[1]) != cudaSuccess)) {
      st = HRB_ECUDA;
    }
    ms[i] = t / static_cast<float>(reps);
  }
  cudaEventDestroy(ev[0]);
  cudaEventDestroy(ev[1]);
  ctx->launches += n;
  if (st != HRB_OK) return st == HRB_ECUDA ? fail(ctx, st, "profiling run failed") : st;
  *nkernels = steps;
  return HRB_OK;
}

hrb_status hrb_conv_plan_destroy(hrb_conv_plan* plan) {
  if (plan == nullptr) return HRB_OK;
  cudaSetDevice(plan->ctx->device);
  cudaStreamSynchronize(plan->ctx->stream);
  cudaFree(plan->d_scratch);
  delete plan;
  return HRB_OK;
}

hrb_status hrb_dense_to_fbuf(hrb_ctx* ctx, const float* c, uint32_t rows, uint32_t cols,
                             float* words, void* stream) {
  if (ctx == nullptr) return HRB_EINVAL;
  if (!c || !words || rows % 4 != 0 || cols % 8 != 0 || rows == 0 || cols == 0) {
    return fail(ctx, HRB_EINVAL, "FBUF matrix %ux%u is not a multiple of 4x8", rows, cols);
  }
  HRB_CUDA(ctx, cudaSetDevice(ctx->device));
  hrb::launch_dense_to_fbuf(c, rows, cols, words, pick(ctx, stream));
  ctx->launches += 1;
  HRB_CUDA(ctx, cudaGetLastError());
  return HRB_OK;
}

}  // extern "C"
