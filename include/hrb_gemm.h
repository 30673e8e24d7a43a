/* hrb_gemm.h — C ABI of the B200 backend for hotarubi's quantized GEMM.
 *
 * The hot path it replaces is the GEMM instruction of hotarubi's NPU as the
 * instruction-set simulator executes it:
 *
 *   void hotarubi::iss::ExecuteGemm(const GemmCommand&, Memories&);
 *       (tools/iss/gemm_array.hpp:33, tools/iss/gemm_array.cpp:112-149,
 *        called from Machine::Execute, tools/iss/machine.cpp:339-343)
 *
 * and the dense Linear that hotarubi's compiler lowers into a chain of such
 * instructions (LinearEmitter::Emit, tools/compiler/kernels.cpp:343-395).
 *
 * Conventions
 *   - Plain C: pointers and sizes only.  No exception or C++ type crosses.
 *   - Every entry point returns an hrb_status.  Where the reference calls
 *     Require() (and aborts), this library returns HRB_EINVAL and keeps a
 *     message for hrb_last_error(); the reference-facing C++ shim
 *     (hotarubi_b200/host/iss_gemm.hpp) turns that back into the reference's
 *     abort.
 *   - FP32 data is IEEE binary32.  Results follow hotarubi's FP32 rules
 *     (round to nearest even, subnormal inputs and results flushed to +0, a
 *     zero result is +0): docs/design.md "Number formats" of the reference.
 *   - "stream" arguments are cudaStream_t values passed as void*; NULL means
 *     the context's own stream.
 */
#ifndef HRB_GEMM_H_
#define HRB_GEMM_H_

#include <stddef.h>
#include <stdint.h>

#if defined(__GNUC__)
#define HRB_API __attribute__((visibility("default")))
#else
#define HRB_API
#endif

#ifdef __cplusplus
extern "C" {
#endif

typedef enum hrb_status {
  HRB_OK = 0,
  HRB_EINVAL = 1,   /* invalid argument: the reference would Require()-fail */
  HRB_ECUDA = 2,    /* a CUDA runtime call failed (message in hrb_last_error) */
  HRB_ENOMEM = 3,   /* device or pinned host allocation failed */
  HRB_ENOTSUP = 4,  /* valid request this build does not serve */
  HRB_EDATA = 5     /* non-finite activation given to the MXINT8 encoder
                       (formats.cpp:37 Require) */
} hrb_status;

typedef struct hrb_ctx hrb_ctx;

/* ---------------------------------------------------------------------
 * Lifecycle
 * ------------------------------------------------------------------- */

/* Creates a context on CUDA device `device` with its own non-blocking
 * stream.  Device buffers the context needs are owned by it, and the calls
 * of one context share them: issue a context's calls from one host thread
 * and on one stream (or order the streams), and use one context per
 * concurrent stream otherwise.  Plans own their own buffers. */
HRB_API hrb_status hrb_create(int device, hrb_ctx** out);
HRB_API hrb_status hrb_destroy(hrb_ctx* ctx);
/* Waits for all work on the context's stream; returns HRB_EDATA when an
 * MXINT8 encode since the last sync met Inf/NaN. */
HRB_API hrb_status hrb_sync(hrb_ctx* ctx);
/* Message of the last failed call on this context ("" if none); with NULL,
 * of the last failed call this thread made without a context. */
HRB_API const char* hrb_last_error(const hrb_ctx* ctx);
HRB_API const char* hrb_status_string(hrb_status status);
/* The context's stream (a cudaStream_t) and a way to replace it. */
HRB_API void* hrb_get_stream(const hrb_ctx* ctx);
HRB_API hrb_status hrb_set_stream(hrb_ctx* ctx, void* stream);
/* Number of this library's kernels launched on the context so far. */
HRB_API uint64_t hrb_launch_count(const hrb_ctx* ctx);

/* ---------------------------------------------------------------------
 * 1. The ISS drop-in: one GEMM instruction over the NPU's on-chip memories
 * ------------------------------------------------------------------- */

/* GemmCommand (tools/iss/gemm_array.hpp:16-27), field for field. */
typedef struct hrb_gemm_cmd {
  uint32_t a_base;   /* ABUF word of token quad 0, block 0 */
  uint32_t a_stride; /* ABUF words between token quads */
  uint32_t kb;       /* K blocks of 32 */
  uint32_t m;        /* tokens: a multiple of 32 from 32 to 992 */
  uint32_t w_base;   /* WBUF word of column group 0, block 0 */
  uint32_t w_stride; /* WBUF words between column groups of 8 */
  uint32_t n8;       /* column groups of 8, 1..255 */
  uint32_t c_base;   /* FBUF word of quad 0, group 0 */
  uint32_t wmode;    /* 0 FP4, 1 W8_HI, 2 and 3 W8_LO (isa.hpp:88-92) */
  uint32_t acc;      /* nonzero: accumulate onto FBUF */
} hrb_gemm_cmd;

/* Memory geometry of the reference (tools/iss/memories.hpp:20-27). */
#define HRB_ABUF_WORDS 8192u
#define HRB_ABUF_WORD_BYTES 132u
#define HRB_WBUF_WORDS 2048u
#define HRB_WBUF_WORD_BYTES 144u
#define HRB_FBUF_WORDS 4096u
#define HRB_FBUF_WORD_FLOATS 32u

/* DecodeGemm (tools/iss/machine.cpp:93-104): the GEMM fields of one 128-bit
 * instruction given as 16 little-endian bytes (isa.hpp:75-86). */
HRB_API hrb_status hrb_gemm_decode(const uint8_t instruction[16], hrb_gemm_cmd* out);

/* The checks of ExecuteGemm (gemm_array.cpp:113-119): HRB_OK or HRB_EINVAL
 * with the reference's message in hrb_last_error (ctx may be NULL). */
HRB_API hrb_status hrb_gemm_check(hrb_ctx* ctx, const hrb_gemm_cmd* cmd);

/* ExecuteGemm (gemm_array.cpp:112-149) on host-resident memories:
 *   abuf: HRB_ABUF_WORDS x 132 bytes, wbuf: HRB_WBUF_WORDS x 144 bytes,
 *   fbuf: HRB_FBUF_WORDS x 32 FP32 bit patterns, updated in place.
 * Addresses are masked to 20 bits and wrap modulo each depth as in the
 * reference.  Bit-exact with the reference.  Synchronous: fbuf holds the
 * result on return, as Machine::Execute requires (machine.cpp:281-298). */
HRB_API hrb_status hrb_gemm_exec(hrb_ctx* ctx, const hrb_gemm_cmd* cmd,
                         const uint8_t* abuf, const uint8_t* wbuf,
                         uint32_t* fbuf);

/* The same on device-resident memories (same layouts), asynchronous on
 * `stream`.  For a simulator that keeps its memories on the GPU. */
HRB_API hrb_status hrb_gemm_exec_device(hrb_ctx* ctx, const hrb_gemm_cmd* cmd,
                                const void* abuf, const void* wbuf,
                                void* fbuf, void* stream);

/* The words ExecuteGemm records in Memories::log (gemm_array.cpp:127,135,
 * 141,145): one byte per word, set to 1 when touched.  Host-only. */
HRB_API hrb_status hrb_gemm_accesses(const hrb_gemm_cmd* cmd, uint8_t* abuf_reads,
                             uint8_t* wbuf_reads, uint8_t* fbuf_reads,
                             uint8_t* fbuf_writes);

/* NPU-equivalent time: the ISS cycle model of one GEMM instruction
 * (CostModel::Gemm, tools/iss/timing.cpp:65-67,89-93, default parameters):
 * n8 * (m / 32) * kb * 8 array cycles plus 51 fixed.  The NPU's clock is
 * 250 MHz (docs/design.md:27). */
HRB_API uint64_t hrb_gemm_npu_cycles(const hrb_gemm_cmd* cmd);

/* ... of a dense M x N x K GEMM run as GEMM instructions the way a runtime
 * must tile it into the on-chip memories (rows in chunks of at most 992 and
 * 8192 / kb quads, 8-column groups in tiles of at most 255 and 2048 / kb,
 * chunk x tile within FBUF's 4096 words), W8 as its two planes.  0 for
 * MXFP8 (no NPU instruction), for N not a multiple of 8 or kb > 2048. */
HRB_API uint64_t hrb_dense_npu_cycles(uint32_t wfmt, uint32_t M, uint32_t N, uint32_t K);

/* ---------------------------------------------------------------------
 * 2. Dense GEMM: a whole Linear as hotarubi's compiler lowers it
 * ------------------------------------------------------------------- */

/* Weight formats.  kp = K rounded up to a multiple of 32, kb = kp / 32;
 * a K tail is zero padding (formats.cpp:60, docs/design.md).  Scales are
 * E8M0 bytes (e + 127), one per (output column, K block): [N][kb]. */
typedef enum hrb_wfmt {
  /* MXFP4: [N][kp/2] bytes, element 2j in the low nibble of byte j (the nibble
   * order of a WBUF word, tensors.cpp:78-84); FP4 mode, SBIAS -7. */
  HRB_WFMT_MXFP4 = 0,
  /* W8: MXINT8 weights [N][kp] int8, run as a W8_HI chain then a W8_LO chain
   * (SplitW8, weights.cpp:72-88; kernels.cpp:35-37). */
  HRB_WFMT_W8 = 1,
  /* MXFP8: [N][kp] OCP E4M3 bytes.  No reference counterpart: block sums are
   * exact and rounded once to FP32 (nearest even), chained like FP4. */
  HRB_WFMT_MXFP8 = 2
} hrb_wfmt;

typedef enum hrb_mode {
  /* Bit-exact with the reference chain: each output's block values are
   * added one by one in K order (W8: all HI blocks, then all LO blocks). */
  HRB_MODE_EXACT = 0,
  /* Tensor-core accumulation: within the stated FP32 tolerance of the exact
   * chain (block values summed in another order). */
  HRB_MODE_FAST = 1
} hrb_mode;

typedef enum hrb_quant {
  HRB_QUANT_HOST = 0, /* EncodeMxint8 (formats.cpp:35-56,138-162) */
  HRB_QUANT_VEC = 1   /* VEC 'q' pass (lane.cpp:384-423): subnormals -> 0 */
} hrb_quant;

typedef struct hrb_gemm_desc {
  uint32_t wfmt;       /* hrb_wfmt */
  uint32_t mode;       /* hrb_mode */
  uint32_t M, N, K;    /* C[M][N] (+)= A[M][K] . W[N][K]^T, then + bias */
  /* Activations: either FP32 `a` [M][lda] (encoded to MXINT8 on the device
   * with `quant`), or pre-encoded `aq` [M][kp] int8 with `ascale` [M][kb]. */
  const float* a;
  uint32_t lda;
  uint32_t quant;      /* hrb_quant, for `a` */
  const int8_t* aq;
  const uint8_t* ascale;
  /* Weights in `wfmt` and their scales [N][kb]. */
  const uint8_t* w;
  const uint8_t* wscale;
  const float* bias;   /* [N] or NULL: one FP32 add after the chain (ADDP,
                          sparsedrive_encoder.cpp:422-428) */
  float* c;            /* [M][ldc] */
  uint32_t ldc;
  uint32_t accumulate; /* nonzero: chains start from C's contents */
  /* K pieces, in blocks (the LinearPiece split of kernels.hpp:70-75): the
   * chain runs piece by piece, planes in order within each piece.  NULL or
   * npieces 0: one piece of kb blocks.  At most 64 pieces. */
  const uint32_t* pieces;
  uint32_t npieces;
  /* Optional MXINT8 copy of the output for the next layer: the VEC 'q' pass
   * that follows GEMM + ADDP on the NPU (QuantizeBlock, lane.cpp:406-423),
   * fused into the GEMM's epilogue.  C's final FP32 values (after bias and
   * accumulate) as codes cq [M][kpN] int8 (kpN = N rounded up to 32; the
   * padding columns hold 0) and scale bytes cscale [M][kpN / 32], rounded
   * with cquant (hrb_quant).  NULL: none.  In HRB_MODE_FAST with FP32
   * activations, c may then be NULL (no FP32 output; not with
   * accumulate). */
  int8_t* cq;
  uint8_t* cscale;
  uint32_t cquant;
  /* Optional FP32 scale per output column [N] (NULL: none): each output's
   * finished chain is multiplied by wcol_scale[n] before the bias is added,
   * in HRB_MODE_EXACT with the ISS's FP32 multiply (fp32.hpp:77-92, bit for
   * bit), in HRB_MODE_FAST with the IEEE multiply (round to nearest even).
   * With W8 codes whose block scale bytes are all 133 (2^6, so every code
   * counts as its integer value) this is int8 weights with a per-output-
   * channel scale and a fused scale/bias epilogue, a format the reference
   * does not have (hotarubi places such a matrix as MXINT8 blocks, PlaceW8).
   * Not with accumulate.  4-byte aligned. */
  const float* wcol_scale;
  /* HRB_MODE_FAST, W8, M <= 64 only (ignored otherwise): which tensor-core
   * kernel runs.  HRB_W8_DIGIT_PLANES (0, the default): the weights as three
   * E2M1 digit planes translated once, kind::mxf4.  HRB_W8_BF16: the int8
   * codes stream as they are (one byte a weight) and the kernel converts
   * them to BF16 in tensor memory, kind::f16.  Both are exact in their
   * products; on the B200 the digit planes are the faster of the two. */
  uint32_t w8_kernel;
  /* Row stride of the MXINT8 copy in codes (a multiple of 32, at least kpN;
   * the scales' row stride is ldcq / 32): cq[m * ldcq + n], cscale[m *
   * ldcq / 32 + n / 32].  0: kpN, the packed layout above.  A GEMM over a
   * column slice of a wider matrix (a rank's N shard) writes its copy into
   * the full matrix's layout with cq and cscale pointing at the slice's
   * first column (a multiple of 32). */
  uint32_t ldcq;
} hrb_gemm_desc;

enum { HRB_W8_DIGIT_PLANES = 0, HRB_W8_BF16 = 1 };

/* One dense GEMM, all pointers device pointers, asynchronous on `stream`. */
HRB_API hrb_status hrb_gemm_dense(hrb_ctx* ctx, const hrb_gemm_desc* desc, void* stream);

/* The same with HOST pointers: copies the operands in, runs, copies C out,
 * synchronizes.  The call a host-side caller (the ISS, a runtime) makes. */
HRB_API hrb_status hrb_gemm_dense_host(hrb_ctx* ctx, const hrb_gemm_desc* desc);

/* hrb_gemm_dense for callers that cannot allocate device memory.  No
 * counterpart in the reference: hotarubi's GEMM runs in the simulator's own
 * host memory.  Some hosts of this backend may not call cudaMalloc (a
 * simulator plugin inside a process whose device memory someone else owns,
 * code that runs during stream capture, a real-time loop): this entry point
 * takes the same descriptor with device pointers for all inputs and outputs,
 * needs no context, and allocates nothing.  Its only scratch, the MXINT8
 * encoding of FP32 activations, lives in a fixed device array of
 * HRB_NOALLOC_SCRATCH_BYTES that every GPU loading the library holds until
 * exit; an FP32-input GEMM whose encoding (M*kp code bytes plus M*kp/32
 * scale bytes, each rounded up to 256) does not fit returns HRB_EINVAL.
 * All calls share that array: calls that overlap on the GPU race, so
 * serialise them on one stream.  The first call on a device (the current
 * device) looks the array's address up; make it before any stream capture.
 * That address belongs to the runtime's primary context, the only context
 * this entry point supports; it is not looked up again after a
 * cudaDeviceReset.  Runs on `stream` (NULL: the default stream).  Failures
 * leave a message for hrb_last_error(NULL); a CUDA error already pending on
 * the calling thread makes the call return HRB_ECUDA without launching.
 * Non-finite activations are not reported. */
#define HRB_NOALLOC_SCRATCH_BYTES (4u << 20)
HRB_API hrb_status hrb_gemm_dense_noalloc(const hrb_gemm_desc* desc, void* stream);

/* FP32 [rows][ldx] -> MXINT8 q [rows][kp] + scale bytes [rows][kb] on the
 * device (the prologue of every GEMM; the VEC 'q' pass on the NPU). */
HRB_API hrb_status hrb_quantize_mxint8(hrb_ctx* ctx, const float* x, uint32_t rows,
                               uint32_t cols, uint32_t ldx, uint32_t quant,
                               int8_t* q, uint8_t* scale, void* stream);

/* ---------------------------------------------------------------------
 * 3. Plans: a batch of independent dense GEMMs, prepared once, launched many
 *    times without allocation or host synchronisation (capturable into a
 *    CUDA graph).  Each GEMM keeps its own operands.
 * ------------------------------------------------------------------- */

typedef struct hrb_plan hrb_plan;

/* Weights are translated once, here: they must not change while the plan
 * lives.  HRB_MODE_FAST GEMMs with wcol_scale also read the column scales
 * and the bias here. */
HRB_API hrb_status hrb_plan_create(hrb_ctx* ctx, const hrb_gemm_desc* descs,
                           uint32_t count, hrb_plan** out);
/* Launches the whole batch on `stream`; returns the number of kernels it
 * launched in *launches (may be NULL). */
HRB_API hrb_status hrb_plan_run(hrb_plan* plan, void* stream, uint32_t* launches);
/* The plan end to end with host buffers, asynchronous on `stream`: for each
 * GEMM i in creation order, copies a_host[i] into the activations the
 * descriptor named (FP32 rows, or MXINT8 codes plus ascale_host[i]), runs the
 * plan, and copies C (M rows of ldc floats) into c_host[i].  A NULL array or
 * NULL entry skips that copy; weights and bias stay resident.  Host buffers
 * should be pinned.  Wait with hrb_sync or on the stream. */
HRB_API hrb_status hrb_plan_run_host(hrb_plan* plan, void* stream, const void* const* a_host,
                                     const void* const* ascale_host, void* const* c_host);
HRB_API hrb_status hrb_plan_destroy(hrb_plan* plan);
/* Measurement aid: runs the plan once, then each of its launches alone,
 * `reps` times back to back between two CUDA events on `stream`, and writes
 * the mean milliseconds of launch i to ms[i] for the first min(launches, cap)
 * launches; *nkernels receives that count.  Launch 0 is the activation
 * encoder when the plan has FP32 inputs, then one GEMM launch per group.
 * Repeated launches recompute the same outputs, except that GEMMs with
 * `accumulate` set add onto C again. */
HRB_API hrb_status hrb_plan_profile(hrb_plan* plan, void* stream, uint32_t reps, float* ms,
                                    uint32_t cap, uint32_t* nkernels);

/* ---------------------------------------------------------------------
 * 4. Layout translation between hotarubi's image.bin word streams and the
 *    dense formats (device pointers, asynchronous).
 * ------------------------------------------------------------------- */

/* A WBUF word stream of one plane as the compiler places it (PackWbuf,
 * tensors.cpp:66-90: word (g * kb + b), 144 bytes, nibbles then 8 scales),
 * to dense 4-bit codes [8*groups][kb*16] bytes and scales [8*groups][kb]. */
HRB_API hrb_status hrb_wbuf_to_dense(hrb_ctx* ctx, const uint8_t* words,
                             uint32_t groups, uint32_t kb, uint8_t* codes,
                             uint8_t* scales, void* stream);

/* Two W8 planes (HI words, LO words, same geometry) back to MXINT8 weights
 * [8*groups][kb*32] int8 and their scales (the inverse of SplitW8). */
HRB_API hrb_status hrb_w8_planes_to_dense(hrb_ctx* ctx, const uint8_t* hi_words,
                                  const uint8_t* lo_words, uint32_t groups,
                                  uint32_t kb, int8_t* q, uint8_t* scales,
                                  void* stream);

/* ABUF words (PackAbuf, formats.cpp:114-136; 144-byte DDR words in (quad,
 * block) order) to MXINT8 activations [4*quads][kb*32] and scales. */
HRB_API hrb_status hrb_abuf_to_dense(hrb_ctx* ctx, const uint8_t* words,
                             uint32_t quads, uint32_t kb, int8_t* q,
                             uint8_t* scales, void* stream);

/* Attention operands from an MXINT8 K/V cache (one head; tokens along rows,
 * one scale byte per token and 32-dim block, as the row format holds them).
 *
 * Q.K^T: the DMA engine's SPLIT8 load (LoadSplit8, dma_engine.cpp:303-334)
 * only splits the K cache's codes into the HI/LO planes of a W8 operand, so
 * the dense K cache [tokens][hd] with its scales [tokens][hd/32] is passed
 * to hrb_gemm_dense as W8 weights as it is (N = tokens, K = hd).
 *
 * P.V: T32_SPLIT8 (LoadT32 + TransposeGroup, dma_engine.cpp:336-405)
 * replaces the V cache by its transpose in 32 x 32 blocks, each token's codes
 * re-aligned to the largest scale of the block's tokens that are not all zero
 * (AlignElement, dma_engine.cpp:532-544: RNE right shift; lossy unless the
 * scales are equal; 127 for a block of zero tokens).  hrb_t32_split8_dense
 * writes that W8 operand: wq [hd][tokens] codes, wscale [hd][tokens/32],
 * from vq [tokens][ldv] and vscale [tokens][ldv/32] (ldv >= hd, both
 * multiples of 32; tokens a multiple of 32, i.e. DMA rows in groups of 8).
 * vq and wq are 16-byte aligned device pointers.  Asynchronous, one launch.
 * HRB_EINVAL with the reference's message for a token count that is not a
 * multiple of 32. */
HRB_API hrb_status hrb_t32_split8_dense(hrb_ctx* ctx, const int8_t* vq, const uint8_t* vscale,
                                        uint32_t tokens, uint32_t hd, uint32_t ldv, int8_t* wq,
                                        uint8_t* wscale, void* stream);

/* Row-major FP32 [rows][cols] to FBUF words (PackFbuf, formats.cpp:72-88). */
HRB_API hrb_status hrb_dense_to_fbuf(hrb_ctx* ctx, const float* c, uint32_t rows,
                             uint32_t cols, float* words, void* stream);

/* ---------------------------------------------------------------------
 * 5. Convolutions as hotarubi's compiler lowers them (ConvEmitter,
 *    tools/compiler/sparsedrive_encoder.cpp:78-168,384-428): one GEMM per
 *    (channel plane, tap) over activations gathered per tap, all chaining
 *    into the same outputs, then ADDP of the bias, then optionally RELU and
 *    the VEC 'q' pass.  A position outside the map reads as the DMA engine's
 *    null entry (a zero token, dma_engine.cpp:247-256), i.e. zero padding
 *    (kh - 1) / 2.  Here the whole conv is one GEMM with gathered activation
 *    rows: M = images * Ho * Wo output positions, N = cout, K = kh * kh * cin
 *    in the chain's order (plane of 256 channels, tap, channel).
 * ------------------------------------------------------------------- */

/* Position order of a feature map (and of the output rows). */
typedef enum hrb_conv_order {
  HRB_CONV_XMAJOR = 0,  /* position x * H + y: the compiler's FMap order */
  HRB_CONV_YMAJOR = 1   /* position y * W + x: NHWC */
} hrb_conv_order;

typedef struct hrb_conv_desc {
  uint32_t wfmt;        /* hrb_wfmt (the compiler's convs are MXFP4) */
  uint32_t mode;        /* hrb_mode */
  uint32_t images, H, W;
  uint32_t cin, cout;   /* cin a multiple of 32, and of 256 when above 256
                           (MakeMap's channel planes, sparsedrive_common.cpp:
                           47-68) */
  uint32_t kh;          /* 1 or 3 */
  uint32_t stride;      /* 1 or 2: Ho = H / stride, Wo = W / stride */
  uint32_t order;       /* hrb_conv_order */
  /* The input map: FP32 `a` [images][H * W][cin] (16-byte aligned), encoded
   * with `quant`, or MXINT8 `aq` [images][H * W][cin] with `ascale`
   * [images][H * W][cin / 32]. */
  const float* a;
  uint32_t quant;
  const int8_t* aq;
  const uint8_t* ascale;
  /* The conv matrix [cout][kh * kh * cin] in `wfmt`, tap-major columns
   * (tap = ky * kh + kx, ConvTile, sparsedrive_common.cpp:136-158), and its
   * scales [cout][kh * kh * cin / 32].  16-byte aligned. */
  const uint8_t* w;
  const uint8_t* wscale;
  const float* bias;    /* [cout] or NULL */
  float* c;             /* [images * Ho * Wo][cout], positions in `order` */
  uint32_t accumulate;  /* chains start from C: a residual (the emitter's
                           residual load into FBUF, :385-390) */
  uint32_t relu;        /* RELU after the bias (lane.cpp:57-70,322-326) */
  int8_t* cq;           /* optional MXINT8 copy [M][kpN] + [M][kpN / 32] of */
  uint8_t* cscale;      /* the final output, as hrb_gemm_desc's */
  uint32_t cquant;
} hrb_conv_desc;

/* One convolution, device pointers, asynchronous on `stream`: HRB_MODE_EXACT
 * gives the compiler's chain bit for bit; HRB_MODE_FAST with FP32 `a` runs
 * the tensor cores (the map is encoded once, each output row's taps are
 * gathered as operand blocks), within the tolerance of hrb_gemm_desc for
 * K = kh * kh * cin. */
HRB_API hrb_status hrb_conv_dense(hrb_ctx* ctx, const hrb_conv_desc* desc, void* stream);

/* A convolution prepared once (weights reordered and translated, scratch
 * allocated), then run many times with no allocation or host sync; the
 * descriptor's pointers must stay valid.  *launched receives the kernels of
 * one run. */
typedef struct hrb_conv_plan hrb_conv_plan;
HRB_API hrb_status hrb_conv_plan_create(hrb_ctx* ctx, const hrb_conv_desc* desc,
                                        hrb_conv_plan** out);
HRB_API hrb_status hrb_conv_plan_run(hrb_conv_plan* plan, void* stream, uint32_t* launched);
/* Measurement aid, as hrb_plan_profile: one run, then each of the run's
 * launches alone `reps` times back to back between two events; ms[i] is the
 * mean of launch i (fast mode: 0 the map's encoder, 1 the gather of the
 * GEMM's operand blocks, 2 the GEMM). */
HRB_API hrb_status hrb_conv_plan_profile(hrb_conv_plan* plan, void* stream, uint32_t reps,
                                         float* ms, uint32_t cap, uint32_t* nkernels);
HRB_API hrb_status hrb_conv_plan_destroy(hrb_conv_plan* plan);
/* Row-sharded convolutions (the images of a batch split over the GPUs of a
 * node, hrb_shard_rows; each rank's plan covers its images, with `c`, `cq`
 * and `cscale` pointing at its rows of full-size buffers): every later run
 * also stores each output byte at address x (C and the MXINT8 copy) into
 * peer_bases[i] + (x - local_base) over NVLink, so that once every rank's
 * run has finished every rank holds all rows.  The outputs must lie in one
 * buffer from local_base (hrb_shared_alloc) whose layout is the same on
 * every rank.  At most 7 peers; HRB_MODE_FAST with FP32 input only (else
 * HRB_ENOTSUP).  With 16-byte aligned buffers the FP32 outputs travel as
 * 16-byte stores. */
HRB_API hrb_status hrb_conv_plan_set_peers(hrb_conv_plan* plan, const void* local_base,
                                           void* const* peer_bases, uint32_t npeers);

/* ---------------------------------------------------------------------
 * 7. GACC, the DMA engine's gather-accumulate (DmaEngine::Gather,
 *    tools/iss/dma_engine.cpp:599-652): SparseDrive's deformable sampling.
 *    Per output token t, the chain over slots s, then corners k, of entry
 *    e = entries[t][s][k] (low 32 bits: feature row index, 0xFFFFFFFF a
 *    null entry that adds nothing; high 32 bits: the FP32 bits of its
 *    bilinear weight bw):
 *      coef_b = ScaleCoefficient(w[t][s][b] * bw, the row's scale byte b)
 *      out[t][32b + v] += Int8ToFp32(the row's code 32b + v) * coef_b
 *    in the ISS's FP32 arithmetic (fp32.hpp:46-92; dma_engine.cpp:478-528),
 *    bit for bit.  One GACC instruction is this for 4 tokens, 4 corners and
 *    at most 8 blocks, its list holding the entries and its coefficient
 *    banks the w values; a sequence with `acc` set is one longer chain.
 * ------------------------------------------------------------------- */

typedef struct hrb_gacc_desc {
  uint32_t tokens, slots, corners;
  uint32_t blocks;          /* 32-channel blocks per feature row (>= 1) */
  const uint64_t* entries;  /* [tokens][slots][corners] */
  const float* w;           /* [tokens][slots][blocks] */
  /* Feature rows in the DMA row format: `blocks` 32-byte blocks of int8
   * codes, then `blocks` scale bytes; row_stride bytes apart (a multiple of
   * 8, at least blocks * 33), nrows of them; 8-byte aligned. */
  const uint8_t* rows;
  uint64_t row_stride;
  uint32_t nrows;
  float* out;               /* [tokens][blocks * 32] */
  uint32_t accumulate;      /* chains start from out's contents, else +0 */
} hrb_gacc_desc;

/* Device pointers, asynchronous.  An entry naming a row at or past nrows is
 * skipped and reported by hrb_sync as HRB_EDATA (the ISS aborts on an
 * address outside its DDR). */
HRB_API hrb_status hrb_gacc_dense(hrb_ctx* ctx, const hrb_gacc_desc* desc, void* stream);

/* ---------------------------------------------------------------------
 * 6. Column-sharded GEMMs over the GPUs of one node (one process per GPU).
 *    Rank r of G computes output columns [n0, n1) (hrb_shard_columns) of
 *    every GEMM with its slice of W.  With peers set on a plan, the kernel's
 *    epilogue stores each output into the local C and, over NVLink, into
 *    every peer's C at the same offset: once every rank's run has finished
 *    (the caller synchronises the ranks, e.g. a barrier), every rank holds
 *    the whole of C.  This is the all-gather of the output slices fused into
 *    the GEMM; peers' buffers are mapped with CUDA IPC handles.
 * ------------------------------------------------------------------- */

typedef struct hrb_ipc_handle {
  uint8_t bytes[64];
} hrb_ipc_handle;

/* Device memory another process can map: `bytes` on the context's device,
 * and the handle that names it. */
HRB_API hrb_status hrb_shared_alloc(hrb_ctx* ctx, size_t bytes, void** ptr,
                                    hrb_ipc_handle* handle);
HRB_API hrb_status hrb_shared_free(hrb_ctx* ctx, void* ptr);
/* Maps a peer's hrb_shared_alloc buffer into this process (peer access over
 * NVLink enabled on first use); the pointer is valid on ctx's device. */
HRB_API hrb_status hrb_peer_open(hrb_ctx* ctx, const hrb_ipc_handle* handle, void** peer_ptr);
HRB_API hrb_status hrb_peer_close(hrb_ctx* ctx, void* peer_ptr);
/* Output columns of rank `rank` of `ranks` for N columns: whole 128-column
 * tiles, spread as evenly as possible (the last ranks may get none). */
HRB_API void hrb_shard_columns(uint32_t N, uint32_t rank, uint32_t ranks, uint32_t* n0,
                               uint32_t* n1);
/* Makes every later run of `plan` also store each output to the peers: for
 * an output byte at address x (C, and the MXINT8 copy when the descriptors
 * ask for one; all in one buffer from local_base), also to
 * peer_bases[i] + (x - local_base).  At most 7 peers; only plans whose GEMMs
 * all take the tensor-core path for MXFP4 or W8 weights
 * (HRB_MODE_FAST, FP32 activations) accept peers (else HRB_ENOTSUP). */
HRB_API hrb_status hrb_plan_set_peers(hrb_plan* plan, const void* local_base,
                                      void* const* peer_bases, uint32_t npeers);

/* ---------------------------------------------------------------------
 * 8. A communicator for hosts without a framework (one process per GPU,
 *    NCCL over NVLink; no counterpart in the reference, whose NPU has no
 *    collective).  It carries what the sharded paths need around their
 *    kernels: the exchange of IPC handles for hrb_plan_set_peers and
 *    hrb_conv_plan_set_peers, a barrier, and an in-place all-gather.  NCCL
 *    is loaded at the first call; without it these return HRB_ENOTSUP and
 *    everything else works.
 * ------------------------------------------------------------------- */

typedef struct hrb_comm hrb_comm;
typedef struct hrb_comm_id {
  uint8_t bytes[128];
} hrb_comm_id;

/* Rank 0 makes the id and hands it to the other ranks by its own means. */
HRB_API hrb_status hrb_comm_id_new(hrb_comm_id* out);
/* Every rank, with the same id and rank count, on the context's device;
 * blocks until all ranks have joined. */
HRB_API hrb_status hrb_comm_create(hrb_ctx* ctx, const hrb_comm_id* id, uint32_t rank,
                                   uint32_t ranks, hrb_comm** out);
HRB_API hrb_status hrb_comm_destroy(hrb_comm* comm);
/* Synchronous: `bytes` of host record `mine` from every rank into host
 * `all` [ranks][bytes], in rank order (e.g. hrb_ipc_handle values). */
HRB_API hrb_status hrb_comm_exchange(hrb_comm* comm, const void* mine, void* all, size_t bytes);
/* Returns once the work queued on every rank's context stream before the
 * call has finished. */
HRB_API hrb_status hrb_comm_barrier(hrb_comm* comm);
/* Asynchronous on `stream` (NULL: the context's): work queued on the
 * stream after the fence starts once every rank's stream has reached its
 * fence (the end of a sharded step whose kernels store into the peers). */
HRB_API hrb_status hrb_comm_fence(hrb_comm* comm, void* stream);
/* In-place all-gather on `stream` (NULL: the context's): rank r has written
 * bytes [offsets[r], offsets[r + 1]) of the device buffer `buf` (offsets:
 * ranks + 1 entries, non-decreasing); afterwards every rank holds all of
 * [offsets[0], offsets[ranks]).  Equal parts take one all-gather, ragged
 * ones a group of broadcasts. */
HRB_API hrb_status hrb_comm_allgather(hrb_comm* comm, void* buf, const uint64_t* offsets,
                                      void* stream);
/* Units (e.g. the images of a convolution batch) of rank `rank` of `ranks`:
 * [u0, u1), as even as possible. */
HRB_API void hrb_shard_rows(uint32_t units, uint32_t rank, uint32_t ranks, uint32_t* u0,
                            uint32_t* u1);

/* ---------------------------------------------------------------------
 * 9. Weights straight from a compiled program: image.bin, the compiler's DDR
 *    image, and meta.json, whose "regions" maps each allocation's name to
 *    [offset, size] (MetaJson, tools/compiler/output.cpp:57-62; LoadProgram,
 *    include/hotarubi/runtime.hpp:44-56).  A Linear's weights are a region of
 *    WBUF words in PackWbuf order (tools/compiler/tensors.cpp:66-90, groups
 *    of 8 columns x kb words of 144 bytes): MXFP4 one region, W8 two,
 *    "<name>_hi" and "<name>_lo" (PlaceW8, smolvla_common.cpp:95-103).
 * ------------------------------------------------------------------- */

typedef struct hrb_image hrb_image;

/* The [offset, size] of region `name` in the text of a meta.json (host
 * only; HRB_EINVAL with a message when it is missing or malformed). */
HRB_API hrb_status hrb_image_region(const char* meta_json, const char* name, uint64_t* offset,
                                    uint64_t* size);
/* Copies image.bin (n host bytes) to the context's device, once. */
HRB_API hrb_status hrb_image_upload(hrb_ctx* ctx, const void* bytes, size_t n, hrb_image** out);
HRB_API hrb_status hrb_image_destroy(hrb_image* image);
/* The device copy of the image. */
HRB_API const void* hrb_image_data(const hrb_image* image);
/* The weights of one Linear from the image, as the dense format of `wfmt`
 * (device buffers w [N][kp(/2)] and wscale [N][kb]): MXFP4 from the region
 * at `offset`, W8 from the HI plane at `offset` and the LO plane at
 * `offset_lo`.  N a multiple of 8, K of 32; MXFP8 has no image format
 * (HRB_ENOTSUP).  Asynchronous on `stream`. */
HRB_API hrb_status hrb_image_weights(hrb_ctx* ctx, const hrb_image* image, uint32_t wfmt,
                                     uint64_t offset, uint64_t offset_lo, uint32_t N,
                                     uint32_t K, uint8_t* w, uint8_t* wscale, void* stream);
/* hrb_gemm_dense with the weights of the region(s) at offset (offset_lo
 * for W8's LO plane) of the image: desc->w and desc->wscale must be NULL.
 * The region becomes dense weights on the device the first time (kept in the
 * image for the calls after); N is rounded up to whole groups of 8 there. */
HRB_API hrb_status hrb_gemm_image(hrb_ctx* ctx, hrb_image* image, const hrb_gemm_desc* desc,
                                  uint64_t offset, uint64_t offset_lo, void* stream);

/* ---------------------------------------------------------------------
 * 10. Activations in the DMA row format, read where a compiled program
 *    keeps them.  An MXINT8 row-format unit holds one token's tok x 32 codes
 *    and then its tok scale bytes, padded to one 16-byte beat (two when
 *    tok > 16): tok * 32 + 16 or + 32 bytes (MakeRowFormat,
 *    tools/iss/dma_engine.cpp:156-183).  A GEMM reads K = planes x tok x 32
 *    values a token, plane p's unit plane_stride bytes after plane 0's, as
 *    the DMA loads one plane per command into its own ABUF range and the
 *    GEMM chains the planes as K pieces of tok blocks.
 *    ROW (LoadRows, :231-262 with kind ROW): token m's unit of plane 0 at
 *    DDR byte address ddr_addr * 16 + (m / row_tokens) * row_stride +
 *    (m % row_tokens) * unit bytes (rows of row_words tokens, ddr_stride
 *    beats apart).  ROW_INDEXED (index != NULL): at index[m] * 16, an index
 *    entry 0xFFFFFFFF being a null unit (codes 0, scale bytes 127).
 * ------------------------------------------------------------------- */

typedef struct hrb_rows {
  const void* window;     /* device copy of DDR bytes [ddr_base, ddr_base + window_bytes),
                             16-byte aligned (e.g. hrb_image_data of an uploaded image) */
  uint64_t ddr_base;      /* DDR byte address of window[0], a multiple of 16 */
  uint64_t window_bytes;
  uint32_t tok;           /* blocks a unit, 1..32 */
  uint32_t planes;        /* units a token; desc->K <= planes * tok * 32 */
  uint64_t plane_stride;  /* bytes, a multiple of 16 */
  uint32_t ddr_addr;      /* ROW: DDR unit address of token 0's unit of plane 0 */
  uint32_t row_tokens;    /* ROW: tokens a row (row_words), a multiple of 4 */
  uint64_t row_stride;    /* ROW: bytes between rows (ddr_stride * 16) */
  const uint32_t* index;  /* ROW_INDEXED: device array [M] of DDR unit addresses, or NULL */
} hrb_rows;

/* hrb_gemm_dense with the activations of `rows` (desc->a, aq and ascale
 * NULL).  desc->pieces NULL: one K piece per plane, the chain the GEMM
 * instructions of a plane-by-plane load give.  HRB_MODE_EXACT gathers the
 * units into dense codes and runs the exact chain (bit-exact with
 * ExecuteGemm over the same loads); HRB_MODE_FAST encodes them straight into
 * the tensor-core operand blocks.  A ROW unit outside the window is
 * HRB_EINVAL at the call; a ROW_INDEXED entry outside it, or (fast mode, W8
 * and MXFP4) a scale byte of 255, is reported by hrb_sync (HRB_EDATA). */
HRB_API hrb_status hrb_gemm_rows(hrb_ctx* ctx, const hrb_gemm_desc* desc, const hrb_rows* rows,
                                 void* stream);

#ifdef __cplusplus
}
#endif

#endif /* HRB_GEMM_H_ */
