/* Test infrastructure only: the CPU restatement ("oracle") of hotarubi's
 * quantized GEMM hot path.  Only tests/, bench.py's CPU-baseline leg and
 * __graft_entry__.smoke() load it, as the checker.  The product library
 * (hotarubi_b200/lib/libhrb_gemm.so) never links or calls it.
 *
 * Every function cites the reference source it restates.  FP32 values travel
 * as their IEEE bit patterns (uint32_t) so that no host FPU rounding mode or
 * flush setting can touch them.
 */
#ifndef HRB_ORACLE_H_
#define HRB_ORACLE_H_

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* Weight modes of the GEMM instruction (include/hotarubi/isa.hpp:88-92), plus
 * MXFP8, which the reference does not have. */
enum {
  HRBO_FP4 = 0,
  HRBO_W8_HI = 1,
  HRBO_W8_LO = 2,
  HRBO_E4M3 = 4
};

/* Scale bias per weight mode: tools/iss/gemm_array.cpp:25-35 for the three
 * reference modes; -15 for E4M3 (activation 2^-6 times E4M3 read as an
 * integer multiple of 2^-9). */
int32_t hrbo_scale_bias(uint32_t mode);

/* FP32 add with the ISS semantics of tools/iss/fp32.hpp:46-75: round to
 * nearest even, subnormal inputs read as zero, subnormal results and exact
 * zeros give +0, overflow gives +-inf, exponent 255 read as an ordinary
 * exponent. */
uint32_t hrbo_fp32_add(uint32_t a, uint32_t b);

/* sum * 2^exponent rounded once to FP32 (nearest even), flushed to +0 below
 * 2^-126 and saturated to +-inf at 2^128.  For |sum| < 2^24 it is the exact
 * BlockValue of tools/iss/gemm_array.cpp:99-110 with
 * exponent = a_scale + w_scale - 254 + SBIAS. */
uint32_t hrbo_round_scaled(int64_t sum, int32_t exponent);

/* BlockValue (tools/iss/gemm_array.cpp:99-110). */
uint32_t hrbo_block_value(int64_t sum, uint32_t a_scale, uint32_t w_scale,
                          uint32_t mode);

/* WeightValue (tools/iss/gemm_array.cpp:84-97): nibble -> small integer. */
int32_t hrbo_weight_value(uint32_t nibble, uint32_t mode);

/* E4M3 byte -> value as an integer multiple of 2^-9 (OCP E4M3; the two NaN
 * codes read as +-480, the ISS-style "no NaN" convention). */
int32_t hrbo_e4m3_units(uint32_t code);

/* GEMM instruction fields (tools/iss/gemm_array.hpp:16-27). */
typedef struct {
  uint32_t a_base, a_stride, kb, m, w_base, w_stride, n8, c_base, wmode, acc;
} hrbo_cmd;

/* 0 when ExecuteGemm would run the command, else 1, 2 or 3 for the three
 * Require checks of tools/iss/gemm_array.cpp:113-119 (m, kb, n8). */
int hrbo_check_command(const hrbo_cmd* cmd);

/* ExecuteGemm (tools/iss/gemm_array.cpp:112-149) over full memories:
 * abuf 8192 x 132 bytes, wbuf 2048 x 144 bytes, fbuf 4096 x 32 FP32 bits.
 * Returns hrbo_check_command's code and leaves fbuf untouched on error. */
int hrbo_execute_gemm(const hrbo_cmd* cmd, const uint8_t* abuf,
                      const uint8_t* wbuf, uint32_t* fbuf);

/* EncodeMxint8 (tools/runtime/formats.cpp:35-56,138-162) on a rows x cols FP32
 * matrix.  q: rows x kp int8 (kp = cols rounded up to 32, padding 0), scale:
 * rows x kp/32 E8M0 bytes (e + 127).  Returns 1 on an Inf/NaN input (the
 * reference's Require), else 0. */
int hrbo_encode_mxint8(const uint32_t* x, uint32_t rows, uint32_t cols,
                       int8_t* q, uint8_t* scale);

/* The VEC 'q' pass of tools/iss/lane.cpp:384-423 on the same layout:
 * subnormal inputs quantize to 0 and an all-zero block gets scale byte 127. */
void hrbo_quantize_vec(const uint32_t* x, uint32_t rows, uint32_t cols,
                       int8_t* q, uint8_t* scale);

/* Weight formats of the dense entry point. */
enum {
  HRBO_WFMT_MXFP4 = 0, /* codes [N][kp/2] nibble pairs, low nibble = even k */
  HRBO_WFMT_W8 = 1,    /* MXINT8 q [N][kp]; run as W8_HI then W8_LO planes */
  HRBO_WFMT_MXFP8 = 2  /* E4M3 [N][kp] */
};

/* The dense GEMM as hotarubi's compiler chains it (LinearEmitter::Emit,
 * tools/compiler/kernels.cpp:343-395): for each K piece in order, for each
 * weight plane in order (W8: HI then LO, kernels.cpp:35-37), one FP32 chain
 * of block values over the piece's blocks; then, when bias is given, one
 * ADDP-style add of bias[n] (tools/compiler/sparsedrive_encoder.cpp:422-428).
 * pieces: npieces block counts summing to kb (NULL: one piece).  c holds
 * M x N FP32 bits; with accumulate != 0 its contents start each chain,
 * otherwise chains start at +0.  Rows [row0, row1) only. */
void hrbo_gemm_dense(uint32_t wfmt, uint32_t M, uint32_t N, uint32_t kb,
                     const int8_t* aq, const uint8_t* ascale,
                     const uint8_t* w, const uint8_t* wscale,
                     const uint32_t* pieces, uint32_t npieces,
                     const uint32_t* bias, uint32_t* c, int accumulate,
                     uint32_t row0, uint32_t row1);

/* Sum of |block value| over the chain of one output, in double: the scale
 * the tolerance of the tensor-core path is stated against. */
double hrbo_abs_chain(uint32_t wfmt, uint32_t N, uint32_t kb,
                      const int8_t* aq_row, const uint8_t* ascale_row,
                      const uint8_t* w, const uint8_t* wscale, uint32_t n);

/* AlignElement (tools/iss/dma_engine.cpp:532-544): the int8 code `value`
 * divided by 2^shift, rounded to nearest, ties to even, as an int8 bit
 * pattern; 0 when shift >= 9. */
uint8_t hrbo_align_element(uint8_t value, uint32_t shift);

/* T32_SPLIT8 in dense form (LoadT32 + TransposeGroup, dma_engine.cpp:336-405):
 * the V cache, MXINT8 codes vq [tokens][ldv] with one scale byte per token and
 * 32-dim block (vs [tokens][ldv/32]), becomes the W8 weight operand of P.V:
 * wq [hd][tokens] codes, ws [hd][tokens/32] scales.  For each 32-token x
 * 32-dim block, emax = the largest scale of the tokens whose 32 codes are not
 * all zero (127 when none is), every such token's codes are aligned to emax
 * with hrbo_align_element(code, emax - scale), all-zero tokens stay 0, and
 * all 32 dims take scale emax.  tokens and hd are multiples of 32, ldv >= hd
 * a multiple of 32.  Returns 0, or -1 on a bad shape. */
int hrbo_t32_split8(const int8_t* vq, const uint8_t* vs, uint32_t tokens,
                    uint32_t hd, uint32_t ldv, int8_t* wq, uint8_t* ws);

/* Convolution as hotarubi's compiler lowers it (ConvEmitter,
 * tools/compiler/sparsedrive_encoder.cpp): one GEMM per (channel plane,
 * tap), all chaining into the same outputs, on activations gathered per tap
 * (faces, :114-168) where a position outside the map is a zero token with
 * scale byte 127 (the DMA engine's null entry, tools/iss/dma_engine.cpp:
 * 247-256).  Geometry: `images` maps of H x W positions and cin channels;
 * kh 1 or 3 (padding (kh-1)/2), stride 1 or 2; Ho = H / stride,
 * Wo = W / stride.  Positions are x-major (order 0: position x*H + y, the
 * compiler's FMap order) or y-major (order 1: y*W + x); outputs use the
 * same order.  Channel planes are 256 channels (all cin when cin <= 256;
 * MakeMap, tools/compiler/sparsedrive_common.cpp:47-68).
 *
 * hrbo_conv_im2col writes the gathered activations in chain order: row
 * img*Ho*Wo + o, columns (plane, tap = ky*kh + kx, channel in plane):
 * aq' [M][kh*kh*cin] and scales [M][kh*kh*cin/32], from the MXINT8 map aq
 * [images][H*W][cin] + ascale [images][H*W][cin/32]. */
int hrbo_conv_im2col(uint32_t images, uint32_t H, uint32_t W, uint32_t cin,
                     uint32_t kh, uint32_t stride, uint32_t order,
                     const int8_t* aq, const uint8_t* ascale,
                     int8_t* out_q, uint8_t* out_scale);

/* The conv weight matrix [cout][kh*kh*cin] (tap-major columns, ConvTile,
 * sparsedrive_common.cpp:136-158) reordered to the chain order of
 * hrbo_conv_im2col: `bytes_per_block` is 16 (MXFP4) or 32 (W8, MXFP8). */
void hrbo_conv_weights(uint32_t cout, uint32_t cin, uint32_t kh,
                       uint32_t bytes_per_block, const uint8_t* w,
                       const uint8_t* wscale, uint8_t* out_w,
                       uint8_t* out_scale);

/* The VEC RELU pass (post op kMax against +0, tools/iss/lane.cpp:57-70,
 * 322-326): x if x is not negative, else +0, then + 0 through the FP32
 * adder.  In place over n FP32 bit patterns. */
void hrbo_relu_n(uint32_t* x, size_t n);

/* The ISS's FP32 multiply (tools/iss/fp32.hpp:77-92): +0 when an operand's
 * exponent field is 0, else the 48-bit product rounded to 24 bits nearest
 * even, +0 below the normal range, +-inf above it (exponent field 255 reads
 * as an ordinary exponent). */
uint32_t hrbo_fp32_mul(uint32_t a, uint32_t b);

/* Int8ToFp32 (tools/iss/dma_engine.cpp:504-514): the int8 code as FP32. */
uint32_t hrbo_int8_to_fp32(uint8_t value);

/* ScaleCoefficient (dma_engine.cpp:516-528): coefficient * 2^(scale - 133)
 * by exponent arithmetic: +0 for a zero coefficient or an exponent <= 0,
 * +-0x7F7FFFFF (the largest finite) from exponent 255 up. */
uint32_t hrbo_scale_coefficient(uint32_t coefficient, uint32_t scale);

/* GACC, the DMA engine's gather-accumulate (DmaEngine::Gather,
 * dma_engine.cpp:599-652, AccumulateGatherBlock :478-488), in dense form.
 * For each output token t, the chain over slots s, then corners k, of entry
 * e = entries[t][s][k] (low 32 bits: feature row index, 0xFFFFFFFF = null
 * entry, skipped; high 32 bits: the FP32 bits of its bilinear weight bw):
 *   coef_b = ScaleCoefficient(Fp32Mul(w[t][s][b], bw), scale byte b of the row)
 *   out[t][32b + v] = Fp32Add(out[t][32b + v],
 *                             Fp32Mul(Int8ToFp32(code 32b + v of the row), coef_b))
 * A feature row is `blocks` 32-byte code blocks then `blocks` scale bytes,
 * rows row_stride bytes apart.  w: FP32 bits [tokens][slots][blocks]; out:
 * FP32 bits [tokens][blocks * 32], starting from its contents when
 * accumulate != 0, else from +0. */
void hrbo_gacc_dense(uint32_t tokens, uint32_t slots, uint32_t corners,
                     uint32_t blocks, const uint64_t* entries,
                     const uint32_t* w, const uint8_t* rows,
                     uint64_t row_stride, uint32_t* out, int accumulate);

/* Element-wise array forms of hrbo_fp32_add, hrbo_fp32_mul and
 * hrbo_round_scaled. */
void hrbo_fp32_add_n(const uint32_t* a, const uint32_t* b, uint32_t* out,
                     size_t n);
void hrbo_fp32_mul_n(const uint32_t* a, const uint32_t* b, uint32_t* out,
                     size_t n);
void hrbo_round_scaled_n(const int64_t* sum, const int32_t* exponent,
                         uint32_t* out, size_t n);

#ifdef __cplusplus
}
#endif

#endif /* HRB_ORACLE_H_ */
