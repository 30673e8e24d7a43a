/* Test infrastructure only: CPU restatement of hotarubi's quantized GEMM
 * (the checker for the CUDA path).  See hrb_oracle.h for the contract of each
 * function and the reference lines it follows.  Nothing in the product links
 * this file.
 *
 * Parity pin: tests/test_oracle.py checks every function here against the
 * reference's own sources built into oracle/_ref/ (when present) and against
 * the committed golden fixtures in tests/golden/, which that build produced.
 */
#include "hrb_oracle.h"

#include <string.h>

#define ABUF_DEPTH 8192u
#define WBUF_DEPTH 2048u
#define FBUF_DEPTH 4096u
#define ABUF_WORD 132u
#define WBUF_WORD 144u
#define ADDRESS_MASK 0xFFFFFu

static uint32_t field_of(uint32_t bits) { return (bits >> 23) & 0xFFu; }

/* Significand with the hidden bit; 0 for zeros and subnormals
 * (tools/iss/fp32.hpp:20-22). */
static uint32_t sig_of(uint32_t bits) {
  return field_of(bits) == 0 ? 0u : ((bits & 0x7FFFFFu) | 0x800000u);
}

static int msb64(uint64_t v) { return 63 - __builtin_clzll(v); }

/* Round magnitude * 2^scale (magnitude != 0) to a 24-bit significand, nearest
 * even, then pack: biased exponent <= 0 gives +0, >= 255 gives +-inf
 * (tools/iss/fp32.hpp:24-44). */
static uint32_t round_pack(uint32_t sign, uint64_t magnitude, int32_t scale) {
  int top = msb64(magnitude);
  uint64_t kept;
  if (top > 23) {
    const int drop = top - 23;
    kept = magnitude >> drop;
    const uint64_t rest = magnitude & ((1ull << drop) - 1u);
    const uint64_t half = 1ull << (drop - 1);
    if (rest > half || (rest == half && (kept & 1u) != 0)) {
      ++kept;
      if (kept == (1ull << 24)) {
        kept >>= 1;
        ++top;
      }
    }
  } else {
    kept = magnitude << (23 - top);
  }
  const int32_t biased = scale + top + 127;
  if (biased <= 0) return 0u;
  if (biased >= 255) return (sign << 31) | 0x7F800000u;
  return (sign << 31) | ((uint32_t)biased << 23) | ((uint32_t)kept & 0x7FFFFFu);
}

uint32_t hrbo_fp32_add(uint32_t a, uint32_t b) {
  /* The larger operand by (exponent field, significand), as in
   * tools/iss/fp32.hpp:46-57, keeps its sign. */
  uint32_t ea = field_of(a), eb = field_of(b);
  uint32_t ma = sig_of(a), mb = sig_of(b);
  if (((ea << 24) | ma) < ((eb << 24) | mb)) {
    uint32_t t = a; a = b; b = t;
    t = ea; ea = eb; eb = t;
    t = ma; ma = mb; mb = t;
  }
  /* Exact alignment over 38 extra bits; anything further right only matters
   * as a sticky bit. */
  const uint64_t big = (uint64_t)ma << 38;
  const uint32_t distance = ea - eb;
  uint64_t small = 0;
  if (mb != 0) {
    if (distance <= 38) {
      small = (uint64_t)mb << (38 - distance);
    } else {
      small = 1;
    }
  }
  const int subtract = ((a ^ b) >> 31) != 0;
  const uint64_t total = subtract ? big - small : big + small;
  if (total == 0) return 0u;
  /* value = total * 2^(ea - 150 - 38) */
  return round_pack(a >> 31, total, (int32_t)ea - 150 - 38);
}

uint32_t hrbo_round_scaled(int64_t sum, int32_t exponent) {
  if (sum == 0) return 0u;
  const uint32_t sign = sum < 0 ? 1u : 0u;
  const uint64_t magnitude = sum < 0 ? (uint64_t)(-sum) : (uint64_t)sum;
  return round_pack(sign, magnitude, exponent);
}

int32_t hrbo_scale_bias(uint32_t mode) {
  switch (mode) {
    case HRBO_FP4: return -7;
    case HRBO_W8_HI: return -8;
    case HRBO_E4M3: return -15;
    default: return -12; /* W8_LO (wmode 2 and 3) */
  }
}

uint32_t hrbo_block_value(int64_t sum, uint32_t a_scale, uint32_t w_scale,
                          uint32_t mode) {
  return hrbo_round_scaled(
      sum, (int32_t)a_scale + (int32_t)w_scale - 254 + hrbo_scale_bias(mode));
}

/* E2M1 magnitude times two, indexed by the low three bits of the code
 * (tools/iss/gemm_array.cpp:18). */
static const int32_t kFp4Twice[8] = {0, 1, 2, 3, 4, 6, 8, 12};

int32_t hrbo_weight_value(uint32_t nibble, uint32_t mode) {
  nibble &= 0xFu;
  switch (mode & 3u) {
    case HRBO_FP4: {
      const int32_t m = kFp4Twice[nibble & 7u];
      return (nibble & 8u) ? -m : m;
    }
    case HRBO_W8_HI:
      return (nibble & 8u) ? (int32_t)nibble - 16 : (int32_t)nibble;
    default:
      return (int32_t)nibble;
  }
}

int32_t hrbo_e4m3_units(uint32_t code) {
  const uint32_t e = (code >> 3) & 0xFu;
  const uint32_t m = code & 7u;
  const int32_t mag = e == 0 ? (int32_t)m : (int32_t)((8u + m) << (e - 1u));
  return (code & 0x80u) ? -mag : mag;
}

int hrbo_check_command(const hrbo_cmd* c) {
  if (!(c->m >= 32 && c->m <= 992 && c->m % 32 == 0)) return 1;
  if (!(c->kb >= 1 && c->kb <= c->a_stride)) return 2;
  if (c->n8 < 1) return 3;
  return 0;
}

int hrbo_execute_gemm(const hrbo_cmd* cmd, const uint8_t* abuf,
                      const uint8_t* wbuf, uint32_t* fbuf) {
  const int status = hrbo_check_command(cmd);
  if (status != 0) return status;
  const uint32_t mode = cmd->wmode & 3u;
  const uint32_t quads = cmd->m / 4;
  for (uint32_t g = 0; g < cmd->n8; ++g) {
    for (uint32_t q = 0; q < quads; ++q) {
      const uint32_t c_addr =
          ((cmd->c_base + q * cmd->n8 + g) & ADDRESS_MASK) % FBUF_DEPTH;
      uint32_t acc[32];
      for (int e = 0; e < 32; ++e) acc[e] = cmd->acc ? fbuf[c_addr * 32 + e] : 0u;
      for (uint32_t b = 0; b < cmd->kb; ++b) {
        const uint32_t a_addr =
            ((cmd->a_base + q * cmd->a_stride + b) & ADDRESS_MASK) % ABUF_DEPTH;
        const uint32_t w_addr =
            ((cmd->w_base + g * cmd->w_stride + b) & ADDRESS_MASK) % WBUF_DEPTH;
        const uint8_t* aw = abuf + (size_t)a_addr * ABUF_WORD;
        const uint8_t* ww = wbuf + (size_t)w_addr * WBUF_WORD;
        for (uint32_t t = 0; t < 4; ++t) {
          for (uint32_t c = 0; c < 8; ++c) {
            int32_t sum = 0;
            for (uint32_t k = 0; k < 32; ++k) {
              const uint32_t idx = c * 32 + k;
              const uint32_t nib = (ww[idx / 2] >> ((idx & 1u) * 4)) & 0xFu;
              sum += (int32_t)(int8_t)aw[t * 32 + k] * hrbo_weight_value(nib, mode);
            }
            const uint32_t bv =
                hrbo_block_value(sum, aw[128 + t], ww[128 + c], mode);
            acc[t * 8 + c] = hrbo_fp32_add(acc[t * 8 + c], bv);
          }
        }
      }
      memcpy(fbuf + (size_t)c_addr * 32, acc, sizeof(acc));
    }
  }
  return 0;
}

/* QuantizeInt8 (tools/runtime/formats.cpp:35-56): x * 2^(6 - e), nearest
 * even, clamped to [-128, 127]. */
static int8_t quantize_host(uint32_t bits, int32_t e) {
  const uint32_t f = field_of(bits);
  const uint64_t significand = f == 0 ? (bits & 0x7FFFFFu) : ((bits & 0x7FFFFFu) | 0x800000u);
  const int64_t shift = (f == 0 ? -149 : (int64_t)f - 150) + 6 - e;
  int64_t magnitude = 0;
  if (shift >= 0) {
    magnitude = shift > 8 ? 256 : (int64_t)(significand << shift);
  } else if (shift > -64) {
    const uint64_t kept = significand >> (-shift);
    const uint64_t rest = significand & ((1ull << (-shift)) - 1u);
    const uint64_t half = 1ull << (-shift - 1);
    magnitude = (int64_t)kept + ((rest > half || (rest == half && (kept & 1u))) ? 1 : 0);
  }
  int64_t v = (bits >> 31) ? -magnitude : magnitude;
  if (v < -128) v = -128;
  if (v > 127) v = 127;
  return (int8_t)v;
}

int hrbo_encode_mxint8(const uint32_t* x, uint32_t rows, uint32_t cols,
                       int8_t* q, uint8_t* scale) {
  const uint32_t kp = (cols + 31u) / 32u * 32u;
  const uint32_t blocks = kp / 32u;
  int bad = 0;
  for (uint32_t r = 0; r < rows; ++r) {
    for (uint32_t b = 0; b < blocks; ++b) {
      const uint32_t end = cols < (b + 1u) * 32u ? cols : (b + 1u) * 32u;
      uint32_t amax = 0;
      for (uint32_t c = b * 32u; c < end; ++c) {
        const uint32_t m = x[(size_t)r * cols + c] & 0x7FFFFFFFu;
        if (field_of(m) == 0xFFu) bad = 1;
        if (m > amax) amax = m;
      }
      const int32_t e = amax != 0 ? (int32_t)field_of(amax) - 127 : 0;
      scale[(size_t)r * blocks + b] = (uint8_t)(e + 127);
      for (uint32_t c = b * 32u; c < (b + 1u) * 32u; ++c) {
        q[(size_t)r * kp + c] = c < end ? quantize_host(x[(size_t)r * cols + c], e) : 0;
      }
    }
  }
  return bad;
}

/* QuantizeElement (tools/iss/lane.cpp:384-403). */
static int8_t quantize_vec_element(uint32_t bits, uint32_t emax) {
  const uint32_t f = field_of(bits);
  const uint32_t s = sig_of(bits);
  if (s == 0) return 0;
  const uint32_t shift = emax - f + 17u;
  uint32_t magnitude = 0;
  if (shift < 25u) {
    const uint32_t whole = s >> shift;
    const uint32_t guard = (s >> (shift - 1u)) & 1u;
    const uint32_t sticky = (s & ((1u << (shift - 1u)) - 1u)) != 0;
    magnitude = whole + ((guard && (sticky || (whole & 1u))) ? 1u : 0u);
  }
  if (bits >> 31) return magnitude >= 128u ? (int8_t)-128 : (int8_t)(-(int32_t)magnitude);
  return magnitude >= 128u ? (int8_t)127 : (int8_t)magnitude;
}

void hrbo_quantize_vec(const uint32_t* x, uint32_t rows, uint32_t cols,
                       int8_t* q, uint8_t* scale) {
  const uint32_t kp = (cols + 31u) / 32u * 32u;
  const uint32_t blocks = kp / 32u;
  for (uint32_t r = 0; r < rows; ++r) {
    for (uint32_t b = 0; b < blocks; ++b) {
      const uint32_t end = cols < (b + 1u) * 32u ? cols : (b + 1u) * 32u;
      uint32_t emax = 0;
      for (uint32_t c = b * 32u; c < end; ++c) {
        const uint32_t f = field_of(x[(size_t)r * cols + c]);
        if (f > emax) emax = f;
      }
      scale[(size_t)r * blocks + b] = (uint8_t)(emax == 0 ? 127u : emax);
      for (uint32_t c = b * 32u; c < (b + 1u) * 32u; ++c) {
        q[(size_t)r * kp + c] =
            c < end ? quantize_vec_element(x[(size_t)r * cols + c], emax) : 0;
      }
    }
  }
}

/* Integer weights of one (column, block) for one plane, plus its mode. */
static uint32_t load_block(uint32_t wfmt, uint32_t plane, uint32_t kb,
                           const uint8_t* w, uint32_t n, uint32_t b,
                           int32_t out[32]) {
  const size_t kp = (size_t)kb * 32u;
  if (wfmt == HRBO_WFMT_MXFP4) {
    const uint8_t* row = w + (size_t)n * (kp / 2) + (size_t)b * 16u;
    for (uint32_t k = 0; k < 32; ++k) {
      out[k] = hrbo_weight_value((row[k / 2] >> ((k & 1u) * 4)) & 0xFu, HRBO_FP4);
    }
    return HRBO_FP4;
  }
  const uint8_t* row = w + (size_t)n * kp + (size_t)b * 32u;
  if (wfmt == HRBO_WFMT_W8) {
    /* SplitW8 (tools/compiler/weights.cpp:72-88): HI = byte >> 4 read as a
     * signed nibble, LO = byte & 15. */
    for (uint32_t k = 0; k < 32; ++k) {
      out[k] = plane == 0 ? hrbo_weight_value(row[k] >> 4, HRBO_W8_HI)
                          : hrbo_weight_value(row[k] & 0xFu, HRBO_W8_LO);
    }
    return plane == 0 ? HRBO_W8_HI : HRBO_W8_LO;
  }
  for (uint32_t k = 0; k < 32; ++k) out[k] = hrbo_e4m3_units(row[k]);
  return HRBO_E4M3;
}

static uint32_t block_product(uint32_t wfmt, uint32_t plane, uint32_t kb,
                              const int8_t* aq_row, const uint8_t* ascale_row,
                              const uint8_t* w, const uint8_t* wscale,
                              uint32_t n, uint32_t b) {
  int32_t wv[32];
  const uint32_t mode = load_block(wfmt, plane, kb, w, n, b, wv);
  int64_t sum = 0;
  for (uint32_t k = 0; k < 32; ++k) sum += (int64_t)aq_row[b * 32u + k] * wv[k];
  return hrbo_block_value(sum, ascale_row[b], wscale[(size_t)n * kb + b], mode);
}

void hrbo_gemm_dense(uint32_t wfmt, uint32_t M, uint32_t N, uint32_t kb,
                     const int8_t* aq, const uint8_t* ascale,
                     const uint8_t* w, const uint8_t* wscale,
                     const uint32_t* pieces, uint32_t npieces,
                     const uint32_t* bias, uint32_t* c, int accumulate,
                     uint32_t row0, uint32_t row1) {
  const uint32_t planes = wfmt == HRBO_WFMT_W8 ? 2u : 1u;
  const uint32_t one_piece = kb;
  if (pieces == NULL || npieces == 0) {
    pieces = &one_piece;
    npieces = 1;
  }
  if (row1 > M) row1 = M;
  for (uint32_t m = row0; m < row1; ++m) {
    const int8_t* arow = aq + (size_t)m * kb * 32u;
    const uint8_t* srow = ascale + (size_t)m * kb;
    for (uint32_t n = 0; n < N; ++n) {
      uint32_t acc = accumulate ? c[(size_t)m * N + n] : 0u;
      uint32_t first = 0;
      for (uint32_t p = 0; p < npieces; ++p) {
        for (uint32_t l = 0; l < planes; ++l) {
          for (uint32_t b = first; b < first + pieces[p]; ++b) {
            acc = hrbo_fp32_add(
                acc, block_product(wfmt, l, kb, arow, srow, w, wscale, n, b));
          }
        }
        first += pieces[p];
      }
      if (bias != NULL) acc = hrbo_fp32_add(acc, bias[n]);
      c[(size_t)m * N + n] = acc;
    }
  }
}

static double bits_to_double(uint32_t bits) {
  if (field_of(bits) == 0) return 0.0;
  double v = (double)sig_of(bits);
  int e = (int)field_of(bits) - 150;
  while (e > 0) { v *= 2.0; --e; }
  while (e < 0) { v *= 0.5; ++e; }
  return (bits >> 31) ? -v : v;
}

double hrbo_abs_chain(uint32_t wfmt, uint32_t N, uint32_t kb,
                      const int8_t* aq_row, const uint8_t* ascale_row,
                      const uint8_t* w, const uint8_t* wscale, uint32_t n) {
  (void)N;
  const uint32_t planes = wfmt == HRBO_WFMT_W8 ? 2u : 1u;
  double total = 0.0;
  for (uint32_t l = 0; l < planes; ++l) {
    for (uint32_t b = 0; b < kb; ++b) {
      const double v = bits_to_double(
          block_product(wfmt, l, kb, aq_row, ascale_row, w, wscale, n, b));
      total += v < 0 ? -v : v;
    }
  }
  return total;
}

void hrbo_fp32_add_n(const uint32_t* a, const uint32_t* b, uint32_t* out,
                     size_t n) {
  for (size_t i = 0; i < n; ++i) out[i] = hrbo_fp32_add(a[i], b[i]);
}

void hrbo_fp32_mul_n(const uint32_t* a, const uint32_t* b, uint32_t* out,
                     size_t n) {
  for (size_t i = 0; i < n; ++i) out[i] = hrbo_fp32_mul(a[i], b[i]);
}

void hrbo_round_scaled_n(const int64_t* sum, const int32_t* exponent,
                         uint32_t* out, size_t n) {
  for (size_t i = 0; i < n; ++i) out[i] = hrbo_round_scaled(sum[i], exponent[i]);
}

uint8_t hrbo_align_element(uint8_t value, uint32_t shift) {
  /* dma_engine.cpp:532-544: scale the code by 2^8, shift right arithmetically
   * (the low 8 bits then hold the discarded fraction), round the integer part
   * to nearest even on the guard bit (bit 7) and the sticky bits (6..0). */
  if (shift >= 9) return 0;
  const int32_t shifted = ((int32_t)(int8_t)value * 256) >> shift;
  const int guard = (shifted >> 7) & 1;
  const int sticky = (shifted & 0x7F) != 0;
  const int odd = (shifted >> 8) & 1;
  return (uint8_t)(((shifted >> 8) + (guard && (sticky || odd) ? 1 : 0)) & 0xFF);
}

int hrbo_t32_split8(const int8_t* vq, const uint8_t* vs, uint32_t tokens,
                    uint32_t hd, uint32_t ldv, int8_t* wq, uint8_t* ws) {
  if (tokens % 32u != 0 || hd % 32u != 0 || ldv % 32u != 0 || ldv < hd) return -1;
  const uint32_t lds = ldv / 32u, kbt = tokens / 32u;
  for (uint32_t tb = 0; tb < kbt; ++tb) {
    for (uint32_t db = 0; db < hd / 32u; ++db) {
      /* TransposeGroup, dma_engine.cpp:338-356: emax over nonzero tokens. */
      int nonzero[32];
      uint32_t scale[32], emax = 0;
      int any = 0;
      for (uint32_t t = 0; t < 32; ++t) {
        const size_t row = (size_t)(tb * 32u + t);
        nonzero[t] = 0;
        for (uint32_t d = 0; d < 32; ++d) nonzero[t] |= vq[row * ldv + db * 32u + d] != 0;
        scale[t] = vs[row * lds + db];
        if (nonzero[t]) {
          any = 1;
          if (scale[t] > emax) emax = scale[t];
        }
      }
      if (!any) emax = 127;
      /* dma_engine.cpp:357-377: aligned codes, transposed; one scale per lane. */
      for (uint32_t d = 0; d < 32; ++d) {
        const size_t n = (size_t)(db * 32u + d);
        for (uint32_t t = 0; t < 32; ++t) {
          const size_t row = (size_t)(tb * 32u + t);
          wq[n * tokens + tb * 32u + t] =
              nonzero[t] ? (int8_t)hrbo_align_element((uint8_t)vq[row * ldv + db * 32u + d],
                                                      emax - scale[t])
                         : 0;
        }
        ws[n * kbt + tb] = (uint8_t)emax;
      }
    }
  }
  return 0;
}

/* Source position of output o's tap (ky, kx), or -1 outside the map:
 * FaceListS1 / FaceListStrided (sparsedrive_encoder.cpp:114-150) with
 * padding (kh-1)/2. */
static int64_t conv_source(uint32_t H, uint32_t W, uint32_t kh, uint32_t stride,
                           uint32_t order, uint32_t o, uint32_t ky, uint32_t kx) {
  const uint32_t Ho = H / stride, Wo = W / stride;
  const uint32_t yo = order == 0 ? o % Ho : o / Wo;
  const uint32_t xo = order == 0 ? o / Ho : o % Wo;
  const int64_t pad = (int64_t)(kh - 1u) / 2;
  const int64_t yi = (int64_t)stride * yo + ky - pad;
  const int64_t xi = (int64_t)stride * xo + kx - pad;
  if (yi < 0 || yi >= H || xi < 0 || xi >= W) return -1;
  return order == 0 ? xi * H + yi : yi * W + xi;
}

int hrbo_conv_im2col(uint32_t images, uint32_t H, uint32_t W, uint32_t cin,
                     uint32_t kh, uint32_t stride, uint32_t order,
                     const int8_t* aq, const uint8_t* ascale,
                     int8_t* out_q, uint8_t* out_scale) {
  if ((kh != 1 && kh != 3) || (stride != 1 && stride != 2) || cin % 32u != 0 ||
      (cin > 256u && cin % 256u != 0) || H / stride == 0 || W / stride == 0) {
    return -1;
  }
  const uint32_t taps = kh * kh, plane = cin < 256u ? cin : 256u, planes = cin / plane;
  const uint32_t kbi = cin / 32u, kbo = taps * kbi, out_per = (H / stride) * (W / stride);
  for (uint32_t img = 0; img < images; ++img) {
    for (uint32_t o = 0; o < out_per; ++o) {
      const size_t row = (size_t)img * out_per + o;
      uint32_t b = 0;
      for (uint32_t p = 0; p < planes; ++p) {
        for (uint32_t t = 0; t < taps; ++t) {
          const int64_t src = conv_source(H, W, kh, stride, order, o, t / kh, t % kh);
          for (uint32_t cb = 0; cb < plane / 32u; ++cb, ++b) {
            const uint32_t ib = p * (plane / 32u) + cb;
            const size_t pos = (size_t)img * H * W + (size_t)(src < 0 ? 0 : src);
            for (uint32_t k = 0; k < 32; ++k) {
              out_q[row * kbo * 32u + (size_t)b * 32u + k] =
                  src < 0 ? 0 : aq[pos * cin + ib * 32u + k];
            }
            /* A null entry's token carries scale byte 127 (kNullScale). */
            out_scale[row * kbo + b] = src < 0 ? 127 : ascale[pos * kbi + ib];
          }
        }
      }
    }
  }
  return 0;
}

void hrbo_conv_weights(uint32_t cout, uint32_t cin, uint32_t kh,
                       uint32_t bytes_per_block, const uint8_t* w,
                       const uint8_t* wscale, uint8_t* out_w,
                       uint8_t* out_scale) {
  const uint32_t taps = kh * kh, plane = cin < 256u ? cin : 256u, planes = cin / plane;
  const uint32_t kbi = cin / 32u, kbo = taps * kbi;
  for (uint32_t n = 0; n < cout; ++n) {
    uint32_t b = 0;
    for (uint32_t p = 0; p < planes; ++p) {
      for (uint32_t t = 0; t < taps; ++t) {
        for (uint32_t cb = 0; cb < plane / 32u; ++cb, ++b) {
          const uint32_t src = t * kbi + p * (plane / 32u) + cb;
          for (uint32_t i = 0; i < bytes_per_block; ++i) {
            out_w[((size_t)n * kbo + b) * bytes_per_block + i] =
                w[((size_t)n * kbo + src) * bytes_per_block + i];
          }
          out_scale[(size_t)n * kbo + b] = wscale[(size_t)n * kbo + src];
        }
      }
    }
  }
}

void hrbo_relu_n(uint32_t* x, size_t n) {
  /* MaxGreaterEqual(x, +0) (lane.cpp:57-70) keeps x unless x is negative
   * with a nonzero magnitude; the pass then adds +0 (lane.cpp:325). */
  for (size_t i = 0; i < n; ++i) {
    const uint32_t keep = (x[i] >> 31) == 0 || (x[i] & 0x7FFFFFFFu) == 0;
    x[i] = hrbo_fp32_add(keep ? x[i] : 0u, 0u);
  }
}

uint32_t hrbo_fp32_mul(uint32_t a, uint32_t b) {
  /* fp32.hpp:77-92: the exact product of the significands, rounded once. */
  if (field_of(a) == 0 || field_of(b) == 0) return 0u;
  const uint64_t product = (uint64_t)sig_of(a) * sig_of(b);
  return round_pack((a ^ b) >> 31, product,
                    (int32_t)field_of(a) + (int32_t)field_of(b) - 300);
}

uint32_t hrbo_int8_to_fp32(uint8_t value) {
  /* dma_engine.cpp:504-514: exact (|value| <= 128 has at most 8 bits). */
  if (value == 0) return 0u;
  const uint32_t negative = value >= 128;
  const uint32_t magnitude = negative ? 256u - value : value;
  const int top = 31 - __builtin_clz(magnitude);
  return (negative << 31) | ((uint32_t)(127 + top) << 23) |
         ((magnitude << (23 - top)) & 0x7FFFFFu);
}

uint32_t hrbo_scale_coefficient(uint32_t coefficient, uint32_t scale) {
  /* dma_engine.cpp:516-528. */
  const int32_t exponent = (int32_t)(field_of(coefficient) + scale) - 133;
  if (field_of(coefficient) == 0 || exponent <= 0) return 0u;
  const uint32_t sign = coefficient & 0x80000000u;
  if (exponent >= 255) return sign | 0x7F7FFFFFu;
  return sign | ((uint32_t)exponent << 23) | (coefficient & 0x7FFFFFu);
}

void hrbo_gacc_dense(uint32_t tokens, uint32_t slots, uint32_t corners,
                     uint32_t blocks, const uint64_t* entries,
                     const uint32_t* w, const uint8_t* rows,
                     uint64_t row_stride, uint32_t* out, int accumulate) {
  const uint32_t channels = blocks * 32u;
  for (uint32_t t = 0; t < tokens; ++t) {
    uint32_t* acc = out + (size_t)t * channels;
    if (!accumulate) {
      for (uint32_t c = 0; c < channels; ++c) acc[c] = 0u;
    }
    /* DmaEngine::Gather (dma_engine.cpp:619-650): slots, then corners; null
     * entries contribute nothing. */
    for (uint32_t s = 0; s < slots; ++s) {
      for (uint32_t k = 0; k < corners; ++k) {
        const uint64_t e = entries[((size_t)t * slots + s) * corners + k];
        const uint32_t index = (uint32_t)e;
        if (index == 0xFFFFFFFFu) continue;
        const uint32_t bw = (uint32_t)(e >> 32);
        const uint8_t* row = rows + (uint64_t)index * row_stride;
        for (uint32_t b = 0; b < blocks; ++b) {
          /* AccumulateGatherBlock (dma_engine.cpp:478-488). */
          const uint32_t coef = hrbo_scale_coefficient(
              hrbo_fp32_mul(w[((size_t)t * slots + s) * blocks + b], bw), row[channels + b]);
          for (uint32_t v = 0; v < 32u; ++v) {
            const uint32_t c = b * 32u + v;
            acc[c] = hrbo_fp32_add(acc[c], hrbo_fp32_mul(hrbo_int8_to_fp32(row[c]), coef));
          }
        }
      }
    }
  }
}
