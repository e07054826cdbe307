/*
 * objeta_oracle.c -- TEST INFRASTRUCTURE ONLY (see objeta_oracle.h).
 *
 * CPU restatement of the reference arithmetic.  Citations are to the objeta
 * repository: crates/objeta-cuda/src/quant.rs (quant.rs),
 * crates/objeta-cuda/src/moe.rs (moe.rs),
 * crates/objeta-parser/src/deepseek.rs (deepseek.rs) and
 * crates/objeta-cuda/src/bin/deepseek_single_layer_moe.rs (dsl_moe.rs).
 */
#include "objeta_oracle.h"

#include <math.h>
#include <pthread.h>
#include <stdlib.h>
#include <string.h>
#include <unistd.h>

static float bits_to_f32(uint32_t b) {
  float f;
  memcpy(&f, &b, 4);
  return f;
}
static uint32_t f32_to_bits(float f) {
  uint32_t b;
  memcpy(&b, &f, 4);
  return b;
}

/* Rust `f32::max`: NaN operands are ignored (IEEE maxNum), as fmaxf. */
static float rs_max(float a, float b) { return fmaxf(a, b); }

/* Rust `f32 as u8` after clamp: saturating, NaN -> 0. */
static uint8_t rs_as_u8(float v) {
  if (v != v) return 0;
  if (v <= 0.0f) return 0;
  if (v >= 255.0f) return 255;
  return (uint8_t)v;
}

/* Rust `f32::clamp(lo, hi)`: NaN stays NaN. */
static float rs_clamp(float v, float lo, float hi) {
  if (v < lo) v = lo;
  if (v > hi) v = hi;
  return v;
}

size_t oro_block_bytes(int fmt) {
  /* QuantFormat::block_bytes, quant.rs:43-50 */
  switch (fmt) {
    case ORO_Q4_0: return 18;
    case ORO_Q5_0: return 22;
    case ORO_IQ3_0: return 14;
    case ORO_FP4_E2M1: return 17;
    default: return 0;
  }
}

/* quant.rs:1046-1079 (f32_to_f16_bits): truncating encode that adds one
 * when mantissa bit 12 is set (round half up on magnitude, not RNE). */
uint16_t oro_f32_to_f16_bits(float value) {
  uint32_t bits = f32_to_bits(value);
  uint16_t sign = (uint16_t)((bits >> 16) & 0x8000u);
  int32_t exp = (int32_t)((bits >> 23) & 0xFFu);
  uint32_t mant = bits & 0x7FFFFFu;
  if (exp == 255) {
    uint16_t nan_bits = mant == 0 ? 0 : 0x0200;
    return (uint16_t)(sign | 0x7C00u | nan_bits);
  }
  int32_t half_exp = exp - 127 + 15;
  if (half_exp >= 0x1F) return (uint16_t)(sign | 0x7C00u);
  if (half_exp <= 0) {
    if (half_exp < -10) return sign;
    uint32_t mantissa = mant | 0x800000u;
    uint32_t shift = (uint32_t)(14 - half_exp);
    uint16_t half = (uint16_t)(mantissa >> shift);
    if ((mantissa >> (shift - 1)) & 1u) half = (uint16_t)(half + 1);
    return (uint16_t)(sign | half);
  }
  uint16_t half = (uint16_t)(sign | ((uint16_t)half_exp << 10) | (uint16_t)(mant >> 13));
  if (mant & 0x1000u) half = (uint16_t)(half + 1);
  return half;
}

/* quant.rs:1021-1044 (f16_to_f32_bits). */
float oro_f16_to_f32_bits(uint16_t bits) {
  uint32_t sign = ((uint32_t)(bits >> 15)) << 31;
  int32_t exp = (bits >> 10) & 0x1F;
  uint32_t mant = bits & 0x03FFu;
  uint32_t f;
  if (exp == 0) {
    if (mant == 0) {
      f = sign;
    } else {
      uint32_t mantissa = mant;
      int32_t exponent = -14;
      while ((mantissa & 0x0400u) == 0) {
        mantissa <<= 1;
        exponent -= 1;
      }
      mantissa &= 0x03FFu;
      f = sign | ((uint32_t)(exponent + 127) << 23) | (mantissa << 13);
    }
  } else if (exp == 0x1F) {
    f = sign | 0x7F800000u | (mant << 13);
  } else {
    f = sign | ((uint32_t)(exp - 15 + 127) << 23) | (mant << 13);
  }
  return bits_to_f32(f);
}

/* quant.rs:886-892 (decode_f8_e8m0): raw 0 -> 2^-127 (bit 22). */
float oro_decode_f8_e8m0(uint8_t raw) {
  if (raw == 0) return bits_to_f32(1u << 22);
  return bits_to_f32((uint32_t)raw << 23);
}

/* deepseek.rs:831-850 (f8e8m0_to_f32). Same values as decode_f8_e8m0 for all
 * 256 codes; kept separate because it is a separate reference function. */
float oro_f8e8m0_to_f32(uint8_t raw) {
  int32_t exponent = (int32_t)raw - 127;
  if (exponent < -126) {
    if (exponent < -149) return 0.0f;
    return bits_to_f32(1u << (23 + (exponent + 126)));
  } else if (exponent > 127) {
    return INFINITY;
  }
  return bits_to_f32((uint32_t)(exponent + 127) << 23);
}

/* deepseek.rs:799-826 (f8e4m3_to_f32); exp 15 clamps to +-448. */
float oro_f8e4m3_to_f32(uint8_t raw) {
  uint32_t sign = raw >> 7;
  uint32_t exp = (raw >> 3) & 0x0F;
  uint32_t mant = raw & 0x07;
  if (exp == 0) {
    if (mant == 0) return bits_to_f32(sign << 31);
    float v = (float)mant * ldexpf(1.0f, 1 - 6);
    return sign == 0 ? v * 1.0f : v * -1.0f;
  } else if (exp == 15) {
    return sign == 0 ? 448.0f : -448.0f;
  }
  uint32_t exp32 = exp + (127 - 7);
  return bits_to_f32((sign << 31) | (exp32 << 23) | (mant << 20));
}

/* quant.rs:814-829 (q4_quantize_block). */
void oro_q4_quantize_block(const float *src, uint8_t *dst) {
  float amax = 0.0f;
  for (int i = 0; i < 32; ++i) amax = rs_max(amax, fabsf(src[i]));
  float scale = amax > 0.0f ? amax / 7.0f : 1.0e-10f;
  uint16_t s16 = oro_f32_to_f16_bits(scale);
  dst[0] = (uint8_t)(s16 & 0xFF);
  dst[1] = (uint8_t)(s16 >> 8);
  for (int i = 0; i < 16; ++i) {
    uint8_t q0 = rs_as_u8(rs_clamp(roundf(src[2 * i] / scale + 8.0f), 0.0f, 15.0f));
    uint8_t q1 = rs_as_u8(rs_clamp(roundf(src[2 * i + 1] / scale + 8.0f), 0.0f, 15.0f));
    dst[2 + i] = (uint8_t)(q0 | (q1 << 4));
  }
}

/* quant.rs:831-858 (q5_quantize_block). */
void oro_q5_quantize_block(const float *src, uint8_t *dst) {
  float amax = 0.0f;
  for (int i = 0; i < 32; ++i) amax = rs_max(amax, fabsf(src[i]));
  float scale = amax > 0.0f ? amax / 15.0f : 1.0e-10f;
  uint16_t s16 = oro_f32_to_f16_bits(scale);
  dst[0] = (uint8_t)(s16 & 0xFF);
  dst[1] = (uint8_t)(s16 >> 8);
  memset(dst + 2, 0, 4);
  for (int i = 0; i < 32; ++i) {
    uint8_t q = rs_as_u8(rs_clamp(roundf(src[i] / scale + 16.0f), 0.0f, 31.0f));
    uint8_t low = q & 0x0F;
    uint8_t high = (q >> 4) & 0x01;
    int nib = i / 2;
    if (i % 2 == 0) dst[6 + nib] = low;
    else dst[6 + nib] |= (uint8_t)(low << 4);
    if (high) dst[2 + i / 8] |= (uint8_t)(1u << (i % 8));
  }
}

/* quant.rs:860-879 (iq3_quantize_block). */
void oro_iq3_quantize_block(const float *src, uint8_t *dst) {
  float amax = 0.0f;
  for (int i = 0; i < 32; ++i) amax = rs_max(amax, fabsf(src[i]));
  float scale = amax > 0.0f ? amax / 4.0f : 1.0e-10f;
  uint16_t s16 = oro_f32_to_f16_bits(scale);
  dst[0] = (uint8_t)(s16 & 0xFF);
  dst[1] = (uint8_t)(s16 >> 8);
  memset(dst + 2, 0, 12);
  for (int i = 0; i < 32; ++i) {
    uint8_t q = rs_as_u8(rs_clamp(roundf(src[i] / scale + 4.0f), 0.0f, 7.0f));
    uint8_t low = q & 0x03;
    uint8_t high = (q >> 2) & 0x01;
    dst[2 + i / 4] |= (uint8_t)(low << (2 * (i % 4)));
    dst[10 + i / 8] |= (uint8_t)(high << (i % 8));
  }
}

/* quant.rs:881-884 (FP4_TABLE): code 8 is -0.0 in the quant.rs table. */
static const float FP4_TABLE[16] = {0.0f,  0.5f,  1.0f,  1.5f,  2.0f,  3.0f,
                                    4.0f,  6.0f,  -0.0f, -0.5f, -1.0f, -1.5f,
                                    -2.0f, -3.0f, -4.0f, -6.0f};
/* deepseek.rs:789-792 (FP4_E2M1FN_TABLE): code 8 is +0.0 in the parser. */
static const float FP4_E2M1FN_TABLE[16] = {
    0.0f, 0.5f,  1.0f,  1.5f,  2.0f,  3.0f,  4.0f,  6.0f,
    0.0f, -0.5f, -1.0f, -1.5f, -2.0f, -3.0f, -4.0f, -6.0f};

/* quant.rs:894-906 (quantize_val): nearest table entry, first minimum wins. */
static uint8_t fp4_quantize_val(float val, float scale) {
  float scaled = val / scale;
  int best_q = 0;
  float min_diff = INFINITY;
  for (int q = 0; q < 16; ++q) {
    float diff = fabsf(scaled - FP4_TABLE[q]);
    if (diff < min_diff) {
      min_diff = diff;
      best_q = q;
    }
  }
  return (uint8_t)best_q;
}

/* quant.rs:908-926 (fp4_quantize_block): E8M0 = clamp(ceil(log2(amax/6))+127). */
void oro_fp4_quantize_block(const float *src, uint8_t *dst) {
  float amax = 0.0f;
  for (int i = 0; i < 32; ++i) amax = rs_max(amax, fabsf(src[i]));
  uint8_t raw = 0;
  if (amax > 0.0f && isfinite(amax)) {
    /* Rust `(amax / 6.0).log2().ceil() as i32` (saturating cast). */
    float c = ceilf(log2f(amax / 6.0f));
    int32_t k;
    if (c != c) k = 0;
    else if (c >= 2147483647.0f) k = 2147483647;
    else if (c <= -2147483648.0f) k = (int32_t)-2147483647 - 1;
    else k = (int32_t)c;
    int64_t r = (int64_t)k + 127;
    raw = (uint8_t)(r < 0 ? 0 : (r > 255 ? 255 : r));
  }
  dst[0] = raw;
  float actual = oro_decode_f8_e8m0(raw);
  for (int i = 0; i < 16; ++i) {
    uint8_t q0 = fp4_quantize_val(src[2 * i], actual);
    uint8_t q1 = fp4_quantize_val(src[2 * i + 1], actual);
    dst[1 + i] = (uint8_t)(q0 | (q1 << 4));
  }
}

/* quant.rs:506-581 (quantize_matrix_cpu) with validate_dense_matrix
 * (quant.rs:725-749): cols must be a multiple of 32. */
int oro_quantize_matrix(int fmt, const float *matrix, size_t rows, size_t cols,
                        uint8_t *out) {
  size_t bb = oro_block_bytes(fmt);
  if (bb == 0 || cols % 32 != 0) return ORO_INVALID_INPUT;
  size_t bpr = cols / 32;
  for (size_t r = 0; r < rows; ++r) {
    for (size_t b = 0; b < bpr; ++b) {
      const float *src = matrix + r * cols + b * 32;
      uint8_t *dst = out + r * bpr * bb + b * bb;
      switch (fmt) {
        case ORO_Q4_0: oro_q4_quantize_block(src, dst); break;
        case ORO_Q5_0: oro_q5_quantize_block(src, dst); break;
        case ORO_IQ3_0: oro_iq3_quantize_block(src, dst); break;
        default: oro_fp4_quantize_block(src, dst); break;
      }
    }
  }
  return ORO_OK;
}

/* quant.rs:951-972 (q4_dot_row). */
static float q4_dot_row(const uint8_t *row_q, const float *x, size_t cols) {
  size_t bpr = cols / 32;
  float sum = 0.0f;
  for (size_t b = 0; b < bpr; ++b) {
    const uint8_t *blk = row_q + b * 18;
    float scale = oro_f16_to_f32_bits((uint16_t)(blk[0] | (blk[1] << 8)));
    for (int lane = 0; lane < 32; ++lane) {
      size_t col = b * 32 + lane;
      uint8_t packed = blk[2 + lane / 2];
      uint8_t q = (lane % 2 == 0) ? (packed & 0x0F) : (packed >> 4);
      float w = (float)((int)q - 8) * scale;
      if (col < cols) sum += w * x[col];
    }
  }
  return sum;
}

/* quant.rs:974-996 (q5_dot_row). */
static float q5_dot_row(const uint8_t *row_q, const float *x, size_t cols) {
  size_t bpr = cols / 32;
  float sum = 0.0f;
  for (size_t b = 0; b < bpr; ++b) {
    const uint8_t *blk = row_q + b * 22;
    float scale = oro_f16_to_f32_bits((uint16_t)(blk[0] | (blk[1] << 8)));
    for (int lane = 0; lane < 32; ++lane) {
      size_t col = b * 32 + lane;
      uint8_t low_byte = blk[6 + lane / 2];
      uint8_t low = (lane % 2 == 0) ? (low_byte & 0x0F) : (low_byte >> 4);
      uint8_t high = (blk[2 + lane / 8] >> (lane % 8)) & 0x01;
      uint8_t q = (uint8_t)(low | (high << 4));
      float w = (float)((int)q - 16) * scale;
      if (col < cols) sum += w * x[col];
    }
  }
  return sum;
}

/* quant.rs:998-1019 (iq3_dot_row). */
static float iq3_dot_row(const uint8_t *row_q, const float *x, size_t cols) {
  size_t bpr = cols / 32;
  float sum = 0.0f;
  for (size_t b = 0; b < bpr; ++b) {
    const uint8_t *blk = row_q + b * 14;
    float scale = oro_f16_to_f32_bits((uint16_t)(blk[0] | (blk[1] << 8)));
    for (int lane = 0; lane < 32; ++lane) {
      size_t col = b * 32 + lane;
      uint8_t low = (blk[2 + lane / 4] >> (2 * (lane % 4))) & 0x03;
      uint8_t high = (blk[10 + lane / 8] >> (lane % 8)) & 0x01;
      uint8_t q = (uint8_t)(low | (high << 2));
      float w = (float)((int)q - 4) * scale;
      if (col < cols) sum += w * x[col];
    }
  }
  return sum;
}

/* quant.rs:928-949 (fp4_dot_row), interleaved 17-byte blocks. */
static float fp4_dot_row(const uint8_t *row_q, const float *x, size_t cols) {
  size_t bpr = cols / 32;
  float sum = 0.0f;
  for (size_t b = 0; b < bpr; ++b) {
    const uint8_t *blk = row_q + b * 17;
    float scale = oro_decode_f8_e8m0(blk[0]);
    for (int lane = 0; lane < 32; ++lane) {
      size_t col = b * 32 + lane;
      if (col < cols) {
        uint8_t packed = blk[1 + lane / 2];
        uint8_t q = (lane % 2 == 0) ? (packed & 0x0F) : (packed >> 4);
        float w = FP4_TABLE[q] * scale;
        sum += w * x[col];
      }
    }
  }
  return sum;
}

float oro_dot_row(int fmt, const uint8_t *row_q, const float *x, size_t cols) {
  switch (fmt) {
    case ORO_Q4_0: return q4_dot_row(row_q, x, cols);
    case ORO_Q5_0: return q5_dot_row(row_q, x, cols);
    case ORO_IQ3_0: return iq3_dot_row(row_q, x, cols);
    default: return fp4_dot_row(row_q, x, cols);
  }
}

/* quant.rs:627-646 (gemv_cpu) with validate_quant_inputs (quant.rs:751-812). */
int oro_gemv(int fmt, const uint8_t *qweights, const float *x, size_t rows,
             size_t cols, float *y) {
  size_t bb = oro_block_bytes(fmt);
  if (bb == 0 || cols % 32 != 0) return ORO_INVALID_INPUT;
  size_t row_bytes = cols / 32 * bb;
  for (size_t r = 0; r < rows; ++r)
    y[r] = oro_dot_row(fmt, qweights + r * row_bytes, x, cols);
  return ORO_OK;
}

typedef struct {
  int fmt;
  const uint8_t *qw;
  const float *x;
  size_t r0, r1, cols, row_bytes;
  float *y;
} gemv_job;

static void *gemv_worker(void *arg) {
  gemv_job *j = (gemv_job *)arg;
  for (size_t r = j->r0; r < j->r1; ++r)
    j->y[r] = oro_dot_row(j->fmt, j->qw + r * j->row_bytes, j->x, j->cols);
  return NULL;
}

static int resolve_threads(int threads) {
  if (threads <= 0) {
    long n = sysconf(_SC_NPROCESSORS_ONLN);
    threads = n > 0 ? (int)n : 1;
  }
  if (threads > 256) threads = 256;
  return threads;
}

int oro_gemv_threads(int fmt, const uint8_t *qweights, const float *x,
                     size_t rows, size_t cols, float *y, int threads) {
  size_t bb = oro_block_bytes(fmt);
  if (bb == 0 || cols % 32 != 0) return ORO_INVALID_INPUT;
  threads = resolve_threads(threads);
  if ((size_t)threads > rows) threads = rows ? (int)rows : 1;
  if (threads <= 1) return oro_gemv(fmt, qweights, x, rows, cols, y);
  pthread_t tid[256];
  gemv_job job[256];
  size_t per = (rows + threads - 1) / threads;
  int started = 0;
  for (int t = 0; t < threads; ++t) {
    size_t r0 = (size_t)t * per, r1 = r0 + per;
    if (r0 >= rows) break;
    if (r1 > rows) r1 = rows;
    job[t] = (gemv_job){fmt, qweights, x, r0, r1, cols, cols / 32 * bb, y};
    if (pthread_create(&tid[t], NULL, gemv_worker, &job[t]) != 0) {
      gemv_worker(&job[t]);
      tid[t] = 0;
    }
    started = t + 1;
  }
  for (int t = 0; t < started; ++t)
    if (tid[t]) pthread_join(tid[t], NULL);
  return ORO_OK;
}

/* The per-weight values the dot rows use (quant.rs:928-1019): w = (q - off)
 * * scale (Q4/Q5/IQ3, f16 scale) or FP4_TABLE[q] * e8m0 (FP4 interleaved).
 * Used by tests to form the tolerance sum_l |w_l x_l| of each row. */
int oro_dequantize_matrix(int fmt, const uint8_t *qw, size_t rows, size_t cols,
                          float *out) {
  size_t bb = oro_block_bytes(fmt);
  if (bb == 0 || cols % 32 != 0) return ORO_INVALID_INPUT;
  size_t bpr = cols / 32;
  for (size_t r = 0; r < rows; ++r) {
    for (size_t b = 0; b < bpr; ++b) {
      const uint8_t *blk = qw + (r * bpr + b) * bb;
      float *o = out + r * cols + b * 32;
      for (int e = 0; e < 32; ++e) {
        float w;
        if (fmt == ORO_Q4_0) {
          float s = oro_f16_to_f32_bits((uint16_t)(blk[0] | (blk[1] << 8)));
          uint8_t by = blk[2 + e / 2];
          uint8_t q = (e % 2 == 0) ? (by & 0x0F) : (by >> 4);
          w = (float)((int)q - 8) * s;
        } else if (fmt == ORO_Q5_0) {
          float s = oro_f16_to_f32_bits((uint16_t)(blk[0] | (blk[1] << 8)));
          uint8_t by = blk[6 + e / 2];
          uint8_t lo = (e % 2 == 0) ? (by & 0x0F) : (by >> 4);
          uint8_t hi = (blk[2 + e / 8] >> (e % 8)) & 1;
          w = (float)((int)(lo | (hi << 4)) - 16) * s;
        } else if (fmt == ORO_IQ3_0) {
          float s = oro_f16_to_f32_bits((uint16_t)(blk[0] | (blk[1] << 8)));
          uint8_t lo = (blk[2 + e / 4] >> (2 * (e % 4))) & 3;
          uint8_t hi = (blk[10 + e / 8] >> (e % 8)) & 1;
          w = (float)((int)(lo | (hi << 2)) - 4) * s;
        } else {
          float s = oro_decode_f8_e8m0(blk[0]);
          uint8_t by = blk[1 + e / 2];
          uint8_t q = (e % 2 == 0) ? (by & 0x0F) : (by >> 4);
          w = FP4_TABLE[q] * s;
        }
        o[e] = w;
      }
    }
  }
  return ORO_OK;
}

/* quant.rs:599-625 (dense_gemv_cpu): `iter().map(w*x).sum()`, a sequential
 * f32 sum.  Rust's float Sum starts from -0.0; -0.0 + v == v for every v. */
void oro_dense_gemv(const float *matrix, const float *x, size_t rows,
                    size_t cols, float *y) {
  for (size_t r = 0; r < rows; ++r) {
    float sum = -0.0f;
    const float *row = matrix + r * cols;
    for (size_t c = 0; c < cols; ++c) sum += row[c] * x[c];
    y[r] = sum;
  }
}

/* deepseek.rs:862-918 (decode_deepseek_fp4_to_f32): split layout, weight
 * [rows, cols/2] low nibble first, scale [rows, cols/block]; code 8 -> +0.0. */
void oro_fp4_decode_split(const uint8_t *weight, const uint8_t *scale,
                          size_t rows, size_t cols, size_t block_size,
                          float *out) {
  size_t phys = cols / 2, scols = cols / block_size;
  for (size_t r = 0; r < rows; ++r) {
    for (size_t g = 0; g < phys; ++g) {
      uint8_t b = weight[r * phys + g];
      size_t lo = g * 2, hi = lo + 1;
      float s_lo = oro_f8e8m0_to_f32(scale[r * scols + lo / block_size]);
      float s_hi = oro_f8e8m0_to_f32(scale[r * scols + hi / block_size]);
      out[r * cols + lo] = FP4_E2M1FN_TABLE[b & 0x0F] * s_lo;
      out[r * cols + hi] = FP4_E2M1FN_TABLE[(b >> 4) & 0x0F] * s_hi;
    }
  }
}

/* moe.rs:1313-1317: act = g / (1 + exp(-g)) * u (no clamp on the CPU path). */
static void swiglu(const float *gate, const float *up, float *act, size_t n) {
  for (size_t i = 0; i < n; ++i) {
    float g = gate[i];
    float silu = g / (1.0f + expf(-g));
    act[i] = silu * up[i];
  }
}

/* moe.rs:1283-1324 (selected_moe_cpu): per selected (e, w) in the given order:
 * gate = gemv_cpu(Q4, Wg, x); up = gemv_cpu(Q4, Wu, x); act = swiglu;
 * down = gemv_cpu(Q4, Wd, act); out[i] += w * down[i]. */
int oro_selected_moe_q4(const uint8_t *const *w_gate,
                        const uint8_t *const *w_up,
                        const uint8_t *const *w_down, size_t num_experts,
                        const int64_t *sel_ids, const float *sel_weights,
                        size_t num_selected, const float *x, size_t hidden,
                        size_t intermediate, size_t out_dim, float *out,
                        int threads) {
  if (hidden % 32 || intermediate % 32) return ORO_INVALID_INPUT;
  for (size_t k = 0; k < num_selected; ++k)
    if (sel_ids[k] < 0 || (size_t)sel_ids[k] >= num_experts) return ORO_INVALID_INPUT;
  float *gate = malloc(intermediate * sizeof(float));
  float *up = malloc(intermediate * sizeof(float));
  float *act = malloc(intermediate * sizeof(float));
  float *down = malloc(out_dim * sizeof(float));
  if (!gate || !up || !act || !down) {
    free(gate); free(up); free(act); free(down);
    return ORO_INVALID_INPUT;
  }
  for (size_t i = 0; i < out_dim; ++i) out[i] = 0.0f;
  for (size_t k = 0; k < num_selected; ++k) {
    size_t e = (size_t)sel_ids[k];
    float w = sel_weights[k];
    oro_gemv_threads(ORO_Q4_0, w_gate[e], x, intermediate, hidden, gate, threads);
    oro_gemv_threads(ORO_Q4_0, w_up[e], x, intermediate, hidden, up, threads);
    swiglu(gate, up, act, intermediate);
    oro_gemv_threads(ORO_Q4_0, w_down[e], act, out_dim, intermediate, down, threads);
    for (size_t i = 0; i < out_dim; ++i) out[i] += w * down[i];
  }
  free(gate); free(up); free(act); free(down);
  return ORO_OK;
}

typedef struct {
  const float *m;
  const float *x;
  size_t r0, r1, cols;
  float *y;
} dense_job;

static void *dense_worker(void *arg) {
  dense_job *j = (dense_job *)arg;
  oro_dense_gemv(j->m + j->r0 * j->cols, j->x, j->r1 - j->r0, j->cols, j->y + j->r0);
  return NULL;
}

static void dense_gemv_threads(const float *m, const float *x, size_t rows,
                               size_t cols, float *y, int threads) {
  threads = resolve_threads(threads);
  if ((size_t)threads > rows) threads = rows ? (int)rows : 1;
  if (threads <= 1) {
    oro_dense_gemv(m, x, rows, cols, y);
    return;
  }
  pthread_t tid[256];
  dense_job job[256];
  size_t per = (rows + threads - 1) / threads;
  int started = 0;
  for (int t = 0; t < threads; ++t) {
    size_t r0 = (size_t)t * per, r1 = r0 + per;
    if (r0 >= rows) break;
    if (r1 > rows) r1 = rows;
    job[t] = (dense_job){m, x, r0, r1, cols, y};
    if (pthread_create(&tid[t], NULL, dense_worker, &job[t]) != 0) {
      dense_worker(&job[t]);
      tid[t] = 0;
    }
    started = t + 1;
  }
  for (int t = 0; t < started; ++t)
    if (tid[t]) pthread_join(tid[t], NULL);
}

/* moe.rs:1665-1735 (selected_moe_cpu_native_fp4): decode each tensor with the
 * parser's FP4 decode (block 32) to dense f32, then dense_gemv_cpu. */
int oro_selected_moe_native_fp4(
    const uint8_t *const *gate_w, const uint8_t *const *gate_s,
    const uint8_t *const *up_w, const uint8_t *const *up_s,
    const uint8_t *const *down_w, const uint8_t *const *down_s,
    size_t num_experts, const int64_t *sel_ids, const float *sel_weights,
    size_t num_selected, const float *x, size_t hidden, size_t intermediate,
    size_t out_dim, float *out, int threads) {
  if (hidden % 32 || intermediate % 32) return ORO_INVALID_INPUT;
  for (size_t k = 0; k < num_selected; ++k)
    if (sel_ids[k] < 0 || (size_t)sel_ids[k] >= num_experts) return ORO_INVALID_INPUT;
  size_t big = intermediate * hidden > out_dim * intermediate ? intermediate * hidden
                                                              : out_dim * intermediate;
  float *dense = malloc(big * sizeof(float));
  float *gate = malloc(intermediate * sizeof(float));
  float *up = malloc(intermediate * sizeof(float));
  float *act = malloc(intermediate * sizeof(float));
  float *down = malloc(out_dim * sizeof(float));
  if (!dense || !gate || !up || !act || !down) {
    free(dense); free(gate); free(up); free(act); free(down);
    return ORO_INVALID_INPUT;
  }
  for (size_t i = 0; i < out_dim; ++i) out[i] = 0.0f;
  for (size_t k = 0; k < num_selected; ++k) {
    size_t e = (size_t)sel_ids[k];
    float w = sel_weights[k];
    oro_fp4_decode_split(gate_w[e], gate_s[e], intermediate, hidden, 32, dense);
    dense_gemv_threads(dense, x, intermediate, hidden, gate, threads);
    oro_fp4_decode_split(up_w[e], up_s[e], intermediate, hidden, 32, dense);
    dense_gemv_threads(dense, x, intermediate, hidden, up, threads);
    swiglu(gate, up, act, intermediate);
    oro_fp4_decode_split(down_w[e], down_s[e], out_dim, intermediate, 32, dense);
    dense_gemv_threads(dense, act, out_dim, intermediate, down, threads);
    for (size_t i = 0; i < out_dim; ++i) out[i] += w * down[i];
  }
  free(dense); free(gate); free(up); free(act); free(down);
  return ORO_OK;
}

/* dsl_moe.rs:720-740 (cpu_router, after the logits): max-subtracted softmax,
 * then a stable descending sort (`sort_by` with partial_cmp, NaN == Equal)
 * truncated to top_k.  `renormalize` divides the kept weights by their
 * sequential f32 sum (the BASELINE layer configs ask for it; the reference
 * router does not renormalise). */
int oro_router_from_logits(const float *logits, size_t n, size_t top_k,
                           int renormalize, int64_t *ids, float *weights) {
  if (n == 0 || top_k > n) return ORO_INVALID_INPUT;
  float maxl = -INFINITY;
  for (size_t e = 0; e < n; ++e) maxl = rs_max(maxl, logits[e]);
  float *probs = malloc(n * sizeof(float));
  size_t *idx = malloc(n * sizeof(size_t));
  size_t *tmp = malloc(n * sizeof(size_t));
  if (!probs || !idx || !tmp) {
    free(probs); free(idx); free(tmp);
    return ORO_INVALID_INPUT;
  }
  float sum_exp = 0.0f;
  for (size_t e = 0; e < n; ++e) {
    float v = expf(logits[e] - maxl);
    probs[e] = v;
    sum_exp += v;
  }
  for (size_t e = 0; e < n; ++e) probs[e] /= sum_exp;
  /* Stable bottom-up merge sort, descending by probability. "a before b"
   * unless b.1 > a.1 strictly (partial_cmp: NaN compares Equal). */
  for (size_t e = 0; e < n; ++e) idx[e] = e;
  for (size_t width = 1; width < n; width *= 2) {
    for (size_t lo = 0; lo < n; lo += 2 * width) {
      size_t mid = lo + width < n ? lo + width : n;
      size_t hi = lo + 2 * width < n ? lo + 2 * width : n;
      size_t i = lo, j = mid, o = lo;
      while (i < mid && j < hi) {
        if (probs[idx[j]] > probs[idx[i]]) tmp[o++] = idx[j++];
        else tmp[o++] = idx[i++];
      }
      while (i < mid) tmp[o++] = idx[i++];
      while (j < hi) tmp[o++] = idx[j++];
    }
    memcpy(idx, tmp, n * sizeof(size_t));
  }
  for (size_t k = 0; k < top_k; ++k) {
    ids[k] = (int64_t)idx[k];
    weights[k] = probs[idx[k]];
  }
  if (renormalize) {
    float s = 0.0f;
    for (size_t k = 0; k < top_k; ++k) s += weights[k];
    if (s > 0.0f)
      for (size_t k = 0; k < top_k; ++k) weights[k] /= s;
  }
  free(probs); free(idx); free(tmp);
  return ORO_OK;
}

/* dsl_moe.rs:687-741 (cpu_router): logits = W.h with a sequential f32 sum. */
int oro_router(const float *router_weights, const float *hidden,
               size_t num_experts, size_t hidden_size, size_t top_k,
               int64_t *ids, float *weights) {
  float *logits = malloc((num_experts ? num_experts : 1) * sizeof(float));
  if (!logits) return ORO_INVALID_INPUT;
  for (size_t e = 0; e < num_experts; ++e) {
    float sum = 0.0f;
    for (size_t h = 0; h < hidden_size; ++h)
      sum += router_weights[e * hidden_size + h] * hidden[h];
    logits[e] = sum;
  }
  int rc = oro_router_from_logits(logits, num_experts, top_k, 0, ids, weights);
  free(logits);
  return rc;
}

/* quant.rs:1610-1620 (seeded_f32s): LCG, unit = (bits|1)/u32::MAX in f32,
 * value = 2*unit - 1.  Identical copies at moe.rs:1743 and bench_qgemv.rs:39. */
void oro_seeded_f32s(size_t len, uint64_t seed, float *out) {
  uint64_t state = seed;
  const float umax = (float)4294967295u;
  for (size_t i = 0; i < len; ++i) {
    state = state * 6364136223846793005ULL + 1ULL;
    uint32_t bits = (uint32_t)(state >> 32) | 1u;
    float unit = (float)bits / umax;
    out[i] = unit * 2.0f - 1.0f;
  }
}

/* ---------------------------------------------------------------------------
 * Official DeepSeek arithmetic (activations quantized to FP8), restated from
 * crates/objeta-parser/src/deepseek.rs:1444-1715.
 * ------------------------------------------------------------------------- */

/* deepseek.rs:1444-1481 (f32_to_f8e4m3_exact).  Below 2^-7 the subnormal
 * branch rounds |v| * 16 (always 0 there); [2^-7, 2^-6) encodes with exponent
 * field 0; >= 448 saturates to 0x7E / 0xFE. */
uint8_t oro_f32_to_f8e4m3_exact(float v) {
  const float a = fabsf(v);
  if (a < 1.0f / 128.0f) {
    const uint8_t sign = v < 0.0f ? 0x80 : 0;
    uint8_t q = rs_as_u8(roundf(a * 16.0f));
    if (q > 7) q = 7;
    return (uint8_t)(sign | q);
  }
  if (a >= 448.0f) return v < 0.0f ? 0xFE : 0x7E;
  const uint8_t sign = v < 0.0f ? 0x80 : 0;
  const uint32_t bits = f32_to_bits(a);
  const int32_t exp32 = (int32_t)((bits >> 23) & 0xFF) - 127;
  int32_t exp_f8 = exp32 + 7;
  if (exp_f8 < 0) exp_f8 = 0;
  const uint32_t mant_bits = bits & 0x7FFFFF;
  uint8_t mant3 = (uint8_t)((mant_bits + (1u << 19)) >> 20);
  uint8_t exp_final = (uint8_t)exp_f8;
  if (mant3 >= 8) {
    mant3 = 0;
    exp_final = exp_final == 255 ? 255 : (uint8_t)(exp_final + 1);
  }
  if (exp_final > 14) {
    exp_final = 14;
    mant3 = 7;
  }
  return (uint8_t)(sign | (uint8_t)(exp_final << 3) | (mant3 & 7));
}

/* deepseek.rs:1484-1525 (cpu_act_quant): per block, amax = max(|x|, 1e-4),
 * scale = 2^ceil(log2(amax * (1/448))), y = e4m3(clamp(x / scale, +-448)),
 * s = clamp(log2 scale + 127, 0, 255).  n % block == 0. */
int oro_act_quant(const float *x, size_t n, size_t block, uint8_t *y, uint8_t *s) {
  if (block == 0 || n % block) return -1;
  const float inv = 1.0f / 448.0f;
  for (size_t b = 0; b < n / block; ++b) {
    float amax = 0.0f;
    for (size_t i = b * block; i < (b + 1) * block; ++i) {
      const float a = fabsf(x[i]);
      if (a > amax) amax = a;
    }
    amax = rs_max(amax, 1e-4f);
    const float raw = amax * inv;
    int32_t lc = -127;
    if (raw > 0.0f) {
      const float c = ceilf(log2f(raw));
      if (c != c) lc = 0;
      else if (c >= 2147483647.0f) lc = 2147483647;
      else if (c <= -2147483648.0f) lc = (int32_t)-2147483647 - 1;
      else lc = (int32_t)c;
    }
    const float scale = ldexpf(1.0f, lc);
    const int64_t e = (int64_t)lc + 127;
    s[b] = (uint8_t)(e < 0 ? 0 : (e > 255 ? 255 : e));
    for (size_t i = b * block; i < (b + 1) * block; ++i)
      y[i] = oro_f32_to_f8e4m3_exact(rs_clamp(x[i] / scale, -448.0f, 448.0f));
  }
  return 0;
}

/* deepseek.rs:1528-1570 (cpu_fp8_act_fp4_weight_gemv_f32): sequential f32
 * sum over the packed bytes, low nibble then high, each term
 * ((act * act_scale) * fp4) * weight_scale; act blocks of 128, weight
 * blocks of 32, parser FP4 table (code 8 = +0.0). */
void oro_fp8_act_fp4_weight_gemv_f32(const uint8_t *act, const uint8_t *act_s, const uint8_t *w,
                                     const uint8_t *ws, size_t rows, size_t cols, float *y) {
  const size_t phys = cols / 2, scols = cols / 32;
  for (size_t r = 0; r < rows; ++r) {
    float sum = 0.0f;
    for (size_t cg = 0; cg < phys; ++cg) {
      const uint8_t b = w[r * phys + cg];
      const size_t lo = cg * 2, hi = lo + 1;
      const float t_lo = oro_f8e4m3_to_f32(act[lo]) * oro_f8e8m0_to_f32(act_s[lo / 128]) *
                         FP4_E2M1FN_TABLE[b & 0x0F] * oro_f8e8m0_to_f32(ws[r * scols + lo / 32]);
      const float t_hi = oro_f8e4m3_to_f32(act[hi]) * oro_f8e8m0_to_f32(act_s[hi / 128]) *
                         FP4_E2M1FN_TABLE[(b >> 4) & 0x0F] * oro_f8e8m0_to_f32(ws[r * scols + hi / 32]);
      sum += t_lo;
      sum += t_hi;
    }
    y[r] = sum;
  }
}

/* deepseek.rs:1630-1660 (cpu_fp8_act_fp8_weight_gemv): f64 sum of
 * act * act_scale * w * w_scale; weight scales on a 128 x 128 tile grid. */
void oro_fp8_act_fp8_weight_gemv(const uint8_t *act, const uint8_t *act_s, const uint8_t *w,
                                 const uint8_t *ws, size_t rows, size_t cols, float *y) {
  const size_t wsc = (cols + 127) / 128;
  for (size_t r = 0; r < rows; ++r) {
    double sum = 0.0;
    for (size_t c = 0; c < cols; ++c) {
      sum += (double)oro_f8e4m3_to_f32(act[c]) * (double)oro_f8e8m0_to_f32(act_s[c / 128]) *
             (double)oro_f8e4m3_to_f32(w[r * cols + c]) * (double)oro_f8e8m0_to_f32(ws[(r / 128) * wsc + c / 128]);
    }
    y[r] = (float)sum;
  }
}

/* SwiGLU of the official experts (deepseek.rs:1675-1680, 1707-1711): only
 * the up value is clamped; act = g / (1 + exp(-g)) * clamp(u). */
static void official_swiglu(const float *g, const float *u, size_t n, float limit, float *act) {
  for (size_t i = 0; i < n; ++i) {
    const float uu = rs_clamp(u[i], -limit, limit);
    act[i] = g[i] / (1.0f + expf(-g[i])) * uu;
  }
}

/* deepseek.rs:1690-1715 (cpu_routed_expert_fp4_official_f32): act_quant(x),
 * gate / up fp8 x fp4 GEMVs, SwiGLU, act_quant(act), down GEMV. */
int oro_routed_expert_fp4_official_f32(const uint8_t *gw, const uint8_t *gs, const uint8_t *uw, const uint8_t *us,
                                       const uint8_t *dw, const uint8_t *ds, const float *x, size_t dim,
                                       size_t inter, size_t out_dim, float swiglu_limit, float *out) {
  if (dim % 128 || inter % 128) return -1;
  uint8_t *a = (uint8_t *)malloc(dim), *as = (uint8_t *)malloc(dim / 128);
  uint8_t *a2 = (uint8_t *)malloc(inter), *as2 = (uint8_t *)malloc(inter / 128);
  float *g = (float *)malloc(inter * 4), *u = (float *)malloc(inter * 4), *act = (float *)malloc(inter * 4);
  int rc = -2;
  if (a && as && a2 && as2 && g && u && act) {
    oro_act_quant(x, dim, 128, a, as);
    oro_fp8_act_fp4_weight_gemv_f32(a, as, gw, gs, inter, dim, g);
    oro_fp8_act_fp4_weight_gemv_f32(a, as, uw, us, inter, dim, u);
    official_swiglu(g, u, inter, swiglu_limit, act);
    oro_act_quant(act, inter, 128, a2, as2);
    oro_fp8_act_fp4_weight_gemv_f32(a2, as2, dw, ds, out_dim, inter, out);
    rc = 0;
  }
  free(a); free(as); free(a2); free(as2); free(g); free(u); free(act);
  return rc;
}

/* deepseek.rs:1662-1688 (cpu_shared_expert_fp8_official): the same with fp8
 * x fp8 GEMVs (f64 sums). */
int oro_shared_expert_fp8_official(const uint8_t *w1, const uint8_t *s1, const uint8_t *w3, const uint8_t *s3,
                                   const uint8_t *w2, const uint8_t *s2, const float *x, size_t dim, size_t inter,
                                   float swiglu_limit, float *out) {
  if (dim % 128 || inter % 128) return -1;
  uint8_t *a = (uint8_t *)malloc(dim), *as = (uint8_t *)malloc(dim / 128);
  uint8_t *a2 = (uint8_t *)malloc(inter), *as2 = (uint8_t *)malloc(inter / 128);
  float *g = (float *)malloc(inter * 4), *u = (float *)malloc(inter * 4), *act = (float *)malloc(inter * 4);
  int rc = -2;
  if (a && as && a2 && as2 && g && u && act) {
    oro_act_quant(x, dim, 128, a, as);
    oro_fp8_act_fp8_weight_gemv(a, as, w1, s1, inter, dim, g);
    oro_fp8_act_fp8_weight_gemv(a, as, w3, s3, inter, dim, u);
    official_swiglu(g, u, inter, swiglu_limit, act);
    oro_act_quant(act, inter, 128, a2, as2);
    oro_fp8_act_fp8_weight_gemv(a2, as2, w2, s2, dim, inter, out);
    rc = 0;
  }
  free(a); free(as); free(a2); free(as2); free(g); free(u); free(act);
  return rc;
}

/* dsl_moe.rs:768-881 (cpu_gate_ref): DeepSeek gate.  logits = W.h (sequential
 * f32, separate multiply and add); scores by score_func (0 softmax, 1 sigmoid,
 * 2 sqrt-softplus with the reference's branches, including ln_1p(exp(-v))
 * below -20); selection = top_k of scores + bias by a stable descending sort,
 * or tid2eid[input_id * top_k + k] for hash layers; weights = scores of the
 * selection, divided by their sequential sum unless softmax, times
 * route_scale.  Returns ORO_INVALID_INPUT when a hash layer's input_id is out
 * of range. */
int oro_deepseek_gate(const float *gate_weight, const float *gate_bias, const int64_t *tid2eid,
                      size_t tid2eid_len, const float *hidden, int64_t input_id, size_t num_experts,
                      size_t hidden_size, size_t top_k, int score_func, float route_scale, int64_t *ids,
                      float *weights) {
  if (num_experts == 0 || top_k > num_experts) return ORO_INVALID_INPUT;
  float *logits = malloc(num_experts * sizeof(float));
  float *scores = malloc(num_experts * sizeof(float));
  float *sel = malloc(num_experts * sizeof(float));
  size_t *idx = malloc(num_experts * sizeof(size_t));
  size_t *tmp = malloc(num_experts * sizeof(size_t));
  int rc = ORO_OK;
  if (!logits || !scores || !sel || !idx || !tmp) {
    rc = ORO_INVALID_INPUT;
    goto done;
  }
  for (size_t e = 0; e < num_experts; ++e) {
    float sum = 0.0f;
    for (size_t h = 0; h < hidden_size; ++h) sum += gate_weight[e * hidden_size + h] * hidden[h];
    logits[e] = sum;
  }
  if (score_func == 0) {
    float m = -INFINITY, s = 0.0f;
    for (size_t e = 0; e < num_experts; ++e) m = rs_max(m, logits[e]);
    for (size_t e = 0; e < num_experts; ++e) {
      scores[e] = expf(logits[e] - m);
      s += scores[e];
    }
    for (size_t e = 0; e < num_experts; ++e) scores[e] /= s;
  } else if (score_func == 1) {
    for (size_t e = 0; e < num_experts; ++e) scores[e] = 1.0f / (1.0f + expf(-logits[e]));
  } else {
    for (size_t e = 0; e < num_experts; ++e) {
      const float v = logits[e];
      const float sp = v > 20.0f ? v : (v < -20.0f ? log1pf(expf(-v)) : log1pf(expf(v)));
      scores[e] = sqrtf(sp);
    }
  }
  if (tid2eid) {
    if (input_id < 0 || (size_t)input_id >= tid2eid_len / top_k) {
      rc = ORO_INVALID_INPUT;
      goto done;
    }
    for (size_t k = 0; k < top_k; ++k) ids[k] = tid2eid[(size_t)input_id * top_k + k];
  } else {
    for (size_t e = 0; e < num_experts; ++e) sel[e] = scores[e] + (gate_bias ? gate_bias[e] : 0.0f);
    if (!gate_bias)
      for (size_t e = 0; e < num_experts; ++e) sel[e] = scores[e];
    for (size_t e = 0; e < num_experts; ++e) idx[e] = e;
    for (size_t width = 1; width < num_experts; width *= 2) {
      for (size_t lo = 0; lo < num_experts; lo += 2 * width) {
        size_t mid = lo + width < num_experts ? lo + width : num_experts;
        size_t hi = lo + 2 * width < num_experts ? lo + 2 * width : num_experts;
        size_t i = lo, j = mid, o = lo;
        while (i < mid && j < hi) {
          if (sel[idx[j]] > sel[idx[i]]) tmp[o++] = idx[j++];
          else tmp[o++] = idx[i++];
        }
        while (i < mid) tmp[o++] = idx[i++];
        while (j < hi) tmp[o++] = idx[j++];
      }
      memcpy(idx, tmp, num_experts * sizeof(size_t));
    }
    for (size_t k = 0; k < top_k; ++k) ids[k] = (int64_t)idx[k];
  }
  for (size_t k = 0; k < top_k; ++k) {
    const int64_t e = ids[k];
    weights[k] = (e >= 0 && (size_t)e < num_experts) ? scores[e] : NAN;
  }
  if (score_func != 0) {
    float s = 0.0f;
    for (size_t k = 0; k < top_k; ++k) s += weights[k];
    if (s > 0.0f)
      for (size_t k = 0; k < top_k; ++k) weights[k] /= s;
  }
  for (size_t k = 0; k < top_k; ++k) weights[k] *= route_scale;
done:
  free(logits); free(scores); free(sel); free(idx); free(tmp);
  return rc;
}
