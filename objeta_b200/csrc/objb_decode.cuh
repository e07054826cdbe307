// objb_decode.cuh -- in-register block decoders for the batch-1 GEMV.
//
// Each format defines a "lane tile": the run of consecutive 32-weight blocks
// one lane owns within a row, sized so the tile is a whole number of 32-bit
// words and the word stride between lanes is odd (bank-conflict-free shared
// memory reads).  A lane keeps the x values of its tile in registers for the
// whole kernel and, for every row that streams through shared memory, returns
// its partial dot product.  Per block the decoders form sum_l (q_l - off) x_l
// in fp32 and multiply by the block scale once, which is the reference's
// arithmetic (w = (q - off) * scale; sum += w * x, quant.rs:928-1019) with the
// scale factored out of the block sum.
//
// Q4_0 uses an exact "magic number" decode: OR-ing a nibble that sits at bit
// 4k of a word into the mantissa of 2^23 gives the float 2^23 + q*16^k, and
// subtracting 2^23 + 8*16^k leaves (q - 8)*16^k exactly.  The matching x
// register holds x * 16^-k (an exact power-of-two scaling), so the product is
// (q - 8) * x rounded once.  Pairs of lanes of that arithmetic run as
// sm_100 packed fp32x2 add / fma (__fadd2_rn, __ffma2_rn).
#pragma once

#include <cuda_fp16.h>
#include <cuda_fp4.h>

#include <cstdint>

#include "../../include/objeta_b200.h"
#include "objb_pipe.cuh"

namespace objb {
namespace dev {

__device__ __forceinline__ float u2f(uint32_t u) { return __uint_as_float(u); }

// IEEE half -> float, exact for every finite and infinite code; equals the
// reference's f16_to_f32_bits (quant.rs:1021-1044) on all non-NaN inputs.
__device__ __forceinline__ float f16_bits_to_f32(uint32_t bits16) {
  return __half2float(__ushort_as_half(static_cast<unsigned short>(bits16 & 0xFFFFu)));
}

// E8M0 -> float (quant.rs:886-892 / deepseek.rs:831-850): raw 0 is 2^-127.
__device__ __forceinline__ float e8m0_to_f32(uint32_t raw) {
  return raw == 0 ? u2f(1u << 22) : u2f(raw << 23);
}

// Small unsigned integer q (< 2^23) minus `off`, as an exact float.
__device__ __forceinline__ float qf(uint32_t q, float off) {
  return u2f(0x4B000000u | q) - (8388608.0f + off);
}

// Byte `i` (compile-time after unrolling) of a little-endian word array.
template <int N>
__device__ __forceinline__ uint32_t byte_at(const uint32_t (&w)[N], int i) {
  return (w[i >> 2] >> ((i & 3) * 8)) & 0xFFu;
}

// A lane's x registers as N 128-bit quads.  Indexed with compile-time
// constants only (after unrolling), so the array stays in registers.
template <int N>
struct Words {
  static constexpr int kQuads = N;
  uint4 q[N];
  __device__ __forceinline__ uint32_t w(int i) const {
    const uint4& v = q[i >> 2];
    switch (i & 3) {
      case 0: return v.x;
      case 1: return v.y;
      case 2: return v.z;
      default: return v.w;
    }
  }
  __device__ __forceinline__ void set(int i, uint32_t val) {
    uint4& v = q[i >> 2];
    switch (i & 3) {
      case 0: v.x = val; break;
      case 1: v.y = val; break;
      case 2: v.z = val; break;
      default: v.w = val; break;
    }
  }
  __device__ __forceinline__ float2 f2(int i) const {
    return make_float2(__uint_as_float(w(2 * i)), __uint_as_float(w(2 * i + 1)));
  }
  __device__ __forceinline__ void set_f2(int i, float2 v) {
    set(2 * i, __float_as_uint(v.x));
    set(2 * i + 1, __float_as_uint(v.y));
  }
};

template <int FMT>
struct Tile;

// ------------------------------------------- integer formats: the digit image
// Q4_0, Q5_0 and IQ3_0 form each block sum exactly in integers.  Every x of a
// block is held as X = rint(x * 2^(20-E)) (2^E > max|x| of the block), split
// into three signed 7-bit digits; a lane keeps, per block, 8 "groups" of four
// elements x 3 digit words (one byte per element) plus the block's 2^(E-20)
// and -off * sum X:  words (b*8 + g)*3 + k, 48 + b, 50 + b of a 13-quad image.
// The row decode unpacks the codes of a group into four bytes (q in 0..31)
// and dp4a-multiplies them with the digit words, so
//   sum_l (q_l - off) x_l = (sum_l q_l X_l - off * sum_l X_l) * 2^(E-20)
// with |sum_l q_l X_l| < 2^30.  The only roundings before the fp32
// accumulation across blocks are that of X (<= 2^-21 of the block's largest
// |x|) and one int -> f32 conversion.  Each format names, for group g and
// byte j, the element of its block (elem) and its offset (kOffset).
using DigitRegs = Words<13>;
__device__ __forceinline__ int dg_word(int b, int g, int k) { return (b * 8 + g) * 3 + k; }

// Block sum for one group set: 8 groups' code bytes against the digits.
__device__ __forceinline__ float digit_block(const uint32_t (&qb)[8], const DigitRegs& xr, int b,
                                             float scale) {
  int q0 = 0, q1 = 0, q2 = 0;
#pragma unroll
  for (int g = 0; g < 8; ++g) {
    const int a = static_cast<int>(qb[g]);
    q0 = __dp4a(a, static_cast<int>(xr.w(dg_word(b, g, 0))), q0);
    q1 = __dp4a(a, static_cast<int>(xr.w(dg_word(b, g, 1))), q1);
    q2 = __dp4a(a, static_cast<int>(xr.w(dg_word(b, g, 2))), q2);
  }
  const int T = q0 + (q1 + q2 * 128) * 128 + static_cast<int>(xr.w(50 + b));
  return __int2float_rn(T) * (scale * __uint_as_float(xr.w(48 + b)));
}

// ------------------------------------------------ wide blocks (exact path)
// Rounding X = rint(x * 2^(20-E)) moves an element by at most half a grid
// step 2^(E-20); a value below half a step rounds to 0 and moves by itself.
// That is harmless while the block's values are comparable, and not when a
// few of them dwarf the rest: an outlier channel of 1e3 among N(0,1) values
// leaves the others only ~10 bits (and at 1e7 none), and the rows that weigh
// the outliers by zero then miss the reference's 1e-5 * sum|w x| bound.
// Per block, with y = x * 2^(20-E) (exact) and in integers, so every image
// builder agrees bit for bit:
//   c = #{l : |y_l| >= 2^-8}     (the values whose rounding error, at most
//                                 half a grid step, is not below 2^-9 of a
//                                 step -- smaller ones move by less than that),
//   R = sum_l min(|X_l|, 2^15)   (the values, each capped at 2^-5 of 2^E),
// and the block is "wide" when c >= 2 and c * 2^13 > R, i.e. the half-step
// rounding of its c values can exceed 2^-14 of its capped mass.  Up to 7
// outliers of up to ~3e6 times the block's ordinary values qualify (beyond
// that an outlier's capped mass hides the others'); an N(0,1) block sits
// about 4x below the line, and values far below the grid (silu of a large
// negative gate) do not count.  A wide block's digit words and block sum are
// zero in the image (it adds nothing to the integer path), its 2^(E-20) word
// holds kWideMark, and the consumer warp adds the block's terms in fp32
// instead, one element per lane: ((q_l - off) * scale) * x_l.
constexpr int kWideCap = 1 << 15;
constexpr float kWideFloor = 0.00390625f;  // 2^-8 of a grid step
constexpr uint32_t kWideMark = 0x80000000u;  // -0.0f: a zero block sum times it stays zero

// The wide test from c and R (above).
__device__ __forceinline__ bool block_is_wide(int c, int R) { return c >= 2 && (c << 13) > R; }

// Code q (unsigned, before the offset) of element l of one block in the
// reference byte layouts (quant.rs:814-879), read with byte loads.
template <int FMT>
__device__ __forceinline__ uint32_t block_code(const uint8_t* blk, int l) {
  if constexpr (FMT == OBJB_Q4_0) {
    return (blk[2 + (l >> 1)] >> ((l & 1) * 4)) & 0xFu;
  } else if constexpr (FMT == OBJB_Q5_0) {
    const uint32_t lo = (blk[6 + (l >> 1)] >> ((l & 1) * 4)) & 0xFu;
    return lo | (((blk[2 + (l >> 3)] >> (l & 7)) & 1u) << 4);
  } else {
    const uint32_t lo = (blk[2 + (l >> 2)] >> (2 * (l & 3))) & 3u;
    return lo | (((blk[10 + (l >> 3)] >> (l & 7)) & 1u) << 2);
  }
}

// Lane l's fp32 term of a wide block, rounded as the reference's dot rows
// round it (quant.rs:950-1019): w = (q_l - off) * scale, then w * x_l.
template <int FMT>
__device__ __forceinline__ float wide_term(const uint8_t* blk, int l, float xl) {
  constexpr float off = FMT == OBJB_Q4_0 ? 8.0f : FMT == OBJB_Q5_0 ? 16.0f : 4.0f;
  const float s = f16_bits_to_f32(blk[0] | (static_cast<uint32_t>(blk[1]) << 8));
  return __fmul_rn(__fmul_rn(qf(block_code<FMT>(blk, l), off), s), xl);
}

// Q5_0 high bits onto bit 4 of the code bytes: bits 0, 2, 4, 6 of hb (the
// low-nibble elements) -> bits 4, 12, 20, 28, and bits 1, 3, 5, 7 (the
// high-nibble elements) -> the same positions.  One multiply each: the
// partial products off the targets never carry into them (checked for every
// hb), and the mask keeps the targets only.
__device__ __forceinline__ uint32_t q5_high_even(uint32_t hb) { return ((hb & 0x55u) * 0x410410u) & 0x10101010u; }
__device__ __forceinline__ uint32_t q5_high_odd(uint32_t hb) { return ((hb & 0xAAu) * 0x208208u) & 0x10101010u; }

// Nibble formats (Q4_0 / Q5_0) share the decode-word layout: in a tile the
// eight decode words are m = [qs0[14], qs0[15], qs0[0], qs0[1]] (a byte
// permute of the two words straddling block 0's scale) and the aligned quant
// words; nibble position p of decode word u is element nib_elem(u, p) of the
// tile, and group g = 2 * uu + h holds the low (h = 0) or high nibbles.
__device__ __forceinline__ int nib_elem(int u, int p) {
  if (u == 0) return p < 4 ? 28 + p : p - 4;
  if (u < 4) return 4 + 8 * (u - 1) + p;
  return 32 + 8 * (u - 4) + p;
}

// ---------------------------------------------------------------- Q4_0
// Tile = 2 blocks = 36 bytes = 9 words:
//   w0 = [s0 lo, s0 hi, qs0[0], qs0[1]]  w1..w3 = qs0[2..13]
//   w4 = [qs0[14], qs0[15], s1 lo, s1 hi]  w5..w8 = qs1[0..15]
// Byte j of qs holds element 2j (low nibble) and 2j+1 (high nibble).
template <>
struct Tile<OBJB_Q4_0> {
  static constexpr int P = 2;
  static constexpr int BB = 18;
  static constexpr int TB = P * BB;
  static constexpr int kOffset = 8;
  using XRegs = DigitRegs;
  __device__ __forceinline__ static int elem(int b, int g, int j) {
    return nib_elem(4 * b + g / 2, 2 * j + (g & 1)) - 32 * b;
  }

  __device__ __forceinline__ static float dot(const uint8_t* t, const XRegs& xr) {
    uint32_t w[9];
#pragma unroll
    for (int i = 0; i < 9; ++i) w[i] = lds32(t + 4 * i);
    const uint32_t D[8] = {__byte_perm(w[0], w[4], 0x3254), w[1], w[2], w[3], w[5], w[6], w[7], w[8]};
    const float s0 = f16_bits_to_f32(w[0]), s1 = f16_bits_to_f32(w[4] >> 16);
    float r = 0.0f;
#pragma unroll
    for (int b = 0; b < 2; ++b) {
      uint32_t qb[8];
#pragma unroll
      for (int uu = 0; uu < 4; ++uu) {
        const uint32_t d = D[4 * b + uu];
        qb[2 * uu] = d & 0x0F0F0F0Fu;
        qb[2 * uu + 1] = (d >> 4) & 0x0F0F0F0Fu;
      }
      r += digit_block(qb, xr, b, b ? s1 : s0);
    }
    return r;
  }
};

// ---------------------------------------------------------------- Q5_0
// Block = [s (2)][qh (4)][qs (16)] (quant.rs:831-858); q = low | high << 4,
// weight (q - 16) * s.  Tile = 2 blocks = 44 bytes = 11 words:
//   w0 = [s0, qh0 b0 b1]  w1 = [qh0 b2 b3, qs0 b0 b1]  w2..w4 = qs0 b2..b13
//   w5 = [qs0 b14 b15, s1]  w6 = qh1  w7..w10 = qs1
// The decode words match Q4_0's element layout; the high bits of a decode
// word's elements are the byte of qh starting at its first element (a funnel
// shift for the merged word), spread onto bit 4 of the nibble bytes.
template <>
struct Tile<OBJB_Q5_0> {
  static constexpr int P = 2;
  static constexpr int BB = 22;
  static constexpr int TB = P * BB;
  static constexpr int kOffset = 16;
  using XRegs = DigitRegs;
  __device__ __forceinline__ static int elem(int b, int g, int j) {
    return nib_elem(4 * b + g / 2, 2 * j + (g & 1)) - 32 * b;
  }

  __device__ __forceinline__ static float dot(const uint8_t* t, const XRegs& xr) {
    uint32_t w[11];
#pragma unroll
    for (int i = 0; i < 11; ++i) w[i] = lds32(t + 4 * i);
    const uint32_t qh[2] = {__byte_perm(w[0], w[1], 0x5432), w[6]};
    const uint32_t D[8] = {__byte_perm(w[1], w[5], 0x3254), w[2], w[3], w[4], w[7], w[8], w[9], w[10]};
    const float s0 = f16_bits_to_f32(w[0]), s1 = f16_bits_to_f32(w[5] >> 16);
    float r = 0.0f;
#pragma unroll
    for (int b = 0; b < 2; ++b) {
      uint32_t qb[8];
#pragma unroll
      for (int uu = 0; uu < 4; ++uu) {
        const uint32_t d = D[4 * b + uu];
        // high bits of the 8 elements of this decode word, element order
        const uint32_t hb = (b == 0 && uu == 0) ? __funnelshift_r(qh[0], qh[0], 28)
                                                : (qh[b] >> (b == 0 ? 4 + 8 * (uu - 1) : 8 * uu));
        qb[2 * uu] = (d & 0x0F0F0F0Fu) | q5_high_even(hb);
        qb[2 * uu + 1] = ((d >> 4) & 0x0F0F0F0Fu) | q5_high_odd(hb);
      }
      r += digit_block(qb, xr, b, b ? s1 : s0);
    }
    return r;
  }
};

// ---------------------------------------------------------------- IQ3_0
// Block = [s (2)][2-bit lows (8)][1-bit highs (4)] (quant.rs:860-879);
// q = low | high << 2, weight (q - 4) * s.  Tile = 2 blocks = 28 bytes:
//   w0 = [s0, L0 b0 b1]  w1 = L0 b2..b5  w2 = [L0 b6 b7, H0 b0 b1]
//   w3 = [H0 b2 b3, s1]  w4, w5 = L1  w6 = H1
// A 32-bit word of lows holds 16 elements; (lw >> 2c) & 0x03030303 are
// elements 4j + c.  The 16 highs of those elements are first moved nibble by
// nibble into bytes (elements 4j .. 4j + 3 in bits 0..3 of byte j: one byte
// permute and one shift-or), so (hs >> c) & 0x01010101 are the highs of
// elements 4j + c.  Group g = 4 * hh + c (hh: which 16 elements).
template <>
struct Tile<OBJB_IQ3_0> {
  static constexpr int P = 2;
  static constexpr int BB = 14;
  static constexpr int TB = P * BB;
  static constexpr int kOffset = 4;
  using XRegs = DigitRegs;
  __device__ __forceinline__ static int elem(int, int g, int j) { return 16 * (g / 4) + 4 * j + (g & 3); }

  __device__ __forceinline__ static float dot(const uint8_t* t, const XRegs& xr) {
    uint32_t w[7];
#pragma unroll
    for (int i = 0; i < 7; ++i) w[i] = lds32(t + 4 * i);
    const uint32_t L[2][2] = {{__byte_perm(w[0], w[1], 0x5432), __byte_perm(w[1], w[2], 0x5432)},
                              {w[4], w[5]}};
    const uint32_t H[2] = {__byte_perm(w[2], w[3], 0x5432), w[6]};
    const float s0 = f16_bits_to_f32(w[0]), s1 = f16_bits_to_f32(w[3] >> 16);
    float r = 0.0f;
#pragma unroll
    for (int b = 0; b < 2; ++b) {
      uint32_t qb[8];
#pragma unroll
      for (int hh = 0; hh < 2; ++hh) {
        const uint32_t v = __byte_perm(H[b], 0u, hh ? 0x4342u : 0x4140u);  // [h b0, 0, h b1, 0] of this half
        const uint32_t hs = (v | (v << 4)) & 0x0F0F0F0Fu;                    // elements 4j..4j+3 in byte j
#pragma unroll
        for (int c = 0; c < 4; ++c)
          qb[4 * hh + c] = ((L[b][hh] >> (2 * c)) & 0x03030303u) | (((hs >> c) & 0x01010101u) << 2);
      }
      r += digit_block(qb, xr, b, b ? s1 : s0);
    }
    return r;
  }
};

// 4 FP4 E2M1 codes (the low 16 bits of u, element order) -> 4 int8 holding
// 2 * value (exact: 0, +-1, +-2, +-3, +-4, +-6, +-8, +-12) by byte-permute
// table lookups; checked for all 65536 inputs.
__device__ __forceinline__ uint32_t prmt_b32(uint32_t a, uint32_t b, uint32_t sel) {
  uint32_t d;
  asm("prmt.b32 %0, %1, %2, %3;" : "=r"(d) : "r"(a), "r"(b), "r"(sel));
  return d;
}
__device__ __forceinline__ uint32_t fp4x4_to_i8x4(uint32_t u) {
  const uint32_t sel = u & 0x7777u;                      // magnitude index per nibble
  const uint32_t pos = prmt_b32(0x03020100u, 0x0C080604u, sel);  // 0 1 2 3 4 6 8 12
  const uint32_t neg = prmt_b32(0xFDFEFF00u, 0xF4F8FAFCu, sel);  // their negatives
  // sign bits (bit 3 of each nibble) on byte sign positions, replicated
  const uint32_t sgn = prmt_b32(u, u << 4, 0x9D8Cu);
  return (pos & ~sgn) | (neg & sgn);
}

// ------------------------------------------------- FP4 E2M1, interleaved
// Block = [E8M0 scale (1)][16 packed bytes] (quant.rs:908-926).  Tile = 2
// blocks = 34 bytes, read as 17 half-words (2-byte aligned).  The E2M1 pairs
// go through the sm_100a hardware e2m1x2 -> f16x2 conversion, which is exact
// (code 8 -> -0.0, as quant.rs's FP4_TABLE).
__device__ __forceinline__ float2 e2m1x2_to_float2(uint32_t byte) {
  __half2_raw h = __nv_cvt_fp4x2_to_halfraw2(static_cast<__nv_fp4x2_storage_t>(byte), __NV_E2M1);
  return __half22float2(*reinterpret_cast<__half2*>(&h));
}

template <>
struct Tile<OBJB_FP4_E2M1> {
  static constexpr int P = 2;
  static constexpr int BB = 17;
  static constexpr int TB = P * BB;
  using XRegs = Words<16>;  // x of the tile as 32 float pairs

  __device__ __forceinline__ static void load_x(const float* __restrict__ x, int col0, bool active,
                                                XRegs& xr) {
#pragma unroll
    for (int i = 0; i < 32; ++i)
      xr.set_f2(i, active ? make_float2(__ldg(x + col0 + 2 * i), __ldg(x + col0 + 2 * i + 1))
                          : make_float2(0.f, 0.f));
  }

  __device__ __forceinline__ static float dot(const uint8_t* t, const XRegs& xr) {
    uint32_t h[17];
#pragma unroll
    for (int i = 0; i < 17; ++i) h[i] = *reinterpret_cast<const uint16_t*>(t + 2 * i);
    float total = 0.0f;
#pragma unroll
    for (int b = 0; b < 2; ++b) {
      const int base = b * BB;
#define OBJB_FP4_BYTE(i) ((h[(i) >> 1] >> (((i) & 1) * 8)) & 0xFFu)
      const float s = e8m0_to_f32(OBJB_FP4_BYTE(base));
      float2 acc = make_float2(0.f, 0.f);
#pragma unroll
      for (int j = 0; j < 16; ++j) {
        const float2 v = e2m1x2_to_float2(OBJB_FP4_BYTE(base + 1 + j));
        acc = __ffma2_rn(v, xr.f2(b * 16 + j), acc);
      }
#undef OBJB_FP4_BYTE
      total = fmaf(acc.x + acc.y, s, total);
    }
    return total;
  }
};


// ------------------------------------------- generic block dot (fallback)
// Reads one block straight from global memory (any alignment) and returns
// sum_l (q_l - off) x_l times the block scale.  Used by the fallback kernel
// for shapes or pointers the TMA path cannot take.
template <int FMT>
__device__ __forceinline__ float block_dot_global(const uint8_t* __restrict__ blk,
                                                  const float* __restrict__ x32) {
  float acc = 0.0f;
  if constexpr (FMT == OBJB_Q4_0) {
    const float s = f16_bits_to_f32(blk[0] | (blk[1] << 8));
#pragma unroll
    for (int j = 0; j < 16; ++j) {
      const uint32_t by = blk[2 + j];
      acc = fmaf(qf(by & 0xFu, 8.0f), __ldg(x32 + 2 * j), acc);
      acc = fmaf(qf(by >> 4, 8.0f), __ldg(x32 + 2 * j + 1), acc);
    }
    return acc * s;
  } else if constexpr (FMT == OBJB_Q5_0) {
    const float s = f16_bits_to_f32(blk[0] | (blk[1] << 8));
    const uint32_t qh = blk[2] | (blk[3] << 8) | (blk[4] << 16) | (static_cast<uint32_t>(blk[5]) << 24);
#pragma unroll
    for (int e = 0; e < 32; ++e) {
      const uint32_t by = blk[6 + e / 2];
      const uint32_t q = ((e & 1) ? (by >> 4) : (by & 0xFu)) | (((qh >> e) & 1u) << 4);
      acc = fmaf(qf(q, 16.0f), __ldg(x32 + e), acc);
    }
    return acc * s;
  } else if constexpr (FMT == OBJB_IQ3_0) {
    const float s = f16_bits_to_f32(blk[0] | (blk[1] << 8));
#pragma unroll
    for (int e = 0; e < 32; ++e) {
      const uint32_t low = (blk[2 + e / 4] >> (2 * (e % 4))) & 3u;
      const uint32_t high = (blk[10 + e / 8] >> (e % 8)) & 1u;
      acc = fmaf(qf(low | (high << 2), 4.0f), __ldg(x32 + e), acc);
    }
    return acc * s;
  } else {
    const float s = e8m0_to_f32(blk[0]);
#pragma unroll
    for (int j = 0; j < 16; ++j) {
      const float2 v = e2m1x2_to_float2(blk[1 + j]);
      acc = fmaf(v.x, __ldg(x32 + 2 * j), acc);
      acc = fmaf(v.y, __ldg(x32 + 2 * j + 1), acc);
    }
    return acc * s;
  }
}

}  // namespace dev
}  // namespace objb
