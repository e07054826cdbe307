// objb_official.cuh -- the official DeepSeek arithmetic on the device:
// activations quantized to F8_E4M3 with one E8M0 scale per 128 values
// (act_quant), FP8 activation x FP4 weight row dots (routed experts) and FP8 x
// FP8 row dots (shared expert).  Codecs follow the reference CPU functions
// (crates/objeta-parser/src/deepseek.rs:799-825, 1444-1525), including their
// quirks: E4M3 exponent-0 codes decode as m * 2^-5, exponent-15 codes as
// +-448, and the encoder flushes |v| < 2^-7 to zero.
#pragma once

#include <cstdint>

#include "objb_gemv.cuh"

namespace objb {
namespace dev {

// deepseek.rs:1444-1481 (f32_to_f8e4m3_exact), operation for operation.
__device__ __forceinline__ uint32_t f32_to_e4m3_ref(float v) {
  const float a = fabsf(v);
  if (a < 1.0f / 128.0f) {
    const uint32_t sign = v < 0.0f ? 0x80u : 0u;
    const float r = roundf(a * 16.0f);  // Rust f32::round: half away from zero
    uint32_t q = (r != r || r <= 0.0f) ? 0u : (r >= 255.0f ? 255u : static_cast<uint32_t>(r));
    q = min(q, 7u);
    return sign | q;
  }
  if (a >= 448.0f) return v < 0.0f ? 0xFEu : 0x7Eu;
  const uint32_t sign = v < 0.0f ? 0x80u : 0u;
  const uint32_t bits = __float_as_uint(a);
  int exp_f8 = static_cast<int>((bits >> 23) & 0xFFu) - 127 + 7;
  if (exp_f8 < 0) exp_f8 = 0;
  uint32_t mant3 = ((bits & 0x7FFFFFu) + (1u << 19)) >> 20;
  uint32_t exp_final = static_cast<uint32_t>(exp_f8) & 0xFFu;
  if (mant3 >= 8u) {
    mant3 = 0u;
    exp_final = exp_final == 255u ? 255u : exp_final + 1u;
  }
  if (exp_final > 14u) {
    exp_final = 14u;
    mant3 = 7u;
  }
  return (sign | (exp_final << 3) | (mant3 & 7u)) & 0xFFu;
}

// The reference E4M3 value (deepseek.rs:799-825) times 2^9, as an exact
// integer: exponent 0 -> 16 m, exponent 15 -> 229376 (448 * 2^9), otherwise
// (8 + m) * 2^(e - 1).  |result| < 2^18.
__device__ __forceinline__ int e4m3_ref_times512(uint32_t c) {
  const uint32_t e = (c >> 3) & 15u, m = c & 7u;
  const int a = e == 0u ? static_cast<int>(16u * m)
                        : (e == 15u ? 229376 : static_cast<int>((8u + m) << (e - 1u)));
  return (c & 0x80u) ? -a : a;
}

// The reference E4M3 value as f32.
__device__ __forceinline__ float e4m3_ref_to_f32(uint32_t c) {
  return ldexpf(static_cast<float>(e4m3_ref_times512(c)), -9);
}

// ceil(log2(y)) for finite y > 0 as glibc log2f + ceilf gives it: the double
// log2 rounded to f32 has the same ceiling for every positive finite float.
__device__ __forceinline__ int ceil_log2_ref(float y) {
  const float c = ceilf(static_cast<float>(log2(static_cast<double>(y))));
  if (c != c) return 0;
  if (c >= 2147483647.0f) return 2147483647;
  if (c <= -2147483648.0f) return -2147483647 - 1;
  return static_cast<int>(c);
}

// ---- FP8 activation x FP4 weight (split layout [rows, K/2] + E8M0 [rows, K/32])
//
// Exact integer block sums: A = act * 2^9 (an integer, see above) is held as
// three signed 7-bit digits; the weight codes become 2 * FP4 value (an int8 in
// [-12, 12]) by a byte-permute table lookup; dp4a forms sum (2w) A exactly and
// the block's f32 contribution is S * (w_scale * act_scale * 2^-10).
//
// Image of a lane tile (blocks b0 and b0 + 32 of the lane, as RowDotSplitFp4Digit):
// words (j * 8 + g) * 3 + k = digit k of elements 4g .. 4g+3 of block slot j,
// word 48 + j = act_scale(block) * 2^-10 as f32, word 50 + j = 0.

// fp4x4_to_i8x4 (objb_decode.cuh): 4 FP4 codes -> 4 int8 (2 * value).

struct RowDotFp8Fp4 {
  using XRegs = DigitRegs;
  int b0, nblocks;
  __device__ __forceinline__ void init(const RowLayout& L, int seg, int lane) {
    b0 = seg * 64 + lane;
    nblocks = L.nblocks;
  }
  __device__ __forceinline__ float dot(const uint8_t* wrow, const uint8_t* srow, const XRegs& xr) const {
    float r = 0.0f;
#pragma unroll
    for (int j = 0; j < 2; ++j) {
      const int b = b0 + 32 * j;
      if (b < nblocks) {
        const uint4 q = *reinterpret_cast<const uint4*>(wrow + 16 * b);
        const uint32_t qw[4] = {q.x, q.y, q.z, q.w};
        int a0 = 0, a1 = 0, a2 = 0;
#pragma unroll
        for (int w = 0; w < 4; ++w) {
#pragma unroll
          for (int h = 0; h < 2; ++h) {
            const int g = 2 * w + h;
            const int v = static_cast<int>(fp4x4_to_i8x4(h ? (qw[w] >> 16) : qw[w]));
            a0 = __dp4a(v, static_cast<int>(xr.w((j * 8 + g) * 3 + 0)), a0);
            a1 = __dp4a(v, static_cast<int>(xr.w((j * 8 + g) * 3 + 1)), a1);
            a2 = __dp4a(v, static_cast<int>(xr.w((j * 8 + g) * 3 + 2)), a2);
          }
        }
        const int S = a0 + (a1 + a2 * 128) * 128;
        r = fmaf(__int2float_rn(S), e8m0_to_f32(srow[b]) * __uint_as_float(xr.w(48 + j)), r);
      }
    }
    return r;
  }
};

}  // namespace dev
}  // namespace objb
