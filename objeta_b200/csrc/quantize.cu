// quantize.cu -- device packers (QuantBackend::quantize_matrix) and the FP4
// split-layout decode, byte- / bit-identical to the reference CPU code.
//
// This file is compiled with -fmad=false: every f32 expression below rounds
// after each operation, as the Rust code it follows does.
#include <cuda_runtime.h>

#include <cstdint>
#include <string>

#include "objb_common.h"
#include "objb_launch.h"

namespace objb {
namespace dev {

// f32_to_f16_bits (quant.rs:1046-1079): truncate, then add one when mantissa
// bit 12 is set (half-up on magnitude).
__device__ __forceinline__ uint32_t f32_to_f16_bits_ref(float value) {
  const uint32_t bits = __float_as_uint(value);
  const uint32_t sign = (bits >> 16) & 0x8000u;
  const int exp = static_cast<int>((bits >> 23) & 0xFFu);
  const uint32_t mant = bits & 0x7FFFFFu;
  if (exp == 255) return sign | 0x7C00u | (mant == 0 ? 0u : 0x0200u);
  const int half_exp = exp - 127 + 15;
  if (half_exp >= 0x1F) return sign | 0x7C00u;
  if (half_exp <= 0) {
    if (half_exp < -10) return sign;
    const uint32_t mantissa = mant | 0x800000u;
    const uint32_t shift = static_cast<uint32_t>(14 - half_exp);
    uint32_t half = (mantissa >> shift) & 0xFFFFu;
    if ((mantissa >> (shift - 1)) & 1u) half = (half + 1u) & 0xFFFFu;
    return (sign | half) & 0xFFFFu;
  }
  uint32_t half = (sign | (static_cast<uint32_t>(half_exp) << 10) | (mant >> 13)) & 0xFFFFu;
  if (mant & 0x1000u) half = (half + 1u) & 0xFFFFu;
  return half;
}

// Rust `v.round().clamp(lo, hi) as u8` (round half away from zero,
// saturating cast, NaN -> 0).
__device__ __forceinline__ uint32_t round_clamp_u8(float v, float lo, float hi) {
  float r = roundf(v);
  if (r != r) return 0u;
  r = fmaxf(lo, fminf(hi, r));
  return static_cast<uint32_t>(r);
}

__device__ __forceinline__ float block_amax(const float* src) {
  float amax = 0.0f;
#pragma unroll
  for (int i = 0; i < 32; ++i) amax = fmaxf(amax, fabsf(src[i]));  // f32::max ignores NaN
  return amax;
}

// quant.rs:881-884, code 8 = -0.0.
__constant__ float kFp4Table[16] = {0.0f,  0.5f,  1.0f,  1.5f,  2.0f,  3.0f,  4.0f,  6.0f,
                                   -0.0f, -0.5f, -1.0f, -1.5f, -2.0f, -3.0f, -4.0f, -6.0f};
// objeta-parser deepseek.rs:789-792, code 8 = +0.0.
__constant__ float kFp4ParserTable[16] = {0.0f, 0.5f,  1.0f,  1.5f,  2.0f,  3.0f,  4.0f,  6.0f,
                                          0.0f, -0.5f, -1.0f, -1.5f, -2.0f, -3.0f, -4.0f, -6.0f};

// One thread packs one 32-value block.
template <int FMT>
__global__ void quantize_kernel(const float* __restrict__ m, uint8_t* __restrict__ out,
                                size_t nblocks_total) {
  const size_t g = blockIdx.x * static_cast<size_t>(blockDim.x) + threadIdx.x;
  if (g >= nblocks_total) return;
  float src[32];
  const float4* s4 = reinterpret_cast<const float4*>(m + g * 32);
  const bool al = (reinterpret_cast<uintptr_t>(m) & 15u) == 0;
#pragma unroll
  for (int i = 0; i < 8; ++i) {
    if (al) {
      const float4 v = s4[i];
      src[4 * i] = v.x;
      src[4 * i + 1] = v.y;
      src[4 * i + 2] = v.z;
      src[4 * i + 3] = v.w;
    } else {
      src[4 * i] = m[g * 32 + 4 * i];
      src[4 * i + 1] = m[g * 32 + 4 * i + 1];
      src[4 * i + 2] = m[g * 32 + 4 * i + 2];
      src[4 * i + 3] = m[g * 32 + 4 * i + 3];
    }
  }
  const float amax = block_amax(src);
  if constexpr (FMT == OBJB_Q4_0) {  // quant.rs:814-829
    uint8_t* d = out + g * 18;
    const float scale = amax > 0.0f ? __fdiv_rn(amax, 7.0f) : 1.0e-10f;
    const uint32_t s16 = f32_to_f16_bits_ref(scale);
    d[0] = s16 & 0xFF;
    d[1] = s16 >> 8;
#pragma unroll
    for (int i = 0; i < 16; ++i) {
      const uint32_t q0 = round_clamp_u8(__fadd_rn(__fdiv_rn(src[2 * i], scale), 8.0f), 0.0f, 15.0f);
      const uint32_t q1 = round_clamp_u8(__fadd_rn(__fdiv_rn(src[2 * i + 1], scale), 8.0f), 0.0f, 15.0f);
      d[2 + i] = static_cast<uint8_t>(q0 | (q1 << 4));
    }
  } else if constexpr (FMT == OBJB_Q5_0) {  // quant.rs:831-858
    uint8_t* d = out + g * 22;
    const float scale = amax > 0.0f ? __fdiv_rn(amax, 15.0f) : 1.0e-10f;
    const uint32_t s16 = f32_to_f16_bits_ref(scale);
    uint32_t qh = 0;
    uint8_t qs[16];
#pragma unroll
    for (int i = 0; i < 16; ++i) qs[i] = 0;
#pragma unroll
    for (int i = 0; i < 32; ++i) {
      const uint32_t q = round_clamp_u8(__fadd_rn(__fdiv_rn(src[i], scale), 16.0f), 0.0f, 31.0f);
      const uint32_t low = q & 0xFu;
      if (i % 2 == 0) qs[i / 2] = static_cast<uint8_t>(low);
      else qs[i / 2] = static_cast<uint8_t>(qs[i / 2] | (low << 4));
      qh |= ((q >> 4) & 1u) << i;
    }
    d[0] = s16 & 0xFF;
    d[1] = s16 >> 8;
    d[2] = qh & 0xFF;
    d[3] = (qh >> 8) & 0xFF;
    d[4] = (qh >> 16) & 0xFF;
    d[5] = qh >> 24;
#pragma unroll
    for (int i = 0; i < 16; ++i) d[6 + i] = qs[i];
  } else if constexpr (FMT == OBJB_IQ3_0) {  // quant.rs:860-879
    uint8_t* d = out + g * 14;
    const float scale = amax > 0.0f ? __fdiv_rn(amax, 4.0f) : 1.0e-10f;
    const uint32_t s16 = f32_to_f16_bits_ref(scale);
    uint32_t lo0 = 0, lo1 = 0, hi = 0;
#pragma unroll
    for (int i = 0; i < 32; ++i) {
      const uint32_t q = round_clamp_u8(__fadd_rn(__fdiv_rn(src[i], scale), 4.0f), 0.0f, 7.0f);
      if (i < 16) lo0 |= (q & 3u) << (2 * i);
      else lo1 |= (q & 3u) << (2 * (i - 16));
      hi |= ((q >> 2) & 1u) << i;
    }
    d[0] = s16 & 0xFF;
    d[1] = s16 >> 8;
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      d[2 + j] = (lo0 >> (8 * j)) & 0xFF;
      d[6 + j] = (lo1 >> (8 * j)) & 0xFF;
      d[10 + j] = (hi >> (8 * j)) & 0xFF;
    }
  } else {  // quant.rs:908-926
    uint8_t* d = out + g * 17;
    uint32_t raw = 0;
    if (amax > 0.0f && isfinite(amax)) {
      // ceil(log2f(amax / 6)): log2 in double rounded to f32 equals glibc's
      // log2f under ceil for every positive finite f32 (checked exhaustively
      // on the host); the cast saturates like Rust's `as i32`.
      const float y = __fdiv_rn(amax, 6.0f);
      const float c = ceilf(__double2float_rn(log2(static_cast<double>(y))));
      const int k = static_cast<int>(c);
      const int r = k + 127;
      raw = static_cast<uint32_t>(r < 0 ? 0 : (r > 255 ? 255 : r));
    }
    const float actual = raw == 0 ? __uint_as_float(1u << 22) : __uint_as_float(raw << 23);
    d[0] = static_cast<uint8_t>(raw);
#pragma unroll
    for (int i = 0; i < 16; ++i) {
      uint32_t qq[2];
#pragma unroll
      for (int h = 0; h < 2; ++h) {
        const float scaled = __fdiv_rn(src[2 * i + h], actual);
        uint32_t best = 0;
        float min_diff = __int_as_float(0x7F800000);
#pragma unroll
        for (int q = 0; q < 16; ++q) {
          const float diff = fabsf(__fsub_rn(scaled, kFp4Table[q]));
          if (diff < min_diff) {
            min_diff = diff;
            best = q;
          }
        }
        qq[h] = best;
      }
      d[1 + i] = static_cast<uint8_t>(qq[0] | (qq[1] << 4));
    }
  }
}

// decode_deepseek_fp4_to_f32 (deepseek.rs:862-918), block 32: one thread per
// packed byte, two outputs each.
__global__ void fp4_decode_split_kernel(const uint8_t* __restrict__ w, const uint8_t* __restrict__ s,
                                        float* __restrict__ out, size_t rows, size_t cols) {
  const size_t phys = cols / 2;
  const size_t total = rows * phys;
  for (size_t i = blockIdx.x * static_cast<size_t>(blockDim.x) + threadIdx.x; i < total;
       i += static_cast<size_t>(gridDim.x) * blockDim.x) {
    const size_t r = i / phys, gcol = i % phys;
    const uint32_t b = w[i];
    const size_t lo = gcol * 2;
    const uint32_t raw = s[r * (cols / 32) + lo / 32];
    // f8e8m0_to_f32 (deepseek.rs:831-850): 0 -> 2^-127, 255 -> +inf.
    const float sc = raw == 0 ? __uint_as_float(1u << 22)
                              : (raw == 255 ? __uint_as_float(0x7F800000u) : __uint_as_float(raw << 23));
    // 0 * inf (codes 0 / 8 with scale byte 255) is NaN; the reference decode
    // runs on x86 hosts, whose SSE multiply returns the default NaN 0xFFC00000,
    // so that exact pattern is written instead of the GPU's canonical NaN.
    float v0 = __fmul_rn(kFp4ParserTable[b & 0xFu], sc);
    float v1 = __fmul_rn(kFp4ParserTable[(b >> 4) & 0xFu], sc);
    if (v0 != v0) v0 = __uint_as_float(0xFFC00000u);
    if (v1 != v1) v1 = __uint_as_float(0xFFC00000u);
    out[r * cols + lo] = v0;
    out[r * cols + lo + 1] = v1;
  }
}

}  // namespace dev
}  // namespace objb

extern "C" {

int objb_quantize_matrix_device(int fmt, const float* d_matrix, size_t rows, size_t cols,
                                void* d_out, objb_stream_t stream_) {
  objb::clear_error();
  OBJB_TRY(objb::validate_gemv_shape(fmt, rows, cols));
  if (rows == 0) return OBJB_OK;
  if (!d_matrix || !d_out) return OBJB_FAIL(OBJB_ERR_INVALID_INPUT, "objb_quantize_matrix_device", "null device pointer");
  cudaStream_t stream = static_cast<cudaStream_t>(stream_);
  const size_t nb = rows * (cols / 32);
  const unsigned threads = 128;
  const size_t grid = (nb + threads - 1) / threads;
  if (grid > 0x7FFFFFFFu) return OBJB_FAIL(OBJB_ERR_INVALID_INPUT, "objb_quantize_matrix_device", "matrix too large");
  uint8_t* o = static_cast<uint8_t*>(d_out);
  switch (fmt) {
    case OBJB_Q4_0: objb::dev::quantize_kernel<OBJB_Q4_0><<<grid, threads, 0, stream>>>(d_matrix, o, nb); break;
    case OBJB_Q5_0: objb::dev::quantize_kernel<OBJB_Q5_0><<<grid, threads, 0, stream>>>(d_matrix, o, nb); break;
    case OBJB_IQ3_0: objb::dev::quantize_kernel<OBJB_IQ3_0><<<grid, threads, 0, stream>>>(d_matrix, o, nb); break;
    default: objb::dev::quantize_kernel<OBJB_FP4_E2M1><<<grid, threads, 0, stream>>>(d_matrix, o, nb); break;
  }
  OBJB_CUDA(cudaGetLastError(), "launch quantize kernel");
  return OBJB_OK;
}

int objb_fp4_decode_split_device(const void* d_weight, const void* d_scale, size_t rows,
                                 size_t cols, float* d_out, objb_stream_t stream_) {
  objb::clear_error();
  if (cols % 32 != 0)
    return OBJB_FAIL(OBJB_ERR_INVALID_INPUT, "validate FP4 decode shape",
                     "logical columns " + std::to_string(cols) + " must be divisible by block_size 32");
  if (rows == 0) return OBJB_OK;
  if (!d_weight || !d_scale || !d_out) return OBJB_FAIL(OBJB_ERR_INVALID_INPUT, "objb_fp4_decode_split_device", "null device pointer");
  const size_t total = rows * (cols / 2);
  size_t grid = (total + 255) / 256;
  if (grid > 148 * 64) grid = 148 * 64;
  objb::dev::fp4_decode_split_kernel<<<static_cast<unsigned>(grid), 256, 0, static_cast<cudaStream_t>(stream_)>>>(
      static_cast<const uint8_t*>(d_weight), static_cast<const uint8_t*>(d_scale), d_out, rows, cols);
  OBJB_CUDA(cudaGetLastError(), "launch FP4 decode kernel");
  return OBJB_OK;
}

}  // extern "C"
