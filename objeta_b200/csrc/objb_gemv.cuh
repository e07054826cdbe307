// objb_gemv.cuh -- the batch-1 block-dequant GEMV pipeline for sm_100a.
//
// One persistent CTA per SM streams a contiguous range of rows through a ring
// of shared-memory stages with 1-D bulk TMA copies (cp.async.bulk, one
// elected producer thread, mbarrier completion, L2 evict-first policy).  The
// consumer warps keep the x values of their lane tiles in registers for the
// whole kernel, decode each row's blocks in registers, reduce the row across
// the lanes that share it with warp shuffles and across column segments in
// shared memory, in a fixed order, so results are bit-stable run to run.
//
// The same pipeline runs the MoE kernels: a "job" is one matrix (plus an
// optional second matrix with identical shape whose rows are consumed in the
// same pass) and an epilogue that receives finished row values.
#pragma once

#include <cstdint>
#include <type_traits>
#include <utility>

#include "objb_decode.cuh"
#include "objb_pipe.cuh"

namespace objb {
namespace dev {

constexpr int kMaxSlots = 4;
constexpr int kMaxConsumerWarps = 15;  // + 1 producer = 16 warps: 4 per SM sub-partition, 128 registers each
constexpr int kMaxRowsPerStage = 64;

// Geometry of one streamed matrix, decided on the host.
struct RowLayout {
  int rows, cols;
  int nblocks;      // cols / 32
  int row_bytes;    // packed bytes per row (weights)
  int srow_bytes;   // split-FP4 scale bytes per row (0 otherwise)
  int nseg;         // column segments (warps per row)
  int lpr;          // lanes per row slot (power of two, <= 32)
  int rpw;          // rows per warp step = 32 / lpr
  int ngrp;         // row groups; consumer warps = nseg * ngrp
  int tstage;       // rows per pipeline stage
  int nslots;       // ring depth
  int stage_bytes;  // bytes of one ring slot (weights + scales of tstage rows)
};

struct SmemPlan {
  uint64_t* full;
  uint64_t* empty;
  uint64_t* img_done;  // every consumer warp holds its x registers (in-kernel x images)
  unsigned* abort;     // CTA-local: a wait of this CTA gave up or a stage was completed without data
  float* red;      // [nslots][tstage][nseg][2]
  uint8_t* stage;  // [nslots][stage_bytes]
};

// 64-bit barrier words at the start of the pipelined kernel's shared memory
// (full and empty per slot, img_done, the abort word).
constexpr int kPipeBarrierWords = 2 * kMaxSlots + 2;

__device__ __forceinline__ SmemPlan carve_smem(uint8_t* base, const RowLayout& L, int nred) {
  SmemPlan p;
  p.full = reinterpret_cast<uint64_t*>(base);
  p.empty = p.full + kMaxSlots;
  p.img_done = p.empty + kMaxSlots;
  p.abort = reinterpret_cast<unsigned*>(p.img_done + 1);
  p.red = reinterpret_cast<float*>(base + kPipeBarrierWords * sizeof(uint64_t));
  size_t red_bytes = static_cast<size_t>(L.nslots) * L.tstage * L.nseg * nred * sizeof(float);
  size_t off = kPipeBarrierWords * sizeof(uint64_t) + red_bytes;
  off = (off + 127) & ~static_cast<size_t>(127);
  p.stage = base + off;
  return p;
}

// Per-format adapter: x registers and the lane-partial dot of one row.  Lane
// `lane` of column segment `seg` owns lane tile lt = seg * 32 + lane.  The x
// registers of every lane tile are built once per x vector by
// ximage_kernel ("x image", quad q of tile lt at img[q * nseg * 32 + lt]) and
// loaded by each consumer lane with coalesced 128-bit loads.
template <int FMT>
struct RowDot {
  using T = Tile<FMT>;
  using XRegs = typename T::XRegs;
  int tile_off;  // byte offset of this lane's tile inside a row
  bool active;
  __device__ __forceinline__ void init(const RowLayout& L, int seg, int lane) {
    const int lt = seg * 32 + lane;
    active = (lt * T::P) < L.nblocks;
    tile_off = lt * T::TB;
  }
  // First x column of quad q of tile lt (natural order tiles), -1 if idle.
  __device__ __forceinline__ static int quad_col(const RowLayout& L, int lt, int q) {
    return (lt * T::P) < L.nblocks ? lt * T::P * 32 + 4 * q : -1;
  }
  __device__ __forceinline__ float dot(const uint8_t* wrow, const uint8_t*, const XRegs& xr) const {
    return active ? T::dot(wrow + tile_off, xr) : 0.0f;
  }
};

template <class RD>
struct IsDigitRD {
  static constexpr bool value = false;
  static constexpr int fmt = -1;
};
template <int FMT>
struct IsDigitRD<RowDot<FMT>> {
  static constexpr bool value = FMT != OBJB_FP4_E2M1;
  static constexpr int fmt = FMT;
};


// Split FP4 E2M1 rows on the integer path: x as the digits of
// X = rint(x * 2^(20-E)) (the digit image of Q4_0 / Q5_0 / IQ3_0), the codes
// as 2 * value in int8 (fp4x4_to_i8x4), their products summed exactly by
// dp4a; one int -> f32 conversion and one FMA by scale * 2^(E-21) per block.
// A lane owns P blocks b = seg * 32 P + lane + 32 j (j < P): consecutive
// lanes read consecutive 16-byte blocks (conflict-free 128-bit shared loads);
// P = 1 spreads a row over twice the warps (the MoE down rows, whose CTAs own
// few rows per expert).  Its image: words (j * 8 + g) * 3 + k = digit k of
// elements 4g .. 4g+3 of slot j; word 24 P + j = 2^(E-21) of slot j's block
// (kWideMark for a wide block, NaN for a block that is not finite).
template <int P_>
struct RowDotSplitFp4DigitT {
  static constexpr int P = P_;
  static constexpr int kBlocksPerLane = P;
  using XRegs = Words<(25 * P + 3) / 4>;
  int b0, nblocks;
  __device__ __forceinline__ void init(const RowLayout& L, int seg, int lane) {
    b0 = seg * 32 * P + lane;
    nblocks = L.nblocks;
  }
  __device__ __forceinline__ static int scale_word(int j) { return 24 * P + j; }
  __device__ __forceinline__ float dot(const uint8_t* wrow, const uint8_t* srow, const XRegs& xr) const {
    float r = 0.0f;
#pragma unroll
    for (int j = 0; j < P; ++j) {
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
        r = fmaf(__int2float_rn(S), e8m0_to_f32(srow[b]) * __uint_as_float(xr.w(scale_word(j))), r);
      }
    }
    return r;
  }
};
using RowDotSplitFp4Digit = RowDotSplitFp4DigitT<2>;

template <class RD>
struct IsSplitDigitRD : std::false_type {};
template <int P>
struct IsSplitDigitRD<RowDotSplitFp4DigitT<P>> : std::true_type {};

// Dense bf16 rows (the shared expert of a DeepSeek-style layer; not a
// reference QuantFormat).  A lane reads CPL 16-byte chunks (8 columns each)
// c0 + 32 i, i < CPL, so consecutive lanes read consecutive chunks
// (conflict-free 128-bit shared loads); its 8 CPL x values are the matching
// columns, as float pairs.  CPL = 8 puts 2048 columns on a warp; fewer chunks
// per lane spread a wide row over more warps (a stage then holds few rows,
// and the host picks the CPL that keeps every warp busy).
__device__ __forceinline__ float2 bf16x2_to_float2(uint32_t w) {
  return make_float2(__uint_as_float(w << 16), __uint_as_float(w & 0xFFFF0000u));
}

template <int CPL>
struct RowDotBf16T {
  static constexpr int kChunksPerLane = CPL;
  using XRegs = Words<2 * CPL>;
  int c0, nchunks;
  __device__ __forceinline__ void init(const RowLayout& L, int seg, int lane) {
    c0 = seg * 32 * CPL + lane;
    nchunks = L.cols / 8;
  }
  __device__ __forceinline__ static int quad_col(const RowLayout& L, int lt, int q) {
    const int c = (lt / 32) * 32 * CPL + (q / 2) * 32 + lt % 32;
    return c < L.cols / 8 ? c * 8 + 4 * (q % 2) : -1;
  }
  __device__ __forceinline__ float dot(const uint8_t* wrow, const uint8_t*, const XRegs& xr) const {
    float2 a0 = make_float2(0.f, 0.f), a1 = make_float2(0.f, 0.f);
#pragma unroll
    for (int i = 0; i < CPL; ++i) {
      const int c = c0 + 32 * i;
      if (c < nchunks) {
        const uint4 v = *reinterpret_cast<const uint4*>(wrow + 16 * c);
        a0 = __ffma2_rn(bf16x2_to_float2(v.x), xr.f2(4 * i + 0), a0);
        a1 = __ffma2_rn(bf16x2_to_float2(v.y), xr.f2(4 * i + 1), a1);
        a0 = __ffma2_rn(bf16x2_to_float2(v.z), xr.f2(4 * i + 2), a0);
        a1 = __ffma2_rn(bf16x2_to_float2(v.w), xr.f2(4 * i + 3), a1);
      }
    }
    return (a0.x + a0.y) + (a1.x + a1.y);
  }
};
using RowDotBf16 = RowDotBf16T<8>;

template <class XR>
__device__ __forceinline__ void load_ximage(const uint4* __restrict__ img, int ntp, int lt, XR& xr) {
#pragma unroll
  for (int q = 0; q < XR::kQuads; ++q) xr.q[q] = __ldg(img + q * ntp + lt);
}

// x-image builders.  The image of vector v is quads img[v * img_stride_quads +
// q * ntp + lt] (ntp = nseg * 32 lane tiles).  Both kernels start their
// dependents immediately: the consumer kernel is launched with programmatic
// stream serialization and waits (griddepcontrol.wait) before reading the
// image, so its launch and first weight copies overlap the build.
//
// Float tiles: one thread per (vector, tile, quad); quad q of a tile is four
// consecutive x values whose first column RD::quad_col gives (-1: zeros).
template <class RD>
__global__ void __launch_bounds__(256) ximage_f32_kernel(const RowLayout L, const float* __restrict__ x,
                                                         size_t x_stride, int nvec, uint4* __restrict__ img,
                                                         size_t img_stride_quads, const int32_t* count) {
  asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
  // x may be the output of the kernel this one was launched behind.
  asm volatile("griddepcontrol.wait;" ::: "memory");
  if (count) nvec = min(max(*count, 0), nvec);  // vectors to build (device), at most nvec
  constexpr int NQ = RD::XRegs::kQuads;
  const int ntp = L.nseg * 32;
  const int total = nvec * ntp * NQ;
  for (int idx = blockIdx.x * blockDim.x + threadIdx.x; idx < total; idx += gridDim.x * blockDim.x) {
    const int v = idx / (ntp * NQ);
    const int r = idx % (ntp * NQ);
    const int q = r / ntp, lt = r % ntp;
    const int c = RD::quad_col(L, lt, q);
    float4 f = make_float4(0.f, 0.f, 0.f, 0.f);
    if (c >= 0) {
      const float* src = x + v * x_stride + c;
      f = make_float4(__ldg(src), __ldg(src + 1), __ldg(src + 2), __ldg(src + 3));
    }
    img[v * img_stride_quads + static_cast<size_t>(q) * ntp + lt] =
        make_uint4(__float_as_uint(f.x), __float_as_uint(f.y), __float_as_uint(f.z), __float_as_uint(f.w));
  }
}

// Digit images (Q4_0 / Q5_0 / IQ3_0): one warp per 32-value block.  Lane e
// holds x_e; the warp forms the block's exponent, X_e = rint(x_e * 2^(20-E)),
// its three signed 7-bit digits and sum X; lanes 0..23 then assemble the 24
// digit words of the block (group g, digit k -> word (b*8 + g)*3 + k, byte j
// = element Tile::elem(b, g, j)) and lanes 24 / 25 the block's 2^(E-20) and
// -offset * sum X.  A wide block (block_is_wide) gets zero digits and sum and
// kWideMark in place of 2^(E-20).
template <int FMT>
__global__ void __launch_bounds__(256) ximage_digits_kernel(const RowLayout L, const float* __restrict__ x,
                                                            size_t x_stride, int nvec, uint4* __restrict__ img,
                                                            size_t img_stride_quads, const int32_t* count) {
  asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
  // x may be the output of the kernel this one was launched behind.
  asm volatile("griddepcontrol.wait;" ::: "memory");
  if (count) nvec = min(max(*count, 0), nvec);  // vectors to build (device), at most nvec
  using T = Tile<FMT>;
  const int ntp = L.nseg * 32;
  const int nb_img = ntp * T::P;  // blocks covered by the image (incl. idle lanes)
  const int lane = threadIdx.x & 31;
  const int warps = (gridDim.x * blockDim.x) >> 5;
  for (int wi = (blockIdx.x * blockDim.x + threadIdx.x) >> 5; wi < nvec * nb_img; wi += warps) {
    const int v = wi / nb_img, gb = wi % nb_img;
    const float xe = gb < L.nblocks ? __ldg(x + v * x_stride + gb * 32 + lane) : 0.0f;
    float m = fabsf(xe);
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) m = fmaxf(m, __shfl_xor_sync(0xFFFFFFFFu, m, o));
    int E = 0;
    frexpf(m, &E);  // m < 2^E (E = 0 for m = 0)
    const float y = ldexpf(xe, 20 - E);
    const int X0 = __float2int_rn(y);
    const int cnt = __popc(__ballot_sync(0xFFFFFFFFu, fabsf(y) >= kWideFloor));
    const int capped = __reduce_add_sync(0xFFFFFFFFu, min(abs(X0), kWideCap));
    const bool wide = isfinite(m) && block_is_wide(cnt, capped);
    const int X = wide ? 0 : X0;
    const int d0 = ((X + 64) & 127) - 64;
    const int X1 = (X - d0) / 128;
    const int d1 = ((X1 + 64) & 127) - 64;
    const int d2 = (X1 - d1) / 128;
    const int sx = __reduce_add_sync(0xFFFFFFFFu, X);
    const int lt = gb / T::P, b = gb % T::P;
    const int t = lane < 24 ? lane : 0;  // word t = g * 3 + k of this block
    const int g = t / 3, k = t % 3;
    uint32_t word = 0;
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      const int el = T::elem(b, g, j);
      const int s0 = __shfl_sync(0xFFFFFFFFu, d0, el);
      const int s1 = __shfl_sync(0xFFFFFFFFu, d1, el);
      const int s2 = __shfl_sync(0xFFFFFFFFu, d2, el);
      const int dk = k == 0 ? s0 : (k == 1 ? s1 : s2);
      word |= (static_cast<uint32_t>(dk) & 0xFFu) << (8 * j);
    }
    uint32_t* out = reinterpret_cast<uint32_t*>(img + v * img_stride_quads);
    int widx = -1;
    uint32_t val = 0;
    if (lane < 24) {
      widx = dg_word(b, g, k);
      val = word;
    } else if (lane == 24) {
      widx = 48 + b;
      val = wide ? kWideMark : __float_as_uint(isfinite(m) ? ldexpf(1.0f, E - 20) : __int_as_float(0x7FC00000));
    } else if (lane == 25) {
      widx = 50 + b;
      val = static_cast<uint32_t>(-T::kOffset * sx);
    }
    if (widx >= 0) out[(static_cast<size_t>(widx >> 2) * ntp + lt) * 4 + (widx & 3)] = val;
  }
}

// Digit images of split FP4 rows (RowDotSplitFp4DigitT<P>): one warp per
// (vector, block); the block's X, its digits and the wide test as in
// ximage_digits_kernel; group g of slot j holds elements 4g .. 4g+3, and the
// slot's scale word is 2^(E-21) (the weights enter as 2 * value).
template <int P>
__global__ void __launch_bounds__(256) ximage_split_digits_kernel(const RowLayout L, const float* __restrict__ x,
                                                                  size_t x_stride, int nvec, uint4* __restrict__ img,
                                                                  size_t img_stride_quads, const int32_t* count) {
  asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
  // x may be the output of the kernel this one was launched behind.
  asm volatile("griddepcontrol.wait;" ::: "memory");
  if (count) nvec = min(max(*count, 0), nvec);  // vectors to build (device), at most nvec
  const int ntp = L.nseg * 32;
  const int nb_img = ntp * P;  // block slots covered by the image (incl. idle lanes)
  const int lane = threadIdx.x & 31;
  const int warps = (gridDim.x * blockDim.x) >> 5;
  for (int wi = (blockIdx.x * blockDim.x + threadIdx.x) >> 5; wi < nvec * nb_img; wi += warps) {
    const int v = wi / nb_img, b = wi % nb_img;  // slot b covers global block b
    const float xe = b < L.nblocks ? __ldg(x + v * x_stride + b * 32 + lane) : 0.0f;
    float m = fabsf(xe);
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) m = fmaxf(m, __shfl_xor_sync(0xFFFFFFFFu, m, o));
    int E = 0;
    frexpf(m, &E);  // m < 2^E (E = 0 for m = 0)
    const float y = ldexpf(xe, 20 - E);
    const int X0 = __float2int_rn(y);
    const int cnt = __popc(__ballot_sync(0xFFFFFFFFu, fabsf(y) >= kWideFloor));
    const int capped = __reduce_add_sync(0xFFFFFFFFu, min(abs(X0), kWideCap));
    const bool wide = isfinite(m) && block_is_wide(cnt, capped);
    const int X = wide ? 0 : X0;
    const int d0 = ((X + 64) & 127) - 64;
    const int X1 = (X - d0) / 128;
    const int d1 = ((X1 + 64) & 127) - 64;
    const int d2 = (X1 - d1) / 128;
    const int seg = b / (32 * P), j = (b % (32 * P)) / 32, lt = seg * 32 + b % 32;
    const int t = lane < 24 ? lane : 0;  // word t = g * 3 + k of this slot
    const int g = t / 3, k = t % 3;
    uint32_t word = 0;
#pragma unroll
    for (int e = 0; e < 4; ++e) {
      const int s0 = __shfl_sync(0xFFFFFFFFu, d0, 4 * g + e);
      const int s1 = __shfl_sync(0xFFFFFFFFu, d1, 4 * g + e);
      const int s2 = __shfl_sync(0xFFFFFFFFu, d2, 4 * g + e);
      const int dk = k == 0 ? s0 : (k == 1 ? s1 : s2);
      word |= (static_cast<uint32_t>(dk) & 0xFFu) << (8 * e);
    }
    uint32_t* out = reinterpret_cast<uint32_t*>(img + v * img_stride_quads);
    int widx = -1;
    uint32_t val = 0;
    if (lane < 24) {
      widx = (j * 8 + g) * 3 + k;
      val = word;
    } else if (lane == 24) {
      widx = RowDotSplitFp4DigitT<P>::scale_word(j);
      val = wide ? kWideMark : __float_as_uint(isfinite(m) ? ldexpf(1.0f, E - 21) : __int_as_float(0x7FC00000));
    }
    if (widx >= 0) out[(static_cast<size_t>(widx >> 2) * ntp + lt) * 4 + (widx & 3)] = val;
  }
}

// In-kernel x images.  Where the host allows it (inline_x_ok / direct_x_ok)
// the pipelined kernel forms its x registers itself, after its
// griddepcontrol.wait, instead of behind a separate ximage launch: one grid
// completion less on the path of every call.  Float tiles load their quads
// straight from x.  Digit tiles are built by the consumer threads together,
// four threads per 32-value block, to the same bits as ximage_digits_kernel,
// into the shared memory of the ring's last slot; the producer holds that
// slot's first copy until every consumer warp has its registers.

// max with NaN propagation (PTX max.NaN): a block holding a NaN is detected
// by the result alone.
__device__ __forceinline__ float max_nan(float a, float b) {
  float r;
  asm("max.NaN.f32 %0, %1, %2;" : "=f"(r) : "f"(a), "f"(b));
  return r;
}

// Quarter Q of block B of lane tile lt (groups 2Q, 2Q + 1 of the block: 8 of
// its elements; the four quarters of a block are consecutive lanes of one
// warp, `gmask` those four lanes).  For a block of finite values, x * 2^(20-E)
// is one or two exact power-of-two products and the rounding to an integer
// (|value| < 2^21) one magic-number addition, both equal to ldexpf and
// __float2int_rn; a block holding NaN or Inf takes those functions as is.
// Wide blocks are marked as ximage_digits_kernel marks them.
template <int FMT>
__device__ __forceinline__ void digit_quarter(const float* __restrict__ xb, bool live, int B, int Q, unsigned gmask,
                                              int lt, int ntp, uint32_t* img) {
  using T = Tile<FMT>;
  float v[8];
#pragma unroll
  for (int i = 0; i < 8; ++i) v[i] = live ? __ldg(xb + T::elem(B, 2 * Q + (i >> 2), i & 3)) : 0.0f;
  float m = fabsf(v[0]);
#pragma unroll
  for (int i = 1; i < 8; ++i) m = max_nan(m, fabsf(v[i]));
  m = max_nan(m, __shfl_xor_sync(gmask, m, 1));
  m = max_nan(m, __shfl_xor_sync(gmask, m, 2));
  int X[8];
  int E = 0;
  bool wide = false;
  if (m < INFINITY) {  // no NaN (max.NaN would carry it) and no Inf in the block
    frexpf(m, &E);     // m < 2^E (E = 0 for m = 0)
    const int k = 20 - E, k1 = min(k, 127);
    const float s1 = __int_as_float((k1 + 127) << 23), s2 = __int_as_float((k - k1 + 127) << 23);
    int acc = 0;  // capped sum (< 2^21) and count (<= 32, from bit 24), packed
#pragma unroll
    for (int i = 0; i < 8; ++i) {
      const float y = (v[i] * s1) * s2;  // exact: x * 2^(20-E)
      X[i] = __float_as_int(y + 12582912.0f) - 0x4B400000;
      acc += min(abs(X[i]), kWideCap) + (fabsf(y) >= kWideFloor ? (1 << 24) : 0);
    }
    // over the block's four quarters
    acc += __shfl_xor_sync(gmask, acc, 1);
    acc += __shfl_xor_sync(gmask, acc, 2);
    wide = block_is_wide(acc >> 24, acc & 0xFFFFFF);
    if (wide) {
#pragma unroll
      for (int i = 0; i < 8; ++i) X[i] = 0;
    }
  } else {
    m = fabsf(v[0]);
#pragma unroll
    for (int i = 1; i < 8; ++i) m = fmaxf(m, fabsf(v[i]));
    m = fmaxf(m, __shfl_xor_sync(gmask, m, 1));
    m = fmaxf(m, __shfl_xor_sync(gmask, m, 2));
    frexpf(m, &E);
#pragma unroll
    for (int i = 0; i < 8; ++i) X[i] = __float2int_rn(ldexpf(v[i], 20 - E));
  }
  uint32_t sx = 0;
#pragma unroll
  for (int i = 0; i < 8; ++i) sx += static_cast<uint32_t>(X[i]);
  sx += __shfl_xor_sync(gmask, sx, 1);
  sx += __shfl_xor_sync(gmask, sx, 2);
  auto put = [&](int widx, uint32_t val) { img[(static_cast<size_t>(widx >> 2) * ntp + lt) * 4 + (widx & 3)] = val; };
#pragma unroll
  for (int h = 0; h < 2; ++h) {
    uint32_t w0 = 0, w1 = 0, w2 = 0;
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      const int Xe = X[4 * h + j];
      const int d0 = ((Xe + 64) & 127) - 64;
      const int X1 = (Xe - d0) / 128;
      const int d1 = ((X1 + 64) & 127) - 64;
      const int d2 = (X1 - d1) / 128;
      w0 |= (static_cast<uint32_t>(d0) & 0xFFu) << (8 * j);
      w1 |= (static_cast<uint32_t>(d1) & 0xFFu) << (8 * j);
      w2 |= (static_cast<uint32_t>(d2) & 0xFFu) << (8 * j);
    }
    put(dg_word(B, 2 * Q + h, 0), w0);
    put(dg_word(B, 2 * Q + h, 1), w1);
    put(dg_word(B, 2 * Q + h, 2), w2);
  }
  if (Q == 0) {
    put(48 + B, wide ? kWideMark : __float_as_uint(isfinite(m) ? ldexpf(1.0f, E - 20) : __int_as_float(0x7FC00000)));
    put(50 + B, static_cast<uint32_t>(-T::kOffset) * sx);
  }
}

// Item i (< ntp * 8) of a digit image: quarter i % 4 of block i / 4.
template <int FMT>
__device__ __forceinline__ void build_digit_item(const float* __restrict__ x, int item, int nblocks, int ntp,
                                                 uint32_t* img) {
  static_assert(Tile<FMT>::P == 2, "digit tiles hold two blocks");
  const int gb = item >> 2, lt = gb >> 1;
  const bool live = gb < nblocks;
  const float* xb = x + static_cast<size_t>(live ? gb : 0) * 32;
  const unsigned gmask = 0xFu << (threadIdx.x & 28);
  digit_quarter<FMT>(xb, live, gb & 1, item & 3, gmask, lt, ntp, img);
}

// Float tiles: quad q of lane tile lt is x[c .. c + 3], c = RD::quad_col.
template <class RD, class XR>
__device__ __forceinline__ void load_x_direct(const RowLayout& L, const float* __restrict__ x, int lt, XR& xr) {
#pragma unroll
  for (int q = 0; q < XR::kQuads; ++q) {
    const int c = RD::quad_col(L, lt, q);
    xr.q[q] = c >= 0 ? __ldg(reinterpret_cast<const uint4*>(x + c)) : make_uint4(0u, 0u, 0u, 0u);
  }
}

template <class RD, class = void>
struct HasQuadCol : std::false_type {};
template <class RD>
struct HasQuadCol<RD, std::void_t<decltype(&RD::quad_col)>> : std::true_type {};

// Row formats whose x registers are plain float quads of x.
template <class RD>
struct IsFloatRD {
  static constexpr bool value = HasQuadCol<RD>::value && !IsDigitRD<RD>::value;
};

// Float-quad rows whose direct x loads are near-coalesced (neighbouring lanes
// read quads at most 32 bytes apart): worth reading a fresh vector per job.
template <class RD>
struct NearCoalescedQuads : std::false_type {};
template <int CPL>
struct NearCoalescedQuads<RowDotBf16T<CPL>> : std::true_type {};

// Float-quad rows for which one direct read of x per CTA beats an image
// launch (measured on B200): bf16 rows and interleaved FP4 tiles; split FP4
// rows read 128-byte-strided quads and keep the image launch.
template <class RD>
struct DirectQuadsOnce : std::false_type {};
template <int CPL>
struct DirectQuadsOnce<RowDotBf16T<CPL>> : std::true_type {};
template <>
struct DirectQuadsOnce<RowDot<OBJB_FP4_E2M1>> : std::true_type {};

template <class XR>
__device__ __forceinline__ void load_ximage_shared(const uint32_t* img, int ntp, int lt, XR& xr) {
#pragma unroll
  for (int q = 0; q < XR::kQuads; ++q) xr.q[q] = *reinterpret_cast<const uint4*>(img + (q * ntp + lt) * 4);
}

// Programs whose x registers the kernel forms itself name the vector in a
// member `x` (nullptr: the images come from a preceding ximage launch).
template <class P, class = void>
struct ProgInlineX {
  static constexpr bool value = false;
  __device__ __forceinline__ static const float* get(const P&) { return nullptr; }
};
template <class P>
struct ProgInlineX<P, std::void_t<decltype(std::declval<const P&>().x)>> {
  static constexpr bool value = true;
  __device__ __forceinline__ static const float* get(const P& p) { return p.x; }
};

// Reduces NV per-lane values over the 32 lanes of a warp with a transposed
// butterfly: log2(NV) exchange steps that halve the value set, then plain
// xor-shuffle steps.  Afterwards v[0] of lane L holds the full sum of value
// index (L / (32 / NV)).  NV - 1 + (5 - log2 NV) shuffles instead of 5 * NV.
template <int NV>
__device__ __forceinline__ void butterfly(float (&v)[NV], int lane) {
#pragma unroll
  for (int n = NV, off = 16; n > 1; n >>= 1, off >>= 1) {
    const bool upper = (lane & off) != 0;
#pragma unroll
    for (int i = 0; i < n / 2; ++i) {
      const float keep = upper ? v[i + n / 2] : v[i];
      const float send = upper ? v[i] : v[i + n / 2];
      v[i] = keep + __shfl_xor_sync(0xFFFFFFFFu, send, off);
    }
  }
#pragma unroll
  for (int off = 16 / NV; off > 0; off >>= 1) v[0] += __shfl_xor_sync(0xFFFFFFFFu, v[0], off);
}

// The producer side: issues the bulk copies of `nst` stages of up to two
// matrices (A and, when dual, B) into the ring.  Stage i covers rows
// [row0 + i*tstage, ...).  Weights of A land at slot offset 0, scales of A
// after tstage weight rows; B's weights and scales follow A's.
struct StageSource {
  const uint8_t* wa;
  const uint8_t* sa;
  const uint8_t* wb;
  const uint8_t* sb;
};

__device__ __forceinline__ int slot_part_bytes(const RowLayout& L) {
  return L.tstage * (L.row_bytes + L.srow_bytes);
}

// Issues stage `i` (row range [r0, r0 + nr)) into `slot`.
__device__ __forceinline__ void issue_stage(const RowLayout& L, const SmemPlan& sp, int slot,
                                            const StageSource& src, bool dual, int r0, int nr,
                                            uint64_t pol, unsigned* err) {
  uint8_t* dst = sp.stage + static_cast<size_t>(slot) * L.stage_bytes;
  // Bulk copies need 16-byte aligned sources: a misaligned expert pointer is
  // recorded and its stage completed without data instead of faulting.
  const uintptr_t mis = (reinterpret_cast<uintptr_t>(src.wa) | reinterpret_cast<uintptr_t>(src.sa) |
                         (dual ? (reinterpret_cast<uintptr_t>(src.wb) | reinterpret_cast<uintptr_t>(src.sb)) : 0)) & 15u;
  if (mis || src.wa == nullptr || (dual && src.wb == nullptr)) {
    if (err) atomicOr(err, kErrMisaligned);
    *reinterpret_cast<volatile unsigned*>(sp.abort) = 1u;  // the rows of this launch come out NaN
    mbar_arrive(&sp.full[slot]);
    return;
  }
  const uint32_t wbytes = static_cast<uint32_t>(nr) * L.row_bytes;
  const uint32_t sbytes = static_cast<uint32_t>(nr) * L.srow_bytes;
  const uint32_t per = wbytes + sbytes;
  mbar_arrive_expect_tx(&sp.full[slot], dual ? 2 * per : per);
  bulk_g2s(dst, src.wa + static_cast<size_t>(r0) * L.row_bytes, wbytes, &sp.full[slot], pol);
  if (sbytes)
    bulk_g2s(dst + static_cast<size_t>(L.tstage) * L.row_bytes,
             src.sa + static_cast<size_t>(r0) * L.srow_bytes, sbytes, &sp.full[slot], pol);
  if (dual) {
    uint8_t* dstb = dst + slot_part_bytes(L);
    bulk_g2s(dstb, src.wb + static_cast<size_t>(r0) * L.row_bytes, wbytes, &sp.full[slot], pol);
    if (sbytes)
      bulk_g2s(dstb + static_cast<size_t>(L.tstage) * L.row_bytes,
               src.sb + static_cast<size_t>(r0) * L.srow_bytes, sbytes, &sp.full[slot], pol);
  }
}


// One job = a row range of one matrix (or a matching pair) against one x.
struct Job {
  StageSource src;
  const uint4* ximg;  // x image of this job's vector
  int row_begin, row_end;
  const float* x = nullptr;  // float-quad rows: this job's vector, read directly (ximg unused)
  const float* xd = nullptr;  // digit rows: this job's vector as floats, for the terms of wide blocks
};

// The fp32 terms of the wide blocks of a digit image (flagged kWideMark),
// added after a stage's integer row dots: w0 / w1 are the lanes of this warp
// whose tile block 0 / 1 is wide.  For each of the warp's rows of the stage
// every lane forms its element's term of every wide block, the warp sums
// them, and lane 0 adds the sum to the row's partial of this column segment
// (the slot the row dot wrote in `red`).  Runs only when the vector has a
// wide block, outside the integer loop, so that loop keeps its registers.
template <int FMT, bool DUAL>
__device__ __noinline__ void add_wide_terms(float* red, const uint8_t* stg, int part, int row_bytes, int nseg,
                                            int seg, int grp, int ngrp, int nr, uint32_t w0, uint32_t w1,
                                            const float* __restrict__ xd) {
  using T = Tile<FMT>;
  const int lane = threadIdx.x & 31;
  for (int t = grp * 4; t < nr; t += ngrp * 4) {
    const int tend = min(nr, t + 4);
    for (int r = t; r < tend; ++r) {
      float sa = 0.0f, sb = 0.0f;
#pragma unroll 1
      for (int b = 0; b < 2; ++b) {
        uint32_t m = b ? w1 : w0;
#pragma unroll 1
        while (m) {
          const int src = __ffs(m) - 1;
          m &= m - 1;
          const int lt = seg * 32 + src;
          const int boff = lt * T::TB + b * T::BB;
          const float xl = __ldg(xd + static_cast<size_t>(lt * T::P + b) * 32 + lane);
          sa += wide_term<FMT>(stg + r * row_bytes + boff, lane, xl);
          if constexpr (DUAL) sb += wide_term<FMT>(stg + part + r * row_bytes + boff, lane, xl);
        }
      }
#pragma unroll
      for (int o = 16; o > 0; o >>= 1) {
        sa += __shfl_xor_sync(0xFFFFFFFFu, sa, o);
        if constexpr (DUAL) sb += __shfl_xor_sync(0xFFFFFFFFu, sb, o);
      }
      if (lane == 0) {
        red[(r * nseg + seg) * 2] += sa;
        if constexpr (DUAL) red[(r * nseg + seg) * 2 + 1] += sb;
      }
    }
  }
}

// The wide-block pass of split FP4 rows (RowDotSplitFp4DigitT<P>): as
// add_wide_terms, with the slot-j block of lane `src` at global block
// seg * 32 P + src + 32 j, its 16 code bytes in the row and its E8M0 scale in
// the stage's scale rows (`srows`, `srow_bytes` apart; the second matrix's
// weights and scale rows `part` and `sb_part` bytes further).  A term is
// (value * scale) * x_l, the reference's w * x (decode_deepseek_fp4_to_f32,
// deepseek.rs:862-918, then a dense dot).
template <int P, bool DUAL>
__device__ __noinline__ void add_wide_terms_split(float* red, const uint8_t* stg, const uint8_t* srows, int part,
                                                  int sb_part, int row_bytes, int srow_bytes, int nseg, int seg,
                                                  int grp, int ngrp, int nr, uint32_t w0, uint32_t w1,
                                                  const float* __restrict__ xd) {
  const int lane = threadIdx.x & 31;
  for (int t = grp * 4; t < nr; t += ngrp * 4) {
    const int tend = min(nr, t + 4);
    for (int r = t; r < tend; ++r) {
      float sa = 0.0f, sb = 0.0f;
#pragma unroll 1
      for (int j = 0; j < P; ++j) {
        uint32_t m = j ? w1 : w0;
#pragma unroll 1
        while (m) {
          const int src = __ffs(m) - 1;
          m &= m - 1;
          const int b = seg * 32 * P + src + 32 * j;
          const float xl = __ldg(xd + static_cast<size_t>(b) * 32 + lane);
          const uint32_t byte = stg[r * row_bytes + 16 * b + (lane >> 1)];
          const uint32_t c = (lane & 1) ? (byte >> 4) : (byte & 0xFu);
          const int v2 = static_cast<int8_t>(fp4x4_to_i8x4(c) & 0xFFu);  // 2 * value
          const float scale = e8m0_to_f32(srows[r * srow_bytes + b]);
          sa += __fmul_rn(static_cast<float>(v2) * (0.5f * scale), xl);
          if constexpr (DUAL) {
            const uint32_t byte2 = stg[part + r * row_bytes + 16 * b + (lane >> 1)];
            const uint32_t c2 = (lane & 1) ? (byte2 >> 4) : (byte2 & 0xFu);
            const int u2 = static_cast<int8_t>(fp4x4_to_i8x4(c2) & 0xFFu);
            const float scale2 = e8m0_to_f32(srows[sb_part + r * srow_bytes + b]);
            sb += __fmul_rn(static_cast<float>(u2) * (0.5f * scale2), xl);
          }
        }
      }
#pragma unroll
      for (int o = 16; o > 0; o >>= 1) {
        sa += __shfl_xor_sync(0xFFFFFFFFu, sa, o);
        if constexpr (DUAL) sb += __shfl_xor_sync(0xFFFFFFFFu, sb, o);
      }
      if (lane == 0) {
        red[(r * nseg + seg) * 2] += sa;
        if constexpr (DUAL) red[(r * nseg + seg) * 2 + 1] += sb;
      }
    }
  }
}

// Row formats whose digit images may mark wide blocks, and their fp32 pass.
template <class RD>
struct WideTerms {
  static constexpr bool value = false;
};
template <int FMT>
struct WideTerms<RowDot<FMT>> {
  static constexpr bool value = IsDigitRD<RowDot<FMT>>::value;
  static constexpr int kSlots = 2;
  template <class XR>
  __device__ __forceinline__ static uint32_t mark_word(const XR& xr, int j) { return xr.w(48 + j); }
  template <bool DUAL>
  __device__ __forceinline__ static void add(float* red, const uint8_t* stg, const uint8_t*, int part, int,
                                             const RowLayout& L, int seg, int grp, int nr, uint32_t w0, uint32_t w1,
                                             const float* xd) {
    add_wide_terms<FMT, DUAL>(red, stg, part, L.row_bytes, L.nseg, seg, grp, L.ngrp, nr, w0, w1, xd);
  }
};
template <int P>
struct WideTerms<RowDotSplitFp4DigitT<P>> {
  static constexpr bool value = true;
  static constexpr int kSlots = P;
  template <class XR>
  __device__ __forceinline__ static uint32_t mark_word(const XR& xr, int j) {
    return xr.w(RowDotSplitFp4DigitT<P>::scale_word(j));
  }
  template <bool DUAL>
  __device__ __forceinline__ static void add(float* red, const uint8_t* stg, const uint8_t* srows, int part,
                                             int sb_part, const RowLayout& L, int seg, int grp, int nr, uint32_t w0,
                                             uint32_t w1, const float* xd) {
    add_wide_terms_split<P, DUAL>(red, stg, srows, part, sb_part, L.row_bytes, L.srow_bytes, L.nseg, seg, grp, L.ngrp,
                                  nr, w0, w1, xd);
  }
};

// One stage's wide-block pass of a warp (row formats with WideTerms).
template <class RD, bool DUAL, class XR>
__device__ __forceinline__ void wide_stage(const XR& xr, float* red, const uint8_t* stg, const uint8_t* sca, int part,
                                           const RowLayout& L, int seg, int grp, int nr, const float* xd,
                                           unsigned* err) {
  if constexpr (WideTerms<RD>::value) {
    using WT = WideTerms<RD>;
    // the lanes whose slot-0 / slot-1 block is wide
    const uint32_t w0 = __ballot_sync(0xFFFFFFFFu, WT::mark_word(xr, 0) == kWideMark);
    uint32_t w1 = 0u;
    if constexpr (WT::kSlots > 1) w1 = __ballot_sync(0xFFFFFFFFu, WT::mark_word(xr, 1) == kWideMark);
    __syncwarp();
    if (xd != nullptr)
      WT::template add<DUAL>(red, stg, sca, part, part, L, seg, grp, nr, w0, w1, xd);
    else if ((threadIdx.x & 31) == 0 && err)
      atomicOr(err, kErrNoWideSource);
  }
}

// Whether this warp's x registers mark a wide block.
template <class RD, class XR>
__device__ __forceinline__ bool warp_has_wide(const XR& xr) {
  if constexpr (WideTerms<RD>::value) {
    using WT = WideTerms<RD>;
    bool mine = WT::mark_word(xr, 0) == kWideMark;
    if constexpr (WT::kSlots > 1) mine = mine || WT::mark_word(xr, 1) == kWideMark;
    return __any_sync(0xFFFFFFFFu, mine);
  } else {
    return false;
  }
}

// Consumer warps: nseg * ngrp (<= kMaxConsumerWarps); one producer warp more.
constexpr int kPipeThreads = (kMaxConsumerWarps + 1) * 32;

// The pipelined kernel.  `Prog` supplies, for this CTA, a list of jobs and an
// epilogue that receives each finished row (va for matrix A, vb for B):
//   int njobs(int cta) const;   Job job(int cta, int j) const;
//   void epilogue(int cta, int j, int row, float va, float vb) const;
//   void finalize(int cta, int tid, int nthreads) const;   // after all jobs
//   unsigned* err;
// DUAL streams a second matrix of the same shape through the same stages.
template <class RD, class Prog, bool DUAL>
__global__ void __launch_bounds__(kPipeThreads, 1) pipe_kernel(const RowLayout L, const Prog prog) {
  // Let the next launch of the stream (when it was launched with programmatic
  // serialization: an x-image prep, which waits for this grid before reading
  // anything) be scheduled now, so its launch and this grid's tail overlap.
  asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
  extern __shared__ __align__(128) uint8_t smem_raw[];
  const SmemPlan sp = carve_smem(smem_raw, L, 2);
  const int ncw = L.nseg * L.ngrp;
  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const int cta = blockIdx.x;
  const int S = L.nslots;
  const int T = L.tstage;
  unsigned* err = prog.err;

  if (threadIdx.x == 0) {
    for (int i = 0; i < S; ++i) {
      mbar_init(&sp.full[i], 1);
      mbar_init(&sp.empty[i], ncw);
    }
    mbar_init(sp.img_done, ncw);
    *sp.abort = 0u;
    fence_mbar_init();
  }
  __syncthreads();

  const int njobs = prog.njobs(cta);
  // (row formats whose x registers are x quads or a digit image only)
  constexpr bool kInlineX = ProgInlineX<Prog>::value && (IsDigitRD<RD>::value || HasQuadCol<RD>::value);
  const float* xin = kInlineX ? ProgInlineX<Prog>::get(prog) : nullptr;
  // in-kernel digit image: built in the last slot before that slot's first copy
  const bool img_in_ring = xin != nullptr && IsDigitRD<RD>::value;

  if (warp == ncw) {
    // ---------------- producer: one elected thread issues every stage.
    if (lane == 0) {
      const uint64_t pol = l2_policy_evict_first();
      uint32_t it = 0;
      bool ok = true;
      for (int j = 0; j < njobs && ok; ++j) {
        const Job J = prog.job(cta, j);
        for (int r0 = J.row_begin; r0 < J.row_end; r0 += T) {
          const int slot = static_cast<int>(it % S);
          if (it >= static_cast<uint32_t>(S)) {
            if (!mbar_wait_bounded(&sp.empty[slot], ((it / S) - 1) & 1u, err, kErrEmptyWaitTimeout, sp.abort)) {
              ok = false;
              break;
            }
          } else if (img_in_ring && it == static_cast<uint32_t>(S - 1)) {
            if (!mbar_wait_bounded(sp.img_done, 0u, err, kErrEmptyWaitTimeout, sp.abort)) {
              ok = false;
              break;
            }
          }
          const int nr = min(T, J.row_end - r0);
          issue_stage(L, sp, slot, J.src, DUAL, r0, nr, pol, err);
          ++it;
        }
      }
      // Never leave while this CTA's own copies may still be landing.
      const uint32_t first = it > static_cast<uint32_t>(S) ? it - S : 0u;
      for (uint32_t k = first; k < it; ++k)
        mbar_wait_bounded(&sp.full[k % S], (k / S) & 1u, nullptr, 0u);
    }
    return;
  }

  // ---------------- consumers
  // Warp (seg, grp) computes, for batches of RB rows, the partial dot of its
  // column segment; rows of a stage are dealt to row groups RB at a time.
  constexpr int RB = 4;
  constexpr int NV = DUAL ? 2 * RB : RB;
  constexpr int W = 32 / NV;
  const int seg = warp % L.nseg;
  const int grp = warp / L.nseg;
  const int nthr = ncw * 32;
  bool ok = true;
  uint32_t it = 0;
  RD rd;
  rd.init(L, seg, lane);
  typename RD::XRegs xr;
  const int part = slot_part_bytes(L);
  // x (or its image, written by the preceding ximage launch) may come from
  // the kernel this one was launched behind (programmatic launch).
  asm volatile("griddepcontrol.wait;" ::: "memory");
  if constexpr (kInlineX) {
    if (xin != nullptr) {
      const int ntp = L.nseg * 32;
      if constexpr (IsDigitRD<RD>::value) {
        uint32_t* img = reinterpret_cast<uint32_t*>(sp.stage + static_cast<size_t>(S - 1) * L.stage_bytes);
        for (int item = threadIdx.x; item < ntp * 8; item += nthr)
          build_digit_item<IsDigitRD<RD>::fmt>(xin, item, L.nblocks, ntp, img);
        named_bar_sync(1, nthr);
        load_ximage_shared(img, ntp, seg * 32 + lane, xr);
        // the slot's bulk copies (async proxy) come after these accesses
        asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
        __syncwarp();
        if (lane == 0) mbar_arrive(sp.img_done);
      } else if constexpr (HasQuadCol<RD>::value) {
        load_x_direct<RD>(L, xin, seg * 32 + lane, xr);
      }
    }
  }

  for (int j = 0; j < njobs; ++j) {
    const Job J = prog.job(cta, j);
    if constexpr (IsFloatRD<RD>::value) {
      if (J.x != nullptr) load_x_direct<RD>(L, J.x, seg * 32 + lane, xr);
      else if (xin == nullptr) load_ximage(J.ximg, L.nseg * 32, seg * 32 + lane, xr);
    } else if (xin == nullptr) {
      load_ximage(J.ximg, L.nseg * 32, seg * 32 + lane, xr);
    }
    // The job's stages, in two instantiations: with the fp32 pass for wide
    // blocks (digit rows whose vector has one in this warp's tiles) and
    // without, so ordinary vectors run the integer loop untouched.  Warps of
    // one CTA may take different ones: both pass the same barriers in the
    // same order.
    auto stages = [&](auto wide_tag) {
      constexpr bool kWide = decltype(wide_tag)::value;
      for (int r0 = J.row_begin; r0 < J.row_end; r0 += T) {
        const int slot = static_cast<int>(it % S);
        if (ok) ok = mbar_wait_bounded(&sp.full[slot], (it / S) & 1u, err, kErrFullWaitTimeout, sp.abort);
        const int nr = min(T, J.row_end - r0);
        const uint8_t* stg = sp.stage + static_cast<size_t>(slot) * L.stage_bytes;
        const uint8_t* sca = stg + static_cast<size_t>(T) * L.row_bytes;
        float* red = sp.red + static_cast<size_t>(slot) * T * L.nseg * 2;
        for (int bt = grp * RB; bt < nr; bt += L.ngrp * RB) {
          float v[NV];
#pragma unroll
          for (int i = 0; i < RB; ++i) {
            const int t = min(bt + i, nr - 1);
            v[i] = rd.dot(stg + t * L.row_bytes, sca + t * L.srow_bytes, xr);
            if constexpr (DUAL)
              v[RB + i] = rd.dot(stg + part + t * L.row_bytes,
                                 stg + part + static_cast<size_t>(T) * L.row_bytes + t * L.srow_bytes, xr);
          }
          butterfly<NV>(v, lane);
          if ((lane & (W - 1)) == 0) {
            const int idx = lane / W;
            const int t = bt + (idx % RB);
            if (t < nr) red[(t * L.nseg + seg) * 2 + idx / RB] = v[0];
          }
        }
        if constexpr (kWide) wide_stage<RD, DUAL>(xr, red, stg, sca, part, L, seg, grp, nr, J.xd, err);
        __syncwarp();
        if (lane == 0) mbar_arrive(&sp.empty[slot]);
        named_bar_sync(1, nthr);
        // a stage that never landed (or landed without data) yields NaN rows,
        // not values reduced from stale shared memory
        const bool aborted = *reinterpret_cast<volatile unsigned*>(sp.abort) != 0u;
        for (int t = threadIdx.x; t < nr; t += nthr) {
          float va = 0.0f, vb = 0.0f;
          for (int s2 = 0; s2 < L.nseg; ++s2) {
            va += red[(t * L.nseg + s2) * 2];
            if constexpr (DUAL) vb += red[(t * L.nseg + s2) * 2 + 1];
          }
          if (aborted) va = vb = __int_as_float(0x7FC00000);
          prog.epilogue(cta, j, r0 + t, va, vb);
        }
        ++it;
      }
    };
    if constexpr (WideTerms<RD>::value) {
      if (warp_has_wide<RD>(xr)) stages(std::true_type{});
      else stages(std::false_type{});
    } else {
      stages(std::false_type{});
    }
  }
  named_bar_sync(1, nthr);
  prog.finalize(cta, threadIdx.x, nthr);
}

// Plain GEMV: each CTA owns `rows_per_cta` consecutive rows.  x != nullptr:
// the kernel forms its x registers from x itself (ximg unused).
struct GemvProg {
  StageSource src;
  const uint4* ximg;
  const float* x = nullptr;
  const float* xd = nullptr;  // the vector, for the terms of wide digit blocks
  float* y;
  int rows;
  int rows_per_cta;
  unsigned* err;
  __device__ __forceinline__ int njobs(int) const { return 1; }
  __device__ __forceinline__ Job job(int cta, int) const {
    Job J;
    J.src = src;
    J.ximg = ximg;
    J.xd = xd;
    J.row_begin = cta * rows_per_cta;
    J.row_end = min(rows, J.row_begin + rows_per_cta);
    return J;
  }
  __device__ __forceinline__ void epilogue(int, int, int row, float va, float) const { y[row] = va; }
  __device__ __forceinline__ void finalize(int, int, int) const {}
};

// Fallback for shapes / pointers the bulk-copy path cannot take: one warp
// per row, blocks read straight from global memory with byte loads.
template <int FMT>
__global__ void __launch_bounds__(256) gemv_fallback_kernel(const uint8_t* __restrict__ w,
                                                            const float* __restrict__ x,
                                                            float* __restrict__ y, int rows,
                                                            int cols, size_t row_bytes) {
  const int row = blockIdx.x * 8 + (threadIdx.x >> 5);
  const int lane = threadIdx.x & 31;
  if (row >= rows) return;
  constexpr int BB = FMT == OBJB_Q4_0 ? 18 : FMT == OBJB_Q5_0 ? 22 : FMT == OBJB_IQ3_0 ? 14 : 17;
  const int nb = cols / 32;
  const uint8_t* rw = w + static_cast<size_t>(row) * row_bytes;
  float acc = 0.0f;
  for (int b = lane; b < nb; b += 32) acc += block_dot_global<FMT>(rw + static_cast<size_t>(b) * BB, x + b * 32);
  for (int o = 16; o > 0; o >>= 1) acc += __shfl_xor_sync(0xFFFFFFFFu, acc, o);
  if (lane == 0) y[row] = acc;
}

}  // namespace dev
}  // namespace objb
