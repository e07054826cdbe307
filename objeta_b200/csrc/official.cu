// official.cu -- the official DeepSeek activation path as device entry points:
// act_quant (cuda_act_quant / cuda_act_quant_device, quant.rs:1119-1282), the
// FP8 activation x FP4 weight GEMV (cuda_fp8_act_fp4_weight_gemv_device,
// quant.rs:1284-1326) and the FP8 x FP8 GEMV of the shared expert
// (cuda_fp8_act_fp8_weight_gemv_device, quant.rs:1328-1363).
#include <cuda_runtime.h>

#include <algorithm>
#include <cstring>
#include <string>

#include "objb_common.h"
#include "objb_host_launch.cuh"
#include "objb_moe.cuh"
#include "objb_official.cuh"
#include "objb_official_launch.h"

namespace objb {
namespace dev {

// act_quant (deepseek.rs:1484-1525) for `nblocks` blocks of 128 values: one
// warp per block, 4 values per lane.  Values and scales bit-identical to the
// CPU reference.
__global__ void __launch_bounds__(256) act_quant_kernel(const float* __restrict__ x, size_t nblocks,
                                                        uint8_t* __restrict__ y, uint8_t* __restrict__ s) {
  asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
  asm volatile("griddepcontrol.wait;" ::: "memory");
  const int lane = threadIdx.x & 31;
  const size_t warps = (static_cast<size_t>(gridDim.x) * blockDim.x) >> 5;
  for (size_t wb = (static_cast<size_t>(blockIdx.x) * blockDim.x + threadIdx.x) >> 5; wb < nblocks; wb += warps) {
    const float* xb = x + wb * 128 + lane * 4;
    float v[4];
    float amax = 0.0f;
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      v[i] = xb[i];
      const float a = fabsf(v[i]);
      if (a > amax) amax = a;
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) amax = fmaxf(amax, __shfl_xor_sync(0xFFFFFFFFu, amax, o));
    amax = fmaxf(amax, 1e-4f);
    const float raw = amax * (1.0f / 448.0f);
    const int lc = raw > 0.0f ? ceil_log2_ref(raw) : -127;
    const float scale = ldexpf(1.0f, lc);
    if (lane == 0) {
      const long long e = static_cast<long long>(lc) + 127;
      s[wb] = static_cast<uint8_t>(e < 0 ? 0 : (e > 255 ? 255 : e));
    }
    uint32_t packed = 0;
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      float q = __fdiv_rn(v[i], scale);
      if (q < -448.0f) q = -448.0f;  // Rust clamp: NaN stays NaN
      if (q > 448.0f) q = 448.0f;
      packed |= f32_to_e4m3_ref(q) << (8 * i);
    }
    *reinterpret_cast<uint32_t*>(y + wb * 128 + lane * 4) = packed;
  }
}

// Image builder for RowDotFp8Fp4 from act_quant output: codes [nvec][cols],
// scales [nvec][cols / 128].  One warp per (vector, 32-value block).
__global__ void __launch_bounds__(256) ximage_fp8_kernel(const RowLayout L, const uint8_t* __restrict__ codes,
                                                         const uint8_t* __restrict__ scales, int nvec,
                                                         uint4* __restrict__ img, size_t img_stride_quads) {
  asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
  asm volatile("griddepcontrol.wait;" ::: "memory");  // codes may come from the previous kernel
  const int ntp = L.nseg * 32;
  const int nb_img = L.nseg * 64;  // block slots covered by the image (incl. idle lanes)
  const int cols = L.cols;
  const int lane = threadIdx.x & 31;
  const int warps = (gridDim.x * blockDim.x) >> 5;
  for (int wi = (blockIdx.x * blockDim.x + threadIdx.x) >> 5; wi < nvec * nb_img; wi += warps) {
    const int v = wi / nb_img, b = wi % nb_img;
    const bool live = b < L.nblocks;
    const int A = live ? e4m3_ref_times512(codes[static_cast<size_t>(v) * cols + b * 32 + lane]) : 0;
    const int d0 = ((A + 64) & 127) - 64;
    const int A1 = (A - d0) / 128;
    const int d1 = ((A1 + 64) & 127) - 64;
    const int d2 = (A1 - d1) / 128;
    const int seg = b / 64, j = (b % 64) / 32, owner = b % 32;
    const int lt = seg * 32 + owner;
    const int t = lane < 24 ? lane : 0;  // word t = g * 3 + k of this block
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
    uint32_t* out = reinterpret_cast<uint32_t*>(img + static_cast<size_t>(v) * img_stride_quads);
    int widx = -1;
    uint32_t val = 0;
    if (lane < 24) {
      widx = (j * 8 + g) * 3 + k;
      val = word;
    } else if (lane == 24) {
      widx = 48 + j;
      val = live ? __float_as_uint(e8m0_to_f32(scales[static_cast<size_t>(v) * (cols / 128) + (b * 32) / 128]) *
                                   (1.0f / 1024.0f))
                 : 0u;
    } else if (lane == 25) {
      widx = 50 + j;
    }
    if (widx >= 0) out[(static_cast<size_t>(widx >> 2) * ntp + lt) * 4 + (widx & 3)] = val;
  }
}

// ---- FP8 activation x FP8 weight (shared expert): weight E4M3 [rows, K],
// E8M0 scales on a 128 x 128 tile grid [ceil(rows/128)][ceil(K/128)].  One
// warp per row, 16-byte loads; per 128-column tile the exact products
// (act * 2^9) * (w * 2^9) are summed in f32 and scaled by
// act_scale * w_scale * 2^-18.
__global__ void __launch_bounds__(256) fp8_fp8_gemv_kernel(const uint8_t* __restrict__ act,
                                                           const uint8_t* __restrict__ act_s,
                                                           const uint8_t* __restrict__ w,
                                                           const uint8_t* __restrict__ ws, float* __restrict__ y,
                                                           int rows, int K) {
  asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
  asm volatile("griddepcontrol.wait;" ::: "memory");
  const int row = blockIdx.x * 8 + (threadIdx.x >> 5);
  const int lane = threadIdx.x & 31;
  if (row >= rows) return;
  const int tiles = (K + 127) / 128;
  const uint8_t* wr = w + static_cast<size_t>(row) * K;
  const uint8_t* wsr = ws + static_cast<size_t>(row / 128) * tiles;
  float acc = 0.0f;
  // a tile is 128 columns = 8 chunks of 16; lane l takes chunk l % 8 of tile l / 8 (+4 tiles per step)
  for (int t0 = 0; t0 < tiles; t0 += 4) {
    const int t = t0 + lane / 8;
    float part = 0.0f;
    if (t < tiles) {
      const int c = t * 128 + (lane % 8) * 16;
      if (c + 16 <= K) {
        const uint4 wq = *reinterpret_cast<const uint4*>(wr + c);
        const uint4 aq = *reinterpret_cast<const uint4*>(act + c);
        const uint32_t wv[4] = {wq.x, wq.y, wq.z, wq.w}, av[4] = {aq.x, aq.y, aq.z, aq.w};
#pragma unroll
        for (int i = 0; i < 16; ++i) {
          const uint32_t wc = (wv[i >> 2] >> (8 * (i & 3))) & 0xFFu, ac = (av[i >> 2] >> (8 * (i & 3))) & 0xFFu;
          part = fmaf(static_cast<float>(e4m3_ref_times512(wc)), static_cast<float>(e4m3_ref_times512(ac)), part);
        }
      } else {
        for (int i = 0; i < 16 && c + i < K; ++i)
          part = fmaf(static_cast<float>(e4m3_ref_times512(wr[c + i])),
                      static_cast<float>(e4m3_ref_times512(act[c + i])), part);
      }
      part *= e8m0_to_f32(wsr[t]) * e8m0_to_f32(act_s[(t * 128) / 128]) * (1.0f / 262144.0f);
    }
    acc += part;
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) acc += __shfl_xor_sync(0xFFFFFFFFu, acc, o);
  if (lane == 0) y[row] = acc;
}

// Generic FP8 x FP4 row dot (any alignment): one warp per row.
__global__ void __launch_bounds__(256) fp8_fp4_gemv_generic_kernel(const uint8_t* __restrict__ act,
                                                                   const uint8_t* __restrict__ act_s,
                                                                   const uint8_t* __restrict__ w,
                                                                   const uint8_t* __restrict__ ws,
                                                                   float* __restrict__ y, int rows, int K) {
  asm volatile("griddepcontrol.wait;" ::: "memory");
  const int row = blockIdx.x * 8 + (threadIdx.x >> 5);
  const int lane = threadIdx.x & 31;
  if (row >= rows) return;
  const int nb = K / 32;
  const uint8_t* wr = w + static_cast<size_t>(row) * (K / 2);
  float acc = 0.0f;
  for (int b = lane; b < nb; b += 32) {
    int S = 0;
    for (int i = 0; i < 16; ++i) {
      const uint32_t byte = wr[b * 16 + i];
      const int v = static_cast<int>(fp4x4_to_i8x4(byte));  // bytes 0, 1: the two codes
      const int lo = static_cast<int8_t>(v & 0xFF), hi = static_cast<int8_t>((v >> 8) & 0xFF);
      S += lo * e4m3_ref_times512(act[b * 32 + 2 * i]) + hi * e4m3_ref_times512(act[b * 32 + 2 * i + 1]);
    }
    acc = fmaf(__int2float_rn(S),
               e8m0_to_f32(ws[static_cast<size_t>(row) * nb + b]) * e8m0_to_f32(act_s[b / 4]) * (1.0f / 1024.0f),
               acc);
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) acc += __shfl_xor_sync(0xFFFFFFFFu, acc, o);
  if (lane == 0) y[row] = acc;
}

// SwiGLU of the official shared expert (up clamped only, deepseek.rs:1675-1680)
// and out += v.
__global__ void __launch_bounds__(256) official_swiglu_kernel(const float* __restrict__ g, const float* __restrict__ u,
                                                              float* __restrict__ act, int n, float limit) {
  asm volatile("griddepcontrol.wait;" ::: "memory");
  const int i = blockIdx.x * blockDim.x + threadIdx.x;
  if (i < n) act[i] = swiglu(g[i], u[i], limit, false);
}
__global__ void __launch_bounds__(256) official_accum_kernel(const float* __restrict__ v, float* __restrict__ out,
                                                             int n) {
  asm volatile("griddepcontrol.wait;" ::: "memory");
  const int i = blockIdx.x * blockDim.x + threadIdx.x;
  if (i < n) out[i] = __fadd_rn(out[i], __fmul_rn(1.0f, v[i]));
}

}  // namespace dev

int act_quant(const float* x, size_t rows, size_t cols, uint8_t* values, uint8_t* scales, cudaStream_t stream,
              const char* action) {
  if (cols % 128)
    return OBJB_FAIL(OBJB_ERR_INVALID_INPUT, action, "cols " + std::to_string(cols) + " not divisible by 128");
  if (!x || !values || !scales) return OBJB_FAIL(OBJB_ERR_INVALID_INPUT, action, "null device pointer");
  if (reinterpret_cast<uintptr_t>(values) & 3u)
    return OBJB_FAIL(OBJB_ERR_INVALID_INPUT, action, "values must be 4-byte aligned");
  const size_t nblocks = rows * cols / 128;
  if (nblocks == 0) return OBJB_OK;
  const int grid = static_cast<int>(std::min<size_t>((nblocks + 7) / 8, 4096));
  return launch_pdl(dev::act_quant_kernel, grid, 256, 0, stream, x, nblocks, values, scales);
}

size_t fp8_image_quads(const RowLayoutHost& L) { return static_cast<size_t>(13) * L.nseg * 32; }

int launch_ximage_fp8(const RowLayoutHost& L, const uint8_t* codes, const uint8_t* scales, int nvec, uint4* img,
                      size_t img_stride_quads, cudaStream_t stream) {
  dev::RowLayout dl;
  std::memcpy(&dl, &L, sizeof(dl));
  const int warps = L.nseg * 64 * nvec;
  const int grid = std::max(1, std::min((warps + 7) / 8, 4096));
  return launch_pdl(dev::ximage_fp8_kernel, grid, 256, 0, stream, dl, codes, scales, nvec, img, img_stride_quads);
}

bool plan_fp8_fp4(int rows, int cols, bool dual, RowLayoutHost* L) {
  return plan_rows(rows, cols, cols / 2, cols / 32, 2, dual, dev::kMaxConsumerWarps, L, kMoeSmemBudget);
}

namespace {

int gemv_fp8_fp4(const uint8_t* act, const uint8_t* act_s, const uint8_t* w, const uint8_t* ws, float* y, int rows,
                 int cols, cudaStream_t stream) {
  int device = 0;
  OBJB_TRY(current_device(&device));
  DeviceProps props;
  OBJB_TRY(device_props(device, &props));
  RowLayoutHost L;
  const bool fast = aligned16(w) && aligned16(ws) && plan_fp8_fp4(rows, cols, false, &L);
  if (!fast) {
    dev::fp8_fp4_gemv_generic_kernel<<<(rows + 7) / 8, 256, 0, stream>>>(act, act_s, w, ws, y, rows, cols);
    OBJB_CUDA(cudaGetLastError(), "launch generic FP8 x FP4 GEMV");
    return OBJB_OK;
  }
  unsigned* err = nullptr;
  OBJB_TRY(device_error_word(device, &err));
  void* wsp = nullptr;
  OBJB_TRY(workspace_get(device, stream, fp8_image_quads(L) * 16, &wsp));
  uint4* img = static_cast<uint4*>(wsp);
  OBJB_TRY(launch_ximage_fp8(L, act, act_s, 1, img, 0, stream));
  int per = (rows + props.sm_count - 1) / props.sm_count;
  per = (per + 3) / 4 * 4;
  dev::GemvProg prog;
  prog.src = dev::StageSource{w, ws, nullptr, nullptr};
  prog.ximg = img;
  prog.x = nullptr;
  prog.y = y;
  prog.rows = rows;
  prog.rows_per_cta = per;
  prog.err = err;
  const size_t smem = pipe_smem_bytes(L);
  auto kernel = dev::pipe_kernel<dev::RowDotFp8Fp4, dev::GemvProg, false>;
  OBJB_TRY(ensure_smem_attr(kernel, device, smem));
  dev::RowLayout dl;
  std::memcpy(&dl, &L, sizeof(dl));
  return launch_pdl(kernel, (rows + per - 1) / per, (L.nseg * L.ngrp + 1) * 32, smem, stream, dl, prog);
}

}  // namespace

int gemv_fp8_fp8(const uint8_t* act, const uint8_t* act_s, const uint8_t* w, const uint8_t* ws, float* y, int rows,
                 int cols, cudaStream_t stream) {
  if (cols % 128)
    return OBJB_FAIL(OBJB_ERR_INVALID_INPUT, "cuda_fp8_act_fp8_weight_gemv_device",
                     "cols " + std::to_string(cols) + " not divisible by 128");
  if (!aligned16(w) || !aligned16(act))
    return OBJB_FAIL(OBJB_ERR_INVALID_INPUT, "cuda_fp8_act_fp8_weight_gemv_device",
                     "weight and activation buffers must be 16-byte aligned");
  return launch_pdl(dev::fp8_fp8_gemv_kernel, (rows + 7) / 8, 256, 0, stream, act, act_s, w, ws, y, rows, cols);
}

size_t shared_expert_fp8_scratch(int H, int I, int O) {
  auto r256 = [](size_t b) { return (b + 255) / 256 * 256; };
  return r256(H) + r256(H / 128) + 3 * r256(static_cast<size_t>(I) * 4) + r256(I) + r256(I / 128) +
         r256(static_cast<size_t>(O) * 4);
}

int shared_expert_fp8(const objb_fp8_shared_expert* sh, const float* x, int H, int I, int O, float limit, float* out,
                      cudaStream_t stream, void* scratch, size_t scratch_bytes) {
  if (!sh || !sh->gate_weight || !sh->gate_scale || !sh->up_weight || !sh->up_scale || !sh->down_weight ||
      !sh->down_scale)
    return OBJB_FAIL(OBJB_ERR_INVALID_INPUT, "run FP8 shared expert", "null shared expert pointer");
  if (scratch_bytes < shared_expert_fp8_scratch(H, I, O))
    return OBJB_FAIL(OBJB_ERR_INTERNAL, "run FP8 shared expert", "scratch too small");
  auto r256 = [](size_t b) { return (b + 255) / 256 * 256; };
  uint8_t* p = static_cast<uint8_t*>(scratch);
  uint8_t* cx = p;
  p += r256(H);
  uint8_t* sx = p;
  p += r256(H / 128);
  float* g = reinterpret_cast<float*>(p);
  p += r256(static_cast<size_t>(I) * 4);
  float* u = reinterpret_cast<float*>(p);
  p += r256(static_cast<size_t>(I) * 4);
  float* act = reinterpret_cast<float*>(p);
  p += r256(static_cast<size_t>(I) * 4);
  uint8_t* ca = p;
  p += r256(I);
  uint8_t* sa = p;
  p += r256(I / 128);
  float* v = reinterpret_cast<float*>(p);
  auto u8 = [](const void* q) { return static_cast<const uint8_t*>(q); };
  OBJB_TRY(act_quant(x, 1, H, cx, sx, stream, "act_quant hidden (shared expert)"));
  OBJB_TRY(gemv_fp8_fp8(cx, sx, u8(sh->gate_weight), u8(sh->gate_scale), g, I, H, stream));
  OBJB_TRY(gemv_fp8_fp8(cx, sx, u8(sh->up_weight), u8(sh->up_scale), u, I, H, stream));
  OBJB_TRY(launch_pdl(dev::official_swiglu_kernel, (I + 255) / 256, 256, 0, stream, g, u, act, I, limit));
  OBJB_TRY(act_quant(act, 1, I, ca, sa, stream, "act_quant intermediate (shared expert)"));
  OBJB_TRY(gemv_fp8_fp8(ca, sa, u8(sh->down_weight), u8(sh->down_scale), v, O, I, stream));
  return launch_pdl(dev::official_accum_kernel, (O + 255) / 256, 256, 0, stream, v, out, O);
}

}  // namespace objb

extern "C" {

int objb_act_quant_device(const float* d_x, size_t rows, size_t cols, uint8_t* d_values, uint8_t* d_scales,
                          objb_stream_t stream) {
  objb::clear_error();
  if (rows > (1u << 24) || cols > (1u << 24))
    return OBJB_FAIL(OBJB_ERR_INVALID_INPUT, "cuda_act_quant_device", "shape out of range");
  return objb::act_quant(d_x, rows, cols, d_values, d_scales, static_cast<cudaStream_t>(stream),
                         "cuda_act_quant_device");
}

int objb_gemv_fp8_fp4_device(const uint8_t* d_act, const uint8_t* d_act_scales, const void* d_weight,
                             const void* d_weight_scales, float* d_y, size_t rows, size_t cols,
                             objb_stream_t stream) {
  objb::clear_error();
  if (!d_act || !d_act_scales || !d_weight || !d_weight_scales || !d_y)
    return OBJB_FAIL(OBJB_ERR_INVALID_INPUT, "cuda_fp8_act_fp4_weight_gemv_device", "null device pointer");
  if (cols % 128 || rows == 0 || rows > (1u << 24) || cols > (1u << 20))
    return OBJB_FAIL(OBJB_ERR_INVALID_INPUT, "cuda_fp8_act_fp4_weight_gemv_device",
                     "cols " + std::to_string(cols) + " not divisible by 128");
  return objb::gemv_fp8_fp4(d_act, d_act_scales, static_cast<const uint8_t*>(d_weight),
                            static_cast<const uint8_t*>(d_weight_scales), d_y, static_cast<int>(rows),
                            static_cast<int>(cols), static_cast<cudaStream_t>(stream));
}

int objb_gemv_fp8_fp8_device(const uint8_t* d_act, const uint8_t* d_act_scales, const void* d_weight,
                             const void* d_weight_scales, float* d_y, size_t rows, size_t cols,
                             objb_stream_t stream) {
  objb::clear_error();
  if (!d_act || !d_act_scales || !d_weight || !d_weight_scales || !d_y)
    return OBJB_FAIL(OBJB_ERR_INVALID_INPUT, "cuda_fp8_act_fp8_weight_gemv_device", "null device pointer");
  if (rows == 0 || rows > (1u << 24) || cols > (1u << 20))
    return OBJB_FAIL(OBJB_ERR_INVALID_INPUT, "cuda_fp8_act_fp8_weight_gemv_device", "shape out of range");
  return objb::gemv_fp8_fp8(d_act, d_act_scales, static_cast<const uint8_t*>(d_weight),
                            static_cast<const uint8_t*>(d_weight_scales), d_y, static_cast<int>(rows),
                            static_cast<int>(cols), static_cast<cudaStream_t>(stream));
}

}  // extern "C"
