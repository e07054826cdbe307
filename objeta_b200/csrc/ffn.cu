// ffn.cu -- dense bf16 GEMV and the dense SwiGLU FFN built on it (the shared
// expert of a DeepSeek-style MoE layer: routed experts in FP4, one shared
// expert in bf16).  The reference has no bf16 kernel; the arithmetic is its
// bf16 -> f32 widening (crates/objeta-parser/src/lib.rs:334-337) followed by
// the f32 dot product and SwiGLU of the MoE path (kernels/moe.cu:2-22).
#include <cuda_runtime.h>

#include <algorithm>
#include <cstring>
#include <string>

#include "objb_common.h"
#include "objb_host_launch.cuh"
#include "objb_moe.cuh"

namespace objb {
namespace dev {

// Generic path (unaligned pointers or shapes): one warp per row, 4-byte loads.
__global__ void __launch_bounds__(256) gemv_bf16_fallback_kernel(const uint16_t* __restrict__ w,
                                                                 const float* __restrict__ x,
                                                                 float* __restrict__ y, int rows, int cols) {
  const int row = blockIdx.x * 8 + (threadIdx.x >> 5);
  const int lane = threadIdx.x & 31;
  if (row >= rows) return;
  const uint16_t* wr = w + static_cast<size_t>(row) * cols;
  float acc = 0.0f;
  for (int c = lane; c < cols; c += 32) acc = fmaf(__uint_as_float(static_cast<uint32_t>(wr[c]) << 16), x[c], acc);
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) acc += __shfl_xor_sync(0xFFFFFFFFu, acc, o);
  if (lane == 0) y[row] = acc;
}

__global__ void __launch_bounds__(256) ffn_generic_act_kernel(const float* __restrict__ g, const float* __restrict__ u,
                                                              float* __restrict__ act, int n, float limit) {
  const int i = blockIdx.x * blockDim.x + threadIdx.x;
  if (i < n) act[i] = swiglu(g[i], u[i], limit);
}

__global__ void __launch_bounds__(256) ffn_generic_out_kernel(const float* __restrict__ v, float* __restrict__ out,
                                                              int n, int accumulate) {
  const int i = blockIdx.x * blockDim.x + threadIdx.x;
  if (i < n) out[i] = accumulate ? __fadd_rn(out[i], v[i]) : v[i];
}

}  // namespace dev

namespace {

bool plan_bf16(int rows, int cols, bool dual, RowLayoutHost* L) {
  return plan_rows(rows, cols, cols * 2, 0, 2, dual, dev::kMaxConsumerWarps, L, kMoeSmemBudget);
}

int even_split(int rows, int sms, int* grid) {
  int per = (rows + sms - 1) / sms;
  per = (per + 3) / 4 * 4;
  *grid = (rows + per - 1) / per;
  return per;
}

int validate_dense(size_t rows, size_t cols, const char* action) {
  if (rows == 0 || cols == 0 || rows > (1u << 24) || cols > (1u << 20) || cols % 32)
    return OBJB_FAIL(OBJB_ERR_INVALID_INPUT, action,
                     "rows " + std::to_string(rows) + " / cols " + std::to_string(cols) +
                         " out of range (cols must be a multiple of 32)");
  return OBJB_OK;
}

int gemv_bf16(const void* w, const float* x, float* y, int rows, int cols, cudaStream_t stream) {
  int device = 0;
  OBJB_TRY(current_device(&device));
  DeviceProps props;
  OBJB_TRY(device_props(device, &props));
  RowLayoutHost L;
  const bool fast = aligned16(w) && plan_bf16(rows, cols, false, &L);
  if (!fast) {
    dev::gemv_bf16_fallback_kernel<<<(rows + 7) / 8, 256, 0, stream>>>(static_cast<const uint16_t*>(w), x, y, rows,
                                                                      cols);
    OBJB_CUDA(cudaGetLastError(), "launch bf16 GEMV fallback");
    return OBJB_OK;
  }
  unsigned* err = nullptr;
  OBJB_TRY(device_error_word(device, &err));
  const bool x_inline = inline_x_ok<dev::RowDotBf16>(L, x);
  uint4* img = nullptr;
  if (!x_inline) {
    void* ws = nullptr;
    OBJB_TRY(workspace_get(device, stream, ximage_quads<dev::RowDotBf16>(L) * 16, &ws));
    img = static_cast<uint4*>(ws);
    OBJB_TRY(launch_ximage<dev::RowDotBf16>(L, x, 0, 1, img, 0, stream));
  }
  int grid = 0;
  dev::GemvProg prog;
  prog.src = dev::StageSource{static_cast<const uint8_t*>(w), nullptr, nullptr, nullptr};
  prog.ximg = img;
  prog.x = x_inline ? x : nullptr;
  prog.y = y;
  prog.rows = rows;
  prog.rows_per_cta = even_split(rows, props.sm_count, &grid);
  prog.err = err;
  const size_t smem = pipe_smem_bytes(L);
  auto kernel = dev::pipe_kernel<dev::RowDotBf16, dev::GemvProg, false>;
  OBJB_TRY(ensure_smem_attr(kernel, device, smem));
  dev::RowLayout dl;
  std::memcpy(&dl, &L, sizeof(dl));
  return launch_pdl(kernel, grid, (L.nseg * L.ngrp + 1) * 32, smem, stream, dl, prog);
}

size_t ffn_scratch(const RowLayoutHost& lg, const RowLayoutHost& ld, int I, bool fast) {
  const size_t act = (static_cast<size_t>(I) * 4 + 255) / 256 * 256;
  if (!fast) return 3 * act;  // gate, up, act
  return act + (ximage_quads<dev::RowDotBf16>(lg) + ximage_quads<dev::RowDotBf16>(ld)) * 16 + 256;
}

int ffn_bf16(const void* gate, const void* up, const void* down, int H, int I, int O, const float* x, float* out,
             int accumulate, float limit, cudaStream_t stream) {
  int device = 0;
  OBJB_TRY(current_device(&device));
  DeviceProps props;
  OBJB_TRY(device_props(device, &props));
  unsigned* err = nullptr;
  OBJB_TRY(device_error_word(device, &err));
  RowLayoutHost lg, ld;
  const bool fast = aligned16(gate) && aligned16(up) && aligned16(down) && plan_bf16(I, H, true, &lg) &&
                    plan_bf16(O, I, false, &ld);
  const size_t need = ffn_scratch(lg, ld, I, fast);
  void* ws = nullptr;
  OBJB_TRY(workspace_get(device, stream, need, &ws));
  uint8_t* sc = static_cast<uint8_t*>(ws);
  const size_t act_bytes = (static_cast<size_t>(I) * 4 + 255) / 256 * 256;
  float* act = reinterpret_cast<float*>(sc);
  if (!fast) {
    float* g = reinterpret_cast<float*>(sc + act_bytes);
    float* u = reinterpret_cast<float*>(sc + 2 * act_bytes);
    OBJB_TRY(gemv_bf16(gate, x, g, I, H, stream));
    OBJB_TRY(gemv_bf16(up, x, u, I, H, stream));
    dev::ffn_generic_act_kernel<<<(I + 255) / 256, 256, 0, stream>>>(g, u, act, I, limit);
    OBJB_CUDA(cudaGetLastError(), "launch FFN activation");
    // down into g (I >= O is not guaranteed: use the act region only when it fits)
    float* v = O <= I ? g : nullptr;
    if (!v) return OBJB_FAIL(OBJB_ERR_UNSUPPORTED, "run bf16 FFN", "unaligned FFN with out_dim > intermediate");
    OBJB_TRY(gemv_bf16(down, act, v, O, I, stream));
    dev::ffn_generic_out_kernel<<<(O + 255) / 256, 256, 0, stream>>>(v, out, O, accumulate);
    OBJB_CUDA(cudaGetLastError(), "launch FFN output");
    return OBJB_OK;
  }
  uint4* imgx = reinterpret_cast<uint4*>(sc + act_bytes);
  uint4* imga = imgx + ximage_quads<dev::RowDotBf16>(lg);
  // the kernels read x and the activation row directly (float quads) when aligned
  const bool x_inline = inline_x_ok<dev::RowDotBf16>(lg, x);
  const bool act_inline = inline_x_ok<dev::RowDotBf16>(ld, act);
  if (!x_inline) OBJB_TRY(launch_ximage<dev::RowDotBf16>(lg, x, 0, 1, imgx, 0, stream));
  {
    int grid = 0;
    dev::FfnGateUpProg prog;
    prog.src = dev::StageSource{static_cast<const uint8_t*>(gate), nullptr, static_cast<const uint8_t*>(up), nullptr};
    prog.ximg = imgx;
    prog.x = x_inline ? x : nullptr;
    prog.act = act;
    prog.I = I;
    prog.rows_per_cta = even_split(I, props.sm_count, &grid);
    prog.swiglu_limit = limit;
    prog.err = err;
    const size_t smem = pipe_smem_bytes(lg);
    auto kernel = dev::pipe_kernel<dev::RowDotBf16, dev::FfnGateUpProg, true>;
    OBJB_TRY(ensure_smem_attr(kernel, device, smem));
    dev::RowLayout dl;
    std::memcpy(&dl, &lg, sizeof(dl));
    OBJB_TRY(launch_pdl(kernel, grid, (lg.nseg * lg.ngrp + 1) * 32, smem, stream, dl, prog));
  }
  if (!act_inline) OBJB_TRY(launch_ximage<dev::RowDotBf16>(ld, act, 0, 1, imga, 0, stream));
  {
    int grid = 0;
    dev::FfnDownProg prog;
    prog.src = dev::StageSource{static_cast<const uint8_t*>(down), nullptr, nullptr, nullptr};
    prog.ximg = imga;
    prog.x = act_inline ? act : nullptr;
    prog.out = out;
    prog.O = O;
    prog.rows_per_cta = even_split(O, props.sm_count, &grid);
    prog.accumulate = accumulate;
    prog.err = err;
    const size_t smem = pipe_smem_bytes(ld);
    auto kernel = dev::pipe_kernel<dev::RowDotBf16, dev::FfnDownProg, false>;
    OBJB_TRY(ensure_smem_attr(kernel, device, smem));
    dev::RowLayout dl;
    std::memcpy(&dl, &ld, sizeof(dl));
    OBJB_TRY(launch_pdl(kernel, grid, (ld.nseg * ld.ngrp + 1) * 32, smem, stream, dl, prog));
  }
  return OBJB_OK;
}

}  // namespace
}  // namespace objb

extern "C" {

int objb_gemv_bf16_device(const void* d_w, const float* d_x, float* d_y, size_t rows, size_t cols,
                          objb_stream_t stream) {
  objb::clear_error();
  OBJB_TRY(objb::validate_dense(rows, cols, "objb_gemv_bf16_device"));
  if (!d_w || !d_x || !d_y) return OBJB_FAIL(OBJB_ERR_INVALID_INPUT, "objb_gemv_bf16_device", "null device pointer");
  return objb::gemv_bf16(d_w, d_x, d_y, static_cast<int>(rows), static_cast<int>(cols),
                         static_cast<cudaStream_t>(stream));
}

int objb_ffn_bf16_device(const void* d_gate, const void* d_up, const void* d_down, size_t hidden,
                         size_t intermediate, size_t out_dim, const float* d_x, float* d_out, int accumulate,
                         float swiglu_limit, objb_stream_t stream) {
  objb::clear_error();
  OBJB_TRY(objb::validate_dense(intermediate, hidden, "objb_ffn_bf16_device"));
  OBJB_TRY(objb::validate_dense(out_dim, intermediate, "objb_ffn_bf16_device"));
  if (!d_gate || !d_up || !d_down || !d_x || !d_out)
    return OBJB_FAIL(OBJB_ERR_INVALID_INPUT, "objb_ffn_bf16_device", "null device pointer");
  return objb::ffn_bf16(d_gate, d_up, d_down, static_cast<int>(hidden), static_cast<int>(intermediate),
                        static_cast<int>(out_dim), d_x, d_out, accumulate, swiglu_limit,
                        static_cast<cudaStream_t>(stream));
}

}  // extern "C"
