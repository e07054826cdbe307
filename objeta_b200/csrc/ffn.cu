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

// Row plan of a bf16 matrix with CPL chunks per lane: cols / (256 CPL) warps
// per row.
bool plan_bf16_cpl(int cpl, int rows, int cols, bool dual, RowLayoutHost* L) {
  const int lanes = (cols / 8 + cpl - 1) / cpl;
  return plan_rows_lanes(rows, cols, cols * 2, 0, lanes, dual, dev::kMaxConsumerWarps, L, kMoeSmemBudget);
}

// Chunks per lane for a matrix: the most (fewest warps per row) whose stage
// still gives every row group one 4-row batch; else the fewest (all warps on
// the rows of a small stage).
int pick_cpl(int rows, int cols, bool dual) {
  const int stage_max = std::min(kMoeSmemBudget, 227 * 1024) / 2 - 4096;
  const size_t per_row = static_cast<size_t>(cols) * 2 * (dual ? 2 : 1);
  for (int cpl : {8, 4}) {
    const int nseg = (cols / 8 + 32 * cpl - 1) / (32 * cpl);
    if (nseg > dev::kMaxConsumerWarps) continue;
    const int quantum = std::max(1, dev::kMaxConsumerWarps / nseg) * 4;
    if (static_cast<size_t>(quantum) * per_row <= static_cast<size_t>(stage_max)) return cpl;
  }
  (void)rows;
  return 2;
}

template <int CPL, class F>
int with_cpl(int cpl, F&& f) {
  switch (cpl) {
    case 8: return f(std::integral_constant<int, 8>{});
    case 4: return f(std::integral_constant<int, 4>{});
    default: return f(std::integral_constant<int, 2>{});
  }
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

template <class RD>
int gemv_bf16_pipe(const RowLayoutHost& L, const void* w, const float* x, float* y, int rows, int device,
                   const DeviceProps& props, cudaStream_t stream) {
  unsigned* err = nullptr;
  OBJB_TRY(device_error_word(device, &err));
  const bool x_inline = inline_x_ok<RD>(L, x);
  uint4* img = nullptr;
  if (!x_inline) {
    void* ws = nullptr;
    OBJB_TRY(workspace_get(device, stream, ximage_quads<RD>(L) * 16, &ws));
    img = static_cast<uint4*>(ws);
    OBJB_TRY(launch_ximage<RD>(L, x, 0, 1, img, 0, stream));
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
  auto kernel = dev::pipe_kernel<RD, dev::GemvProg, false>;
  OBJB_TRY(ensure_smem_attr(kernel, device, smem));
  dev::RowLayout dl;
  std::memcpy(&dl, &L, sizeof(dl));
  return launch_pdl(kernel, grid, (L.nseg * L.ngrp + 1) * 32, smem, stream, dl, prog);
}

int gemv_bf16(const void* w, const float* x, float* y, int rows, int cols, cudaStream_t stream) {
  int device = 0;
  OBJB_TRY(current_device(&device));
  DeviceProps props;
  OBJB_TRY(device_props(device, &props));
  RowLayoutHost L;
  const int cpl = pick_cpl(rows, cols, false);
  const bool fast = aligned16(w) && plan_bf16_cpl(cpl, rows, cols, false, &L);
  if (!fast) {
    dev::gemv_bf16_fallback_kernel<<<(rows + 7) / 8, 256, 0, stream>>>(static_cast<const uint16_t*>(w), x, y, rows,
                                                                      cols);
    OBJB_CUDA(cudaGetLastError(), "launch bf16 GEMV fallback");
    return OBJB_OK;
  }
  return with_cpl<0>(cpl, [&](auto c) {
    return gemv_bf16_pipe<dev::RowDotBf16T<decltype(c)::value>>(L, w, x, y, rows, device, props, stream);
  });
}

template <class RDg, class RDd>
int ffn_bf16_pipe(const RowLayoutHost& lg, const RowLayoutHost& ld, const void* gate, const void* up,
                  const void* down, int I, int O, const float* x, float* out, int accumulate, float limit,
                  cudaStream_t stream, int device, const DeviceProps& props, uint8_t* sc, unsigned* err) {
  const size_t act_bytes = (static_cast<size_t>(I) * 4 + 255) / 256 * 256;
  float* act = reinterpret_cast<float*>(sc);
  uint4* imgx = reinterpret_cast<uint4*>(sc + act_bytes);
  uint4* imga = imgx + ximage_quads<RDg>(lg);
  // the kernels read x and the activation row directly (float quads) when aligned
  const bool x_inline = inline_x_ok<RDg>(lg, x);
  const bool act_inline = inline_x_ok<RDd>(ld, act);
  if (!x_inline) OBJB_TRY(launch_ximage<RDg>(lg, x, 0, 1, imgx, 0, stream));
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
    auto kernel = dev::pipe_kernel<RDg, dev::FfnGateUpProg, true>;
    OBJB_TRY(ensure_smem_attr(kernel, device, smem));
    dev::RowLayout dl;
    std::memcpy(&dl, &lg, sizeof(dl));
    OBJB_TRY(launch_pdl(kernel, grid, (lg.nseg * lg.ngrp + 1) * 32, smem, stream, dl, prog));
  }
  if (!act_inline) OBJB_TRY(launch_ximage<RDd>(ld, act, 0, 1, imga, 0, stream));
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
    auto kernel = dev::pipe_kernel<RDd, dev::FfnDownProg, false>;
    OBJB_TRY(ensure_smem_attr(kernel, device, smem));
    dev::RowLayout dl;
    std::memcpy(&dl, &ld, sizeof(dl));
    OBJB_TRY(launch_pdl(kernel, grid, (ld.nseg * ld.ngrp + 1) * 32, smem, stream, dl, prog));
  }
  return OBJB_OK;
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
  const int cg = pick_cpl(I, H, true), cd = pick_cpl(O, I, false);
  const bool fast = aligned16(gate) && aligned16(up) && aligned16(down) && plan_bf16_cpl(cg, I, H, true, &lg) &&
                    plan_bf16_cpl(cd, O, I, false, &ld);
  const size_t act_bytes = (static_cast<size_t>(I) * 4 + 255) / 256 * 256;
  // scratch: act, then the two x images (at most 16 quads per lane tile)
  const size_t need = fast ? act_bytes + (static_cast<size_t>(16) * lg.nseg * 32 + 16 * ld.nseg * 32) * 16 + 256
                           : 3 * act_bytes;
  void* ws = nullptr;
  OBJB_TRY(workspace_get(device, stream, need, &ws));
  uint8_t* sc = static_cast<uint8_t*>(ws);
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
  return with_cpl<0>(cg, [&](auto a) {
    return with_cpl<0>(cd, [&](auto b) {
      return ffn_bf16_pipe<dev::RowDotBf16T<decltype(a)::value>, dev::RowDotBf16T<decltype(b)::value>>(
          lg, ld, gate, up, down, I, O, x, out, accumulate, limit, stream, device, props, sc, err);
    });
  });
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
