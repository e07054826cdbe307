// gemv.cu -- batch-1 block-dequant GEMV for sm_100a: launch planning, the
// device-pointer entry points and the host-slice QuantBackend of the C ABI.
#include <cuda_runtime.h>

#include <algorithm>
#include <atomic>
#include <cstring>
#include <map>
#include <mutex>
#include <string>
#include <type_traits>

#include "objb_common.h"
#include "objb_gemv.cuh"
#include "objb_launch.h"
#include "objb_host_launch.cuh"

namespace objb {
namespace dev {

// Split-layout FP4 fallback (any alignment).
__global__ void __launch_bounds__(256) gemv_fp4_split_fallback_kernel(
    const uint8_t* __restrict__ w, const uint8_t* __restrict__ s, const float* __restrict__ x,
    float* __restrict__ y, int rows, int cols) {
  const int row = blockIdx.x * 8 + (threadIdx.x >> 5);
  const int lane = threadIdx.x & 31;
  if (row >= rows) return;
  const int nb = cols / 32;
  const uint8_t* rw = w + static_cast<size_t>(row) * (cols / 2);
  const uint8_t* rs = s + static_cast<size_t>(row) * nb;
  float acc = 0.0f;
  for (int b = lane; b < nb; b += 32) {
    float a = 0.0f;
    for (int j = 0; j < 16; ++j) {
      const float2 v = e2m1x2_to_float2(rw[b * 16 + j]);
      a = fmaf(v.x, __ldg(x + b * 32 + 2 * j), a);
      a = fmaf(v.y, __ldg(x + b * 32 + 2 * j + 1), a);
    }
    acc += a * e8m0_to_f32(rs[b]);
  }
  for (int o = 16; o > 0; o >>= 1) acc += __shfl_xor_sync(0xFFFFFFFFu, acc, o);
  if (lane == 0) y[row] = acc;
}

}  // namespace dev

static_assert(sizeof(RowLayoutHost) == sizeof(dev::RowLayout), "layout mirror mismatch");

bool plan_rows(int rows, int cols, int row_bytes, int srow_bytes, int blocks_per_lane, bool dual,
               int max_consumer_warps, RowLayoutHost* L, int smem_budget) {
  if (rows <= 0 || cols <= 0 || cols % 32 || blocks_per_lane <= 0) return false;
  const int lanes = (cols / 32 + blocks_per_lane - 1) / blocks_per_lane;
  return plan_rows_lanes(rows, cols, row_bytes, srow_bytes, lanes, dual, max_consumer_warps, L, smem_budget);
}

bool plan_rows_lanes(int rows, int cols, int row_bytes, int srow_bytes, int lanes, bool dual, int max_consumer_warps,
                     RowLayoutHost* L, int smem_budget) {
  if (rows <= 0 || cols <= 0 || cols % 32 || lanes <= 0) return false;
  const int nblocks = cols / 32;
  if (row_bytes % 16 || srow_bytes % 16) return false;
  const int nseg = (lanes + 31) / 32;
  if (nseg > max_consumer_warps) return false;
  const int lpr = 32;  // one row per warp; idle lanes when the row is narrow
  const int rpw = 1;
  const int ngrp = std::max(1, max_consumer_warps / nseg);
  int per_row = row_bytes + srow_bytes;
  if (dual) per_row *= 2;
  constexpr int kStageTarget = 48 * 1024;
  const int kSmemBudget = std::min(smem_budget, 227 * 1024);
  const int kStageMax = kSmemBudget / 2 - 4096;
  // One stage gives every row group one 4-row batch when that fits; small rows
  // get several batches per stage.
  const int quantum = ngrp * 4;
  int T;
  if (quantum * per_row <= kStageTarget) {
    T = quantum;
    while (T + quantum <= dev::kMaxRowsPerStage && (T + quantum) * per_row <= kStageTarget) T += quantum;
  } else {
    T = std::max(1, std::min(quantum, kStageMax / per_row));
    if (T > 4) T = T / 4 * 4;
  }
  T = std::min(T, dev::kMaxRowsPerStage);
  const int stage_bytes = ((T * per_row) + 127) / 128 * 128;
  const int red_bytes = dev::kMaxSlots * T * nseg * 2 * 4;
  const int fixed = dev::kPipeBarrierWords * 8 + red_bytes + 128;
  int slots = std::min(dev::kMaxSlots, (kSmemBudget - fixed) / stage_bytes);
  if (slots < 2) return false;
  L->rows = rows;
  L->cols = cols;
  L->nblocks = nblocks;
  L->row_bytes = row_bytes;
  L->srow_bytes = srow_bytes;
  L->nseg = nseg;
  L->lpr = lpr;
  L->rpw = rpw;
  L->ngrp = ngrp;
  L->tstage = T;
  L->nslots = slots;
  L->stage_bytes = stage_bytes;
  return true;
}

size_t pipe_smem_bytes(const RowLayoutHost& L) {
  size_t off = dev::kPipeBarrierWords * sizeof(uint64_t) +
               static_cast<size_t>(L.nslots) * L.tstage * L.nseg * 2 * sizeof(float);
  off = (off + 127) & ~static_cast<size_t>(127);
  return off + static_cast<size_t>(L.nslots) * L.stage_bytes;
}

// Opts a kernel into large dynamic shared memory, once per (kernel, device).
int ensure_smem_attr_ptr(const void* kernel, int device, size_t bytes) {
  static std::mutex mu;
  static std::map<std::pair<const void*, int>, size_t> done;
  std::lock_guard<std::mutex> lk(mu);
  auto key = std::make_pair(kernel, device);
  auto it = done.find(key);
  if (it != done.end() && it->second >= bytes) return OBJB_OK;
  const size_t want = std::max<size_t>(bytes, 200 * 1024);
  OBJB_CUDA(cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                 static_cast<int>(want)),
            "opt kernel into large shared memory");
  done[key] = want;
  return OBJB_OK;
}

namespace {

template <class RD>
int launch_gemv_pipe(const RowLayoutHost& L, const uint8_t* w, const uint8_t* s, const float* x,
                     float* y, cudaStream_t stream, int device, const DeviceProps& props) {
  unsigned* err = nullptr;
  OBJB_TRY(device_error_word(device, &err));
  // The kernel forms its x registers itself where that pays; otherwise an
  // ximage launch goes first.
  const bool inline_x = inline_x_ok<RD>(L, x);
  uint4* img = nullptr;
  if (!inline_x) {
    void* ws = nullptr;
    OBJB_TRY(workspace_get(device, stream, ximage_quads<RD>(L) * 16, &ws));
    img = static_cast<uint4*>(ws);
    OBJB_TRY(launch_ximage<RD>(L, x, 0, 1, img, 0, stream));
  }
  // Rows split evenly over the SMs in whole 4-row batches (a CTA's last
  // stage may be short), so every SM streams the same number of bytes.
  int per_cta = (L.rows + props.sm_count - 1) / props.sm_count;
  per_cta = (per_cta + 3) / 4 * 4;
  const int grid = (L.rows + per_cta - 1) / per_cta;
  dev::GemvProg prog;
  prog.src = dev::StageSource{w, s, nullptr, nullptr};
  prog.ximg = img;
  prog.x = inline_x ? x : nullptr;
  prog.xd = x;
  prog.y = y;
  prog.rows = L.rows;
  prog.rows_per_cta = per_cta;
  prog.err = err;
  const size_t smem = pipe_smem_bytes(L);
  auto kernel = dev::pipe_kernel<RD, dev::GemvProg, false>;
  OBJB_TRY(ensure_smem_attr(kernel, device, smem));
  dev::RowLayout dl;
  std::memcpy(&dl, &L, sizeof(dl));
  const int threads = (L.nseg * L.ngrp + 1) * 32;
  return launch_pdl(kernel, grid, threads, smem, stream, dl, prog);
}

template <int FMT>
int gemv_device_fmt(const uint8_t* w, const float* x, float* y, int rows, int cols,
                    cudaStream_t stream) {
  int device = 0;
  OBJB_TRY(current_device(&device));
  DeviceProps props;
  OBJB_TRY(device_props(device, &props));
  using T = dev::Tile<FMT>;
  const int row_bytes = cols / 32 * T::BB;
  RowLayoutHost L;
  const bool fast = aligned16(w) && (cols / 32) % T::P == 0 &&
                    plan_rows(rows, cols, row_bytes, 0, T::P, false, dev::kMaxConsumerWarps, &L);
  if (fast) return launch_gemv_pipe<dev::RowDot<FMT>>(L, w, nullptr, x, y, stream, device, props);
  const int grid = (rows + 7) / 8;
  dev::gemv_fallback_kernel<FMT><<<grid, 256, 0, stream>>>(w, x, y, rows, cols,
                                                           static_cast<size_t>(row_bytes));
  OBJB_CUDA(cudaGetLastError(), "launch fallback GEMV kernel");
  return OBJB_OK;
}

}  // namespace

int gemv_device(int fmt, const void* w, const float* x, float* y, size_t rows, size_t cols,
                cudaStream_t stream) {
  OBJB_TRY(validate_gemv_shape(fmt, rows, cols));
  if (rows == 0) return OBJB_OK;
  if (!w || !x || !y) return OBJB_FAIL(OBJB_ERR_INVALID_INPUT, "objb_gemv_device", "null device pointer");
  if (rows > (1u << 30) || cols > (1u << 24))
    return OBJB_FAIL(OBJB_ERR_INVALID_INPUT, "objb_gemv_device", "shape exceeds the supported range");
  const uint8_t* wb = static_cast<const uint8_t*>(w);
  const int r = static_cast<int>(rows), c = static_cast<int>(cols);
  switch (fmt) {
    case OBJB_Q4_0: return gemv_device_fmt<OBJB_Q4_0>(wb, x, y, r, c, stream);
    case OBJB_Q5_0: return gemv_device_fmt<OBJB_Q5_0>(wb, x, y, r, c, stream);
    case OBJB_IQ3_0: return gemv_device_fmt<OBJB_IQ3_0>(wb, x, y, r, c, stream);
    default: return gemv_device_fmt<OBJB_FP4_E2M1>(wb, x, y, r, c, stream);
  }
}

int gemv_fp4_split_device(const void* w, const void* s, const float* x, float* y, size_t rows,
                          size_t cols, cudaStream_t stream) {
  if (cols % 32 != 0)
    return OBJB_FAIL(OBJB_ERR_INVALID_INPUT, "validate deepseek_fp4_e2m1 split column alignment",
                     "cols " + std::to_string(cols) + " must be a multiple of block_size 32");
  if (rows == 0) return OBJB_OK;
  if (!w || !s || !x || !y) return OBJB_FAIL(OBJB_ERR_INVALID_INPUT, "objb_gemv_fp4_split_device", "null device pointer");
  int device = 0;
  OBJB_TRY(current_device(&device));
  DeviceProps props;
  OBJB_TRY(device_props(device, &props));
  const int r = static_cast<int>(rows), c = static_cast<int>(cols);
  const uint8_t* wb = static_cast<const uint8_t*>(w);
  const uint8_t* sb = static_cast<const uint8_t*>(s);
  RowLayoutHost L;
  const bool fast = aligned16(wb) && aligned16(sb) &&
                    plan_rows(r, c, c / 2, c / 32, dev::RowDotSplitFp4Digit::P, false, dev::kMaxConsumerWarps, &L);
  if (fast) return launch_gemv_pipe<dev::RowDotSplitFp4Digit>(L, wb, sb, x, y, stream, device, props);
  dev::gemv_fp4_split_fallback_kernel<<<(r + 7) / 8, 256, 0, stream>>>(wb, sb, x, y, r, c);
  OBJB_CUDA(cudaGetLastError(), "launch split FP4 fallback kernel");
  return OBJB_OK;
}

}  // namespace objb

// ------------------------------------------------------------------ C ABI

struct objb_quant_backend {
  int device;
  std::mutex mu;
  // Reusable device buffers for the host-slice API (grow only).
  void* d_w = nullptr;
  size_t d_w_cap = 0;
  float* d_x = nullptr;
  size_t d_x_cap = 0;
  float* d_y = nullptr;
  size_t d_y_cap = 0;
  cudaEvent_t ev[8] = {};
};

namespace {

struct DeviceGuard {
  int prev = -1;
  bool switched = false;
  int enter(int device) {
    OBJB_CUDA(cudaGetDevice(&prev), "query current device");
    if (prev != device) {
      OBJB_CUDA(cudaSetDevice(device), "select device");
      switched = true;
    }
    return OBJB_OK;
  }
  ~DeviceGuard() {
    if (switched) cudaSetDevice(prev);
  }
};

int grow(void** p, size_t* cap, size_t need, const char* what) {
  if (need <= *cap) return OBJB_OK;
  if (*p) cudaFree(*p);
  *p = nullptr;
  *cap = 0;
  OBJB_CUDA(cudaMalloc(p, need), what);
  *cap = need;
  return OBJB_OK;
}

}  // namespace

extern "C" {

int objb_gemv_device(int fmt, const void* d_qweights, const float* d_x, float* d_y, size_t rows,
                     size_t cols, objb_stream_t stream) {
  objb::clear_error();
  return objb::gemv_device(fmt, d_qweights, d_x, d_y, rows, cols, static_cast<cudaStream_t>(stream));
}

int objb_gemv_fp4_split_device(const void* d_weight, const void* d_scale, const float* d_x,
                               float* d_y, size_t rows, size_t cols, objb_stream_t stream) {
  objb::clear_error();
  return objb::gemv_fp4_split_device(d_weight, d_scale, d_x, d_y, rows, cols,
                                     static_cast<cudaStream_t>(stream));
}

int objb_pipe_plan_info(int fmt, int split_fp4, size_t rows, size_t cols, int blocks_per_lane, int dual,
                        int moe_program, int32_t* out, int nout) {
  objb::clear_error();
  if (!out || nout < 9) return OBJB_FAIL(OBJB_ERR_INVALID_INPUT, "objb_pipe_plan_info", "output needs 9 entries");
  if (!objb::valid_format(fmt) || (split_fp4 && fmt != OBJB_FP4_E2M1))
    return OBJB_FAIL(OBJB_ERR_INVALID_INPUT, "objb_pipe_plan_info", "unknown format");
  if (blocks_per_lane != 2 && !(blocks_per_lane == 1 && split_fp4))
    return OBJB_FAIL(OBJB_ERR_INVALID_INPUT, "objb_pipe_plan_info",
                     "blocks_per_lane is 2 (1 only for split FP4 rows)");
  if (rows == 0 || cols == 0 || cols % 32 || rows > (1u << 30) || cols > (1u << 24))
    return OBJB_FAIL(OBJB_ERR_INVALID_INPUT, "objb_pipe_plan_info", "shape outside the pipelined kernel's range");
  const int r = static_cast<int>(rows), c = static_cast<int>(cols);
  const int rb = split_fp4 ? c / 2 : c / 32 * objb::block_bytes(fmt), srb = split_fp4 ? c / 32 : 0;
  const int budget = moe_program ? objb::kMoeSmemBudget : objb::kGemvSmemBudget;
  objb::RowLayoutHost L;
  if (!objb::plan_rows(r, c, rb, srb, blocks_per_lane, dual != 0, objb::dev::kMaxConsumerWarps, &L, budget))
    return OBJB_FAIL(OBJB_ERR_UNSUPPORTED, "objb_pipe_plan_info", "the shape cannot use the bulk-copy path");
  // would a 16-byte aligned vector be formed in-kernel (one vector per launch)?
  const float* aligned = reinterpret_cast<const float*>(static_cast<uintptr_t>(256));
  bool inl = false;
  if (split_fp4) inl = blocks_per_lane == 2 ? objb::inline_x_ok<objb::dev::RowDotSplitFp4Digit>(L, aligned)
                                            : objb::inline_x_ok<objb::dev::RowDotSplitFp4DigitT<1>>(L, aligned);
  else if (fmt == OBJB_Q4_0) inl = objb::inline_x_ok<objb::dev::RowDot<OBJB_Q4_0>>(L, aligned);
  else if (fmt == OBJB_Q5_0) inl = objb::inline_x_ok<objb::dev::RowDot<OBJB_Q5_0>>(L, aligned);
  else if (fmt == OBJB_IQ3_0) inl = objb::inline_x_ok<objb::dev::RowDot<OBJB_IQ3_0>>(L, aligned);
  else inl = objb::inline_x_ok<objb::dev::RowDot<OBJB_FP4_E2M1>>(L, aligned);
  const int32_t v[9] = {L.nseg, L.ngrp, L.tstage, L.nslots, L.stage_bytes,
                        static_cast<int32_t>(objb::pipe_smem_bytes(L)), L.ngrp * 4, inl ? 1 : 0, budget};
  for (int i = 0; i < 9; ++i) out[i] = v[i];
  return OBJB_OK;
}

int objb_quant_backend_new(int device, objb_quant_backend** out) {
  objb::clear_error();
  if (!out) return OBJB_FAIL(OBJB_ERR_INVALID_INPUT, "objb_quant_backend_new", "null output pointer");
  objb::DeviceProps props;
  OBJB_TRY(objb::device_props(device, &props));
  auto* qb = new objb_quant_backend();
  qb->device = device;
  DeviceGuard g;
  int rc = g.enter(device);
  if (rc != OBJB_OK) {
    delete qb;
    return rc;
  }
  for (auto& e : qb->ev) {
    if (cudaEventCreate(&e) != cudaSuccess) {
      delete qb;
      return OBJB_FAIL(OBJB_ERR_RUNTIME, "create telemetry events", "cudaEventCreate failed");
    }
  }
  *out = qb;
  return OBJB_OK;
}

void objb_quant_backend_free(objb_quant_backend* qb) {
  if (!qb) return;
  DeviceGuard g;
  g.enter(qb->device);
  for (auto& e : qb->ev)
    if (e) cudaEventDestroy(e);
  if (qb->d_w) cudaFree(qb->d_w);
  if (qb->d_x) cudaFree(qb->d_x);
  if (qb->d_y) cudaFree(qb->d_y);
  delete qb;
}

int objb_quant_backend_compile_format(objb_quant_backend* qb, int fmt) {
  objb::clear_error();
  if (!qb) return OBJB_FAIL(OBJB_ERR_INVALID_INPUT, "objb_quant_backend_compile_format", "null backend");
  if (!objb::valid_format(fmt))
    return OBJB_FAIL(OBJB_ERR_INVALID_INPUT, "compile quant format", "unknown QuantFormat ordinal " + std::to_string(fmt));
  DeviceGuard g;
  OBJB_TRY(g.enter(qb->device));
  // Loading is eager for a prebuilt fatbin; query one kernel so a missing or
  // mismatched image fails here rather than at the first launch.
  cudaFuncAttributes attr;
  cudaError_t e;
  switch (fmt) {
    case OBJB_Q4_0: e = cudaFuncGetAttributes(&attr, objb::dev::gemv_fallback_kernel<OBJB_Q4_0>); break;
    case OBJB_Q5_0: e = cudaFuncGetAttributes(&attr, objb::dev::gemv_fallback_kernel<OBJB_Q5_0>); break;
    case OBJB_IQ3_0: e = cudaFuncGetAttributes(&attr, objb::dev::gemv_fallback_kernel<OBJB_IQ3_0>); break;
    default: e = cudaFuncGetAttributes(&attr, objb::dev::gemv_fallback_kernel<OBJB_FP4_E2M1>); break;
  }
  if (e != cudaSuccess) return objb::cuda_status(e, "load prebuilt sm_100a GEMV kernels", __FILE__, __LINE__);
  return OBJB_OK;
}

int objb_gemv_host(objb_quant_backend* qb, int fmt, objb_stream_t stream_, const uint8_t* qweights,
                   size_t qweights_len, const float* x, size_t x_len, size_t rows, size_t cols,
                   float* y, objb_qgemv_telemetry* tel) {
  objb::clear_error();
  if (!qb) return OBJB_FAIL(OBJB_ERR_INVALID_INPUT, "objb_gemv_host", "null backend");
  OBJB_TRY(objb::validate_gemv_shape(fmt, rows, cols));
  const std::string label = objb::format_label(fmt);
  const size_t qbytes = rows * (cols / 32) * static_cast<size_t>(objb::block_bytes(fmt));
  if (qweights_len != qbytes)
    return OBJB_FAIL(OBJB_ERR_INVALID_INPUT, ("validate " + label + " quantized matrix size").c_str(),
                     "qweights len " + std::to_string(qweights_len) + " != expected " + std::to_string(qbytes));
  if (x_len != cols)
    return OBJB_FAIL(OBJB_ERR_INVALID_INPUT, ("validate " + label + " GEMV vector size").c_str(),
                     "x len " + std::to_string(x_len) + " != cols " + std::to_string(cols));
  std::lock_guard<std::mutex> lk(qb->mu);
  DeviceGuard g;
  OBJB_TRY(g.enter(qb->device));
  cudaStream_t stream = static_cast<cudaStream_t>(stream_);
  OBJB_TRY(grow(&qb->d_w, &qb->d_w_cap, std::max<size_t>(qbytes, 16), "allocate device weights"));
  OBJB_TRY(grow(reinterpret_cast<void**>(&qb->d_x), &qb->d_x_cap, std::max<size_t>(cols * 4, 16), "allocate device x"));
  OBJB_TRY(grow(reinterpret_cast<void**>(&qb->d_y), &qb->d_y_cap, std::max<size_t>(rows * 4, 16), "allocate device y"));
  cudaEvent_t* ev = qb->ev;
  OBJB_CUDA(cudaEventRecord(ev[0], stream), "record total start");
  OBJB_CUDA(cudaEventRecord(ev[1], stream), "record h2d start");
  if (qbytes) OBJB_CUDA(cudaMemcpyAsync(qb->d_w, qweights, qbytes, cudaMemcpyHostToDevice, stream), "copy weights to device");
  if (cols) OBJB_CUDA(cudaMemcpyAsync(qb->d_x, x, cols * 4, cudaMemcpyHostToDevice, stream), "copy x to device");
  OBJB_CUDA(cudaEventRecord(ev[2], stream), "record h2d stop");
  OBJB_CUDA(cudaMemsetAsync(qb->d_y, 0, std::max<size_t>(rows * 4, 4), stream), "zero y");
  OBJB_CUDA(cudaEventRecord(ev[3], stream), "record kernel start");
  OBJB_TRY(objb::gemv_device(fmt, qb->d_w, qb->d_x, qb->d_y, rows, cols, stream));
  OBJB_CUDA(cudaEventRecord(ev[4], stream), "record kernel stop");
  OBJB_CUDA(cudaEventRecord(ev[5], stream), "record d2h start");
  if (rows) OBJB_CUDA(cudaMemcpyAsync(y, qb->d_y, rows * 4, cudaMemcpyDeviceToHost, stream), "copy y to host");
  OBJB_CUDA(cudaEventRecord(ev[6], stream), "record d2h stop");
  OBJB_CUDA(cudaEventRecord(ev[7], stream), "record total stop");
  OBJB_CUDA(cudaStreamSynchronize(stream), "synchronize GEMV stream");
  unsigned werr = 0;
  {
    unsigned* w = nullptr;
    OBJB_TRY(objb::device_error_word(qb->device, &w));
    OBJB_CUDA(cudaMemcpy(&werr, w, sizeof(werr), cudaMemcpyDeviceToHost), "read device error word");
    if (werr) {
      cudaMemset(w, 0, sizeof(unsigned));
      return OBJB_FAIL(OBJB_ERR_INTERNAL, "run pipelined GEMV", "bounded pipeline wait expired (code " + std::to_string(werr) + ")");
    }
  }
  if (tel) {
    float h2d = 0, ker = 0, d2h = 0, tot = 0;
    OBJB_CUDA(cudaEventElapsedTime(&h2d, ev[1], ev[2]), "read h2d time");
    OBJB_CUDA(cudaEventElapsedTime(&ker, ev[3], ev[4]), "read kernel time");
    OBJB_CUDA(cudaEventElapsedTime(&d2h, ev[5], ev[6]), "read d2h time");
    OBJB_CUDA(cudaEventElapsedTime(&tot, ev[0], ev[7]), "read total time");
    tel->h2d_ms = h2d;
    tel->kernel_ms = ker;
    tel->d2h_ms = d2h;
    tel->total_ms = tot;
    tel->unaccounted_ms = std::max(0.0f, tot - h2d - ker - d2h);
    tel->bytes_read = qbytes + cols * 4;  // quant.rs:282
    tel->effective_gbps = ker > 0 ? static_cast<float>(tel->bytes_read) / (ker / 1000.0f) / 1.0e9f : 0.0f;
  }
  return OBJB_OK;
}

}  // extern "C"
