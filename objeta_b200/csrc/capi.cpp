// capi.cpp -- error recording, metadata and device plumbing of the C ABI.
#include <cuda_runtime.h>

#include <cmath>

#include <cstdio>
#include <algorithm>
#include <cstring>
#include <map>
#include <mutex>
#include <string>
#include <vector>

#include "objb_common.h"
#include "objb_launch.h"

namespace objb {
namespace {

thread_local int g_last_status = OBJB_OK;
thread_local std::string g_last_message;

const char* kind_name(int kind) {
  // CudaErrorKind variant names (lib.rs:39-48).
  switch (kind) {
    case OBJB_ERR_DRIVER: return "Driver";
    case OBJB_ERR_RUNTIME: return "Runtime";
    case OBJB_ERR_NVRTC: return "Nvrtc";
    case OBJB_ERR_IO: return "Io";
    case OBJB_ERR_INVALID_INPUT: return "InvalidInput";
    case OBJB_ERR_UNSUPPORTED: return "Unsupported";
    default: return "Internal";
  }
}

std::mutex g_dev_mu;
std::vector<DeviceProps> g_props;
std::vector<bool> g_props_ok;
std::vector<unsigned*> g_err_words;

}  // namespace

int set_error(int kind, const char* action, const std::string& message, const char* file, int line) {
  const char* base = std::strrchr(file, '/');
  base = base ? base + 1 : file;
  char head[512];
  std::snprintf(head, sizeof(head), "%s error during %s at objeta_b200::%s:%d (%s): ",
                kind_name(kind), action, base, line, file);
  g_last_status = kind;
  g_last_message = std::string(head) + message;
  return kind;
}

void clear_error() {
  g_last_status = OBJB_OK;
  g_last_message.clear();
}

int cuda_status(cudaError_t e, const char* action, const char* file, int line) {
  std::string msg = std::string(cudaGetErrorName(e)) + ": " + cudaGetErrorString(e);
  return set_error(OBJB_ERR_RUNTIME, action, msg, file, line);
}

const char* format_label(int fmt) {
  // QuantFormat::format_label (quant.rs:61-68).
  switch (fmt) {
    case OBJB_Q4_0: return "q4_0";
    case OBJB_Q5_0: return "q5_0";
    case OBJB_IQ3_0: return "iq3_0";
    case OBJB_FP4_E2M1: return "deepseek_fp4_e2m1";
    default: return "unknown";
  }
}

int validate_gemv_shape(int fmt, size_t rows, size_t cols) {
  (void)rows;
  if (!valid_format(fmt))
    return OBJB_FAIL(OBJB_ERR_INVALID_INPUT, "validate quant format", "unknown QuantFormat ordinal " + std::to_string(fmt));
  if (cols % 32 != 0) {
    std::string action = std::string("validate ") + format_label(fmt) + " column alignment";
    return OBJB_FAIL(OBJB_ERR_INVALID_INPUT, action.c_str(),
                     "cols " + std::to_string(cols) + " must be a multiple of block_size 32");
  }
  return OBJB_OK;
}

int current_device(int* dev) {
  OBJB_CUDA(cudaGetDevice(dev), "query current CUDA device");
  return OBJB_OK;
}

int device_props(int device, DeviceProps* out) {
  std::lock_guard<std::mutex> lk(g_dev_mu);
  if (device < 0) return OBJB_FAIL(OBJB_ERR_INVALID_INPUT, "query device properties", "negative device ordinal");
  if (static_cast<size_t>(device) >= g_props.size()) {
    g_props.resize(device + 1);
    g_props_ok.resize(device + 1, false);
  }
  if (!g_props_ok[device]) {
    cudaDeviceProp p;
    OBJB_CUDA(cudaGetDeviceProperties(&p, device), "query device properties");
    DeviceProps d;
    d.sm_count = p.multiProcessorCount;
    d.max_smem_optin = static_cast<int>(p.sharedMemPerBlockOptin);
    d.l2_bytes = static_cast<size_t>(p.l2CacheSize);
    d.cc_major = p.major;
    d.cc_minor = p.minor;
    if (d.cc_major != 10) {
      return OBJB_FAIL(OBJB_ERR_UNSUPPORTED, "select kernels for the device",
                       std::string("device ") + p.name + " has compute capability " +
                           std::to_string(p.major) + "." + std::to_string(p.minor) +
                           "; libobjeta_b200 carries sm_100a code only");
    }
    g_props[device] = d;
    g_props_ok[device] = true;
  }
  *out = g_props[device];
  return OBJB_OK;
}

int device_error_word(int device, unsigned** out) {
  std::lock_guard<std::mutex> lk(g_dev_mu);
  if (static_cast<size_t>(device) >= g_err_words.size()) g_err_words.resize(device + 1, nullptr);
  if (!g_err_words[device]) {
    unsigned* w = nullptr;
    OBJB_CUDA(cudaMalloc(&w, sizeof(unsigned)), "allocate device error word");
    OBJB_CUDA(cudaMemset(w, 0, sizeof(unsigned)), "clear device error word");
    g_err_words[device] = w;
  }
  *out = g_err_words[device];
  return OBJB_OK;
}

namespace {
std::mutex g_ws_mu;
struct WsKey {
  int device;
  cudaStream_t stream;
  bool operator<(const WsKey& o) const {
    return device != o.device ? device < o.device : stream < o.stream;
  }
};
struct WsBuf {
  void* ptr = nullptr;
  size_t bytes = 0;
};
std::map<WsKey, WsBuf> g_ws;
}  // namespace

int workspace_get(int device, cudaStream_t stream, size_t bytes, void** out) {
  std::lock_guard<std::mutex> lk(g_ws_mu);
  WsBuf& b = g_ws[WsKey{device, stream}];
  if (b.bytes >= bytes && b.ptr) {
    *out = b.ptr;
    return OBJB_OK;
  }
  cudaStreamCaptureStatus cs = cudaStreamCaptureStatusNone;
  OBJB_CUDA(cudaStreamIsCapturing(stream, &cs), "query stream capture state");
  if (cs != cudaStreamCaptureStatusNone)
    return OBJB_FAIL(OBJB_ERR_INVALID_INPUT, "allocate stream workspace",
                     "the per-stream workspace must be allocated before stream capture: make one "
                     "uncaptured call with this shape on this stream first");
  if (b.ptr) {
    OBJB_CUDA(cudaStreamSynchronize(stream), "drain stream before growing its workspace");
    cudaFree(b.ptr);
    b.ptr = nullptr;
    b.bytes = 0;
  }
  const size_t want = std::max<size_t>(bytes, kWorkspaceMinBytes);
  OBJB_CUDA(cudaMalloc(&b.ptr, want), "allocate stream workspace");
  b.bytes = want;
  *out = b.ptr;
  return OBJB_OK;
}

}  // namespace objb

using namespace objb;

extern "C" {

int objb_last_error(char* buf, size_t len) {
  if (buf && len) {
    size_t n = g_last_message.size() < len - 1 ? g_last_message.size() : len - 1;
    std::memcpy(buf, g_last_message.data(), n);
    buf[n] = '\0';
  }
  return g_last_status;
}

int objb_abi_version(void) { return 100; }

int objb_format_info_get(int fmt, objb_format_info* out) {
  clear_error();
  if (!out) return OBJB_FAIL(OBJB_ERR_INVALID_INPUT, "objb_format_info_get", "null output pointer");
  if (!valid_format(fmt))
    return OBJB_FAIL(OBJB_ERR_INVALID_INPUT, "objb_format_info_get", "unknown QuantFormat ordinal " + std::to_string(fmt));
  // QuantFormat methods, quant.rs:33-96.
  static const char* kernel_names[] = {"q4_gemv", "q5_gemv", "iq3_gemv", "fp4_e2m1_gemv"};
  out->block_size = 32;
  out->block_bytes = static_cast<uint32_t>(block_bytes(fmt));
  out->packed_values_per_byte = 2;
  out->kernel_name = kernel_names[fmt];
  out->format_label = format_label(fmt);
  out->scale_dtype = fmt == OBJB_FP4_E2M1 ? "F8_E8M0" : "F16";
  out->nibble_order = "low_first";
  return OBJB_OK;
}

int objb_qgemv_shape_new(int fmt, size_t rows, size_t cols, objb_qgemv_shape* out) {
  clear_error();
  if (!out) return OBJB_FAIL(OBJB_ERR_INVALID_INPUT, "objb_qgemv_shape_new", "null output pointer");
  OBJB_TRY(validate_gemv_shape(fmt, rows, cols));
  out->rows = rows;
  out->cols = cols;
  out->block_size = 32;
  out->block_bytes = static_cast<size_t>(block_bytes(fmt));
  out->blocks_per_row = cols / 32;
  out->quantized_row_bytes = out->blocks_per_row * out->block_bytes;
  out->quantized_matrix_bytes = rows * out->quantized_row_bytes;
  return OBJB_OK;
}

int objb_device_info_get(int device, objb_device_info* out) {
  clear_error();
  if (!out) return OBJB_FAIL(OBJB_ERR_INVALID_INPUT, "objb_device_info_get", "null output pointer");
  cudaDeviceProp p;
  OBJB_CUDA(cudaGetDeviceProperties(&p, device), "query device properties");
  out->ordinal = device;
  out->total_global_mem_bytes = p.totalGlobalMem;
  out->compute_capability_major = p.major;
  out->compute_capability_minor = p.minor;
  out->multiprocessor_count = p.multiProcessorCount;
  out->l2_cache_bytes = static_cast<size_t>(p.l2CacheSize);
  return OBJB_OK;
}

int objb_host_register(void* ptr, size_t bytes) {
  clear_error();
  if (!ptr || !bytes) return OBJB_FAIL(OBJB_ERR_INVALID_INPUT, "objb_host_register", "empty host range");
  OBJB_CUDA(cudaHostRegister(ptr, bytes, cudaHostRegisterDefault), "pin host range");
  return OBJB_OK;
}

int objb_host_unregister(void* ptr) {
  clear_error();
  OBJB_CUDA(cudaHostUnregister(ptr), "unpin host range");
  return OBJB_OK;
}

int objb_compare_outputs(const float* reference, size_t reference_len, const float* actual, size_t actual_len,
                         objb_qgemv_numerics* out) {
  clear_error();
  if (!out || (reference_len && !reference) || (actual_len && !actual))
    return OBJB_FAIL(OBJB_ERR_INVALID_INPUT, "compare quantized GEMV outputs", "null argument");
  if (reference_len != actual_len)
    return OBJB_FAIL(OBJB_ERR_INVALID_INPUT, "compare quantized GEMV outputs",
                     "reference len " + std::to_string(reference_len) + " != actual len " +
                         std::to_string(actual_len));
  // f64 sums in element order; the difference and its magnitude in f32.
  double dot = 0.0, ref_norm = 0.0, act_norm = 0.0, sq_err = 0.0;
  float max_abs = 0.0f;
  for (size_t i = 0; i < reference_len; ++i) {
    const double r = reference[i], a = actual[i];
    dot += r * a;
    ref_norm += r * r;
    act_norm += a * a;
    const float diff = actual[i] - reference[i];
    sq_err += static_cast<double>(diff) * static_cast<double>(diff);
    max_abs = std::fmax(max_abs, std::fabs(diff));
  }
  out->cosine_similarity =
      ref_norm > 0.0 && act_norm > 0.0 ? static_cast<float>(dot / (std::sqrt(ref_norm) * std::sqrt(act_norm))) : 1.0f;
  out->relative_l2_error = ref_norm > 0.0 ? static_cast<float>(std::sqrt(sq_err) / std::sqrt(ref_norm)) : 0.0f;
  out->max_abs_error = max_abs;
  return OBJB_OK;
}

int objb_device_error_take(int device, unsigned* word) {
  clear_error();
  unsigned* w = nullptr;
  OBJB_TRY(device_error_word(device, &w));
  int prev = 0;
  OBJB_CUDA(cudaGetDevice(&prev), "query current device");
  if (prev != device) OBJB_CUDA(cudaSetDevice(device), "select device");
  unsigned v = 0;
  cudaError_t e = cudaMemcpy(&v, w, sizeof(v), cudaMemcpyDeviceToHost);
  if (e == cudaSuccess) e = cudaMemset(w, 0, sizeof(unsigned));
  if (prev != device) cudaSetDevice(prev);
  if (e != cudaSuccess) return cuda_status(e, "read device error word", __FILE__, __LINE__);
  if (word) *word = v;
  return OBJB_OK;
}

}  // extern "C"
