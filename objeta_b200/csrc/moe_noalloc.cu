// moe_noalloc.cu -- the selected-expert MoE launch for callers that cannot
// allocate device memory.
//
// objb_moe_selected_device takes its scratch (the SwiGLU activations and the
// x images) from a per-stream workspace that it allocates with cudaMalloc the
// first time a stream is used.  Some callers cannot let a library do that:
// a host framework that owns every byte of device memory and forbids
// allocations on its hot path (serving engines that reserve HBM up front),
// code that runs while the framework's own allocator holds its lock, or a
// plugin loaded into a process whose allocator must see every allocation.
// This file gives them the same launch with the scratch taken from a fixed
// array that is part of the library's device image: nothing is allocated,
// ever, by this entry point.
#include <cuda_runtime.h>

#include <mutex>
#include <string>

#include "objb_common.h"
#include "objb_launch.h"
#include "objb_moe_launch.h"

namespace objb {
namespace {

// 4 MiB per GPU, resident from the moment the library is loaded on a device
// until the process exits.  The first 256 bytes hold the launch's error word;
// the rest is MoE scratch.  A BASELINE-size layer (top-8 of 256 FP4 experts,
// hidden 4096, intermediate 2048) needs about 150 KB; top-2 Q4 with
// intermediate 14336 about 230 KB.
constexpr size_t kNoAllocBytes = 4u << 20;
constexpr size_t kNoAllocErrBytes = 256;
static __device__ __align__(256) unsigned char g_noalloc_scratch[kNoAllocBytes];

std::mutex g_mu;
constexpr int kMaxDevices = 64;
void* g_addr[kMaxDevices] = {};

// The device address of g_noalloc_scratch on `device` (the current device).
// In host code the array's name is only a stand-in; the address a kernel may
// use comes from cudaGetSymbolAddress, queried once per device.
int scratch_address(int device, void** out) {
  if (device < 0 || device >= kMaxDevices)
    return OBJB_FAIL(OBJB_ERR_UNSUPPORTED, "locate allocation-free scratch", "device ordinal out of range");
  std::lock_guard<std::mutex> lk(g_mu);
  if (!g_addr[device]) {
    void* p = nullptr;
    const cudaError_t e = cudaGetSymbolAddress(&p, g_noalloc_scratch);
    if (e != cudaSuccess) return cuda_status(e, "look up the allocation-free scratch array", __FILE__, __LINE__);
    g_addr[device] = p;
  }
  *out = g_addr[device];
  return OBJB_OK;
}

// The regular entry point reports device-side errors (an out-of-range expert
// id, a pipeline wait that ran out) through a per-device error word that the
// library allocates; this one cannot allocate, so its error word lives in the
// array and is made visible here instead: when it is nonzero after the launch,
// every output element becomes NaN.
__global__ void poison_on_error_kernel(const unsigned* err, float* out, int n) {
  const int i = blockIdx.x * blockDim.x + threadIdx.x;
  if (i < n && *err != 0u) out[i] = __int_as_float(0x7fc00000);
}

}  // namespace
}  // namespace objb

extern "C" {

int objb_moe_selected_device_noalloc(const objb_moe_layer* layer, const int32_t* d_ids, const float* d_weights,
                                     size_t top_k, const float* d_x, float* d_out, float swiglu_limit,
                                     objb_stream_t stream_) {
  objb::clear_error();
  size_t need = 0;
  OBJB_TRY(objb::moe_scratch_bytes(layer, top_k, &need));
  const size_t have = objb::kNoAllocBytes - objb::kNoAllocErrBytes;
  if (need > have)
    return OBJB_FAIL(OBJB_ERR_INVALID_INPUT, "objb_moe_selected_device_noalloc",
                     "this layer needs " + std::to_string(need) + " bytes of scratch for top_k " +
                         std::to_string(top_k) + "; the allocation-free entry point has a fixed " +
                         std::to_string(have) + "-byte array (use objb_moe_selected_device)");
  int device = 0;
  OBJB_TRY(objb::current_device(&device));
  void* base = nullptr;
  OBJB_TRY(objb::scratch_address(device, &base));
  cudaStream_t stream = static_cast<cudaStream_t>(stream_);
  unsigned* err = static_cast<unsigned*>(base);
  // Only the error word must start at zero; every scratch byte the launch
  // reads is written earlier in the same launch sequence.
  OBJB_CUDA(cudaMemsetAsync(err, 0, sizeof(unsigned), stream), "clear the allocation-free error word");
  void* scratch = static_cast<unsigned char*>(base) + objb::kNoAllocErrBytes;
  OBJB_TRY(objb::moe_selected(layer, d_ids, d_weights, top_k, d_x, d_out, swiglu_limit, stream, scratch, have,
                              nullptr, err));
  const int n = static_cast<int>(layer->out_dim);
  objb::poison_on_error_kernel<<<(n + 255) / 256, 256, 0, stream>>>(err, d_out, n);
  OBJB_CUDA(cudaGetLastError(), "launch the allocation-free error check");
  return OBJB_OK;
}

}  // extern "C"
