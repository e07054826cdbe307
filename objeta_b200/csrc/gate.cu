// gate.cu -- the DeepSeek V4 gate on the device (cpu_gate_ref,
// crates/objeta-cuda/src/bin/deepseek_single_layer_moe.rs:768-881), one CTA
// per token:
//   logits = W h (one thread per expert, sequential f32 multiply-then-add in
//            the reference's order, so the logits are bit-identical);
//   scores = softmax | sigmoid | sqrt(softplus) of the logits (exp / log1p in
//            double, rounded to f32; softplus keeps the reference's branches,
//            including log1p(exp(-v)) below -20);
//   ids    = top_k of scores + bias by a stable descending rank (ties keep the
//            lower index), or tid2eid[input_id * top_k + k] for hash layers;
//   weights = scores[ids], divided by their sequential sum unless softmax,
//            times route_scale.
#include <cuda_runtime.h>

#include <string>

#include "objb_common.h"
#include "objb_launch.h"

namespace objb {
namespace dev {

__global__ void __launch_bounds__(1024) deepseek_gate_kernel(const float* __restrict__ gw,
                                                             const float* __restrict__ bias,
                                                             const int64_t* __restrict__ tid2eid, long long vocab,
                                                             const float* __restrict__ hidden,
                                                             const int64_t* __restrict__ input_ids, int E, int H,
                                                             int K, int score_func, float route_scale,
                                                             int32_t* __restrict__ ids, float* __restrict__ weights,
                                                             unsigned* err) {
  extern __shared__ float sm[];  // scores [E], selection [E]
  float* scores = sm;
  float* sel = sm + E;
  __shared__ float s_red;
  const int t = blockIdx.x;
  const float* h = hidden + static_cast<size_t>(t) * H;
  ids += static_cast<size_t>(t) * K;
  weights += static_cast<size_t>(t) * K;
  for (int e = threadIdx.x; e < E; e += blockDim.x) {
    const float* row = gw + static_cast<size_t>(e) * H;
    float sum = 0.0f;
    for (int i = 0; i < H; ++i) sum = __fadd_rn(sum, __fmul_rn(row[i], h[i]));
    scores[e] = sum;  // logits for now
  }
  __syncthreads();
  if (score_func == 0) {
    if (threadIdx.x == 0) {
      float m = -__int_as_float(0x7F800000);
      for (int e = 0; e < E; ++e) m = fmaxf(m, scores[e]);
      s_red = m;
    }
    __syncthreads();
    for (int e = threadIdx.x; e < E; e += blockDim.x)
      sel[e] = __double2float_rn(exp(static_cast<double>(__fsub_rn(scores[e], s_red))));
    __syncthreads();
    if (threadIdx.x == 0) {
      float s = 0.0f;
      for (int e = 0; e < E; ++e) s = __fadd_rn(s, sel[e]);
      s_red = s;
    }
    __syncthreads();
    for (int e = threadIdx.x; e < E; e += blockDim.x) scores[e] = __fdiv_rn(sel[e], s_red);
  } else {
    for (int e = threadIdx.x; e < E; e += blockDim.x) {
      const float v = scores[e];
      float r;
      if (score_func == 1) {
        r = __fdiv_rn(1.0f, __fadd_rn(1.0f, __double2float_rn(exp(-static_cast<double>(v)))));
      } else {
        float sp;
        if (v > 20.0f) {
          sp = v;
        } else {
          const float ex = __double2float_rn(exp(v < -20.0f ? -static_cast<double>(v) : static_cast<double>(v)));
          sp = __double2float_rn(log1p(static_cast<double>(ex)));
        }
        r = __fsqrt_rn(sp);
      }
      scores[e] = r;
    }
  }
  __syncthreads();
  if (tid2eid) {
    const long long id = input_ids ? input_ids[t] : -1;
    const bool ok = id >= 0 && id < vocab;
    if (!ok && threadIdx.x == 0 && err) atomicOr(err, 8u);  // input id out of range: ids -1, weights NaN
    for (int k = threadIdx.x; k < K; k += blockDim.x) {
      const long long e = ok ? tid2eid[id * K + k] : -1;
      ids[k] = static_cast<int32_t>(e);
    }
  } else {
    for (int e = threadIdx.x; e < E; e += blockDim.x) sel[e] = bias ? __fadd_rn(scores[e], bias[e]) : scores[e];
    __syncthreads();
    for (int e = threadIdx.x; e < E; e += blockDim.x) {
      const float pe = sel[e];
      int rank = 0;
      for (int j = 0; j < E; ++j) {
        const float pj = sel[j];
        rank += (pj > pe) || (pj == pe && j < e);
      }
      if (rank < K) ids[rank] = e;
    }
  }
  __syncthreads();
  if (threadIdx.x == 0) {
    float s = 0.0f;
    for (int k = 0; k < K; ++k) {
      const int e = ids[k];
      const float w = (e >= 0 && e < E) ? scores[e] : __int_as_float(0x7FC00000);
      if (!(e >= 0 && e < E) && err) atomicOr(err, 8u);
      weights[k] = w;
      s = __fadd_rn(s, w);
    }
    for (int k = 0; k < K; ++k) {
      float w = weights[k];
      if (score_func != 0 && s > 0.0f) w = __fdiv_rn(w, s);
      weights[k] = __fmul_rn(w, route_scale);
    }
  }
}

}  // namespace dev
}  // namespace objb

extern "C" {

int objb_deepseek_gate_device(const float* d_gate_weight, const float* d_gate_bias, const int64_t* d_tid2eid,
                              size_t tid2eid_len, const float* d_hidden, const int64_t* d_input_ids,
                              size_t num_tokens, size_t num_experts, size_t hidden_size, size_t top_k,
                              int score_func, float route_scale, int32_t* d_ids, float* d_weights,
                              objb_stream_t stream) {
  objb::clear_error();
  if (!d_gate_weight || !d_hidden || !d_ids || !d_weights)
    return OBJB_FAIL(OBJB_ERR_INVALID_INPUT, "cpu_gate_ref", "null device pointer");
  if (score_func < 0 || score_func > 2)
    return OBJB_FAIL(OBJB_ERR_INVALID_INPUT, "cpu_gate_ref", "score_func must be 0 (softmax), 1 (sigmoid) or 2");
  if (num_tokens == 0 || num_tokens > 65535 || num_experts == 0 || num_experts > 8192 || top_k == 0 ||
      top_k > num_experts || hidden_size == 0 || hidden_size > (1u << 20))
    return OBJB_FAIL(OBJB_ERR_INVALID_INPUT, "cpu_gate_ref", "shape out of range");
  if (d_tid2eid && !d_input_ids)
    return OBJB_FAIL(OBJB_ERR_INVALID_INPUT, "cpu_gate_ref hash layer", "input_id is required for hash layers");
  int device = 0;
  OBJB_TRY(objb::current_device(&device));
  unsigned* err = nullptr;
  OBJB_TRY(objb::device_error_word(device, &err));
  const size_t smem = 2 * num_experts * sizeof(float);
  if (smem > 48 * 1024)
    OBJB_CUDA(cudaFuncSetAttribute(objb::dev::deepseek_gate_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                   static_cast<int>(smem)),
              "opt the gate into large shared memory");
  const int threads = static_cast<int>(num_experts >= 1024 ? 1024 : (num_experts + 31) / 32 * 32);
  objb::dev::deepseek_gate_kernel<<<static_cast<unsigned>(num_tokens), threads, smem,
                                    static_cast<cudaStream_t>(stream)>>>(
      d_gate_weight, d_gate_bias, d_tid2eid, static_cast<long long>(d_tid2eid ? tid2eid_len / top_k : 0), d_hidden,
      d_input_ids, static_cast<int>(num_experts), static_cast<int>(hidden_size), static_cast<int>(top_k), score_func,
      route_scale, d_ids, d_weights, err);
  OBJB_CUDA(cudaGetLastError(), "launch DeepSeek gate");
  return OBJB_OK;
}

}  // extern "C"
