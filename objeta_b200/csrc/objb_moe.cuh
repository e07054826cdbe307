// objb_moe.cuh -- programs for the selected-expert MoE on the row-streaming
// pipeline (objb_gemv.cuh), plus the router.
//
// One token's MoE layer runs as
//   [router]  -> x image -> gate/up (both matrices of every selected expert
//   streamed through the same stages, SwiGLU in the epilogue) -> act images
//   -> down (all selected experts of an output row block in one CTA, the
//   weighted combine in the epilogue, in selection order).
#pragma once

#include <cstdint>

#include "objb_gemv.cuh"

namespace objb {
namespace dev {

// silu_mul (crates/objeta-cuda/kernels/moe.cu:2-22): with limit > 0 the up
// value is clamped to [-limit, limit] and the gate to <= limit; then
// act = g / (1 + exp(-g)) * u.
// The official DeepSeek experts (deepseek.rs:1675-1680, 1707-1711) clamp only
// the up value: clamp_gate = false.
__device__ __forceinline__ float swiglu(float g, float u, float limit, bool clamp_gate = true) {
  if (limit > 0.0f) {
    u = fminf(limit, fmaxf(-limit, u));
    if (clamp_gate) g = fminf(limit, g);
  }
  const float silu = __fdiv_rn(g, __fadd_rn(1.0f, expf(-g)));
  return __fmul_rn(silu, u);
}

// Expert tables as the kernels see them.
struct ExpertTables {
  const uint8_t* const* gate;
  const uint8_t* const* up;
  const uint8_t* const* down;
  const uint8_t* const* gate_scale;  // split FP4 only
  const uint8_t* const* up_scale;
  const uint8_t* const* down_scale;
  int num_experts;
};

__device__ __forceinline__ int checked_expert(const int32_t* ids, int k, int num_experts, unsigned* err) {
  int e = ids[k];
  if (e < 0 || e >= num_experts) {
    if (err) atomicOr(err, 8u);  // out-of-range expert id: computed as expert 0, flagged
    e = 0;
  }
  return e;
}

// gate/up: CTA c covers rows [c * R, (c + 1) * R) of the K * I rows of all
// selected experts concatenated; one job per expert the range touches.
struct GateUpProg {
  ExpertTables t;
  const int32_t* ids;
  const uint4* ximg;
  const float* x = nullptr;  // != nullptr: the kernel forms the x registers itself (ximg unused)
  const float* xd = nullptr;  // the token vector, for the terms of wide digit blocks
  float* act;  // [K][I]
  int K, I;
  int rows_per_cta;
  float swiglu_limit;
  unsigned* err;
  bool clamp_gate = true;  // false: the official experts' SwiGLU (up clamped only)

  __device__ __forceinline__ int first_k(int cta) const { return (cta * rows_per_cta) / I; }
  __device__ __forceinline__ int njobs(int cta) const {
    const int a = cta * rows_per_cta;
    const int b = min(K * I, a + rows_per_cta);
    if (a >= b) return 0;
    return (b - 1) / I - a / I + 1;
  }
  __device__ __forceinline__ Job job(int cta, int j) const {
    const int a = cta * rows_per_cta;
    const int b = min(K * I, a + rows_per_cta);
    const int k = a / I + j;
    Job J;
    const int e = checked_expert(ids, k, t.num_experts, err);
    J.src.wa = t.gate[e];
    J.src.wb = t.up[e];
    J.src.sa = t.gate_scale ? t.gate_scale[e] : nullptr;
    J.src.sb = t.up_scale ? t.up_scale[e] : nullptr;
    J.ximg = ximg;
    J.xd = xd;
    J.row_begin = max(a, k * I) - k * I;
    J.row_end = min(b, (k + 1) * I) - k * I;
    return J;
  }
  __device__ __forceinline__ void epilogue(int cta, int j, int row, float va, float vb) const {
    const int k = first_k(cta) + j;
    act[static_cast<size_t>(k) * I + row] = swiglu(va, vb, swiglu_limit, clamp_gate);
  }
  __device__ __forceinline__ void finalize(int, int, int) const {}
};

// down + combine: CTA c owns output rows [c * R, (c + 1) * R); job j is
// selected expert j.  The epilogue thread of a row is the same for every job
// (identical stage split), so out[row] accumulates in selection order exactly
// as the reference does (moe.rs:1319-1321, 650): out = 0; out += w * down.
struct DownProg {
  ExpertTables t;
  const int32_t* ids;
  const float* weights;
  const uint4* ximg;  // K images, img_stride quads apart
  size_t img_stride;
  const float* xf = nullptr;  // float-quad rows: the K activations, xf_stride floats apart
  size_t xf_stride = 0;
  const float* xd = nullptr;  // digit rows: the K activations (wide-block terms), xf_stride floats apart
  float* out;
  int K, O;
  int rows_per_cta;
  unsigned* err;

  __device__ __forceinline__ int njobs(int cta) const { return cta * rows_per_cta < O ? K : 0; }
  __device__ __forceinline__ Job job(int cta, int j) const {
    Job J;
    const int e = checked_expert(ids, j, t.num_experts, err);
    J.src.wa = t.down[e];
    J.src.sa = t.down_scale ? t.down_scale[e] : nullptr;
    J.src.wb = nullptr;
    J.src.sb = nullptr;
    J.ximg = ximg + j * img_stride;
    J.x = xf ? xf + static_cast<size_t>(j) * xf_stride : nullptr;
    J.xd = xd ? xd + static_cast<size_t>(j) * xf_stride : nullptr;
    J.row_begin = cta * rows_per_cta;
    J.row_end = min(O, J.row_begin + rows_per_cta);
    return J;
  }
  __device__ __forceinline__ void epilogue(int, int j, int row, float va, float) const {
    const float p = __fmul_rn(weights[j], va);
    out[row] = __fadd_rn(j == 0 ? 0.0f : out[row], p);
  }
  __device__ __forceinline__ void finalize(int, int, int) const {}
};

// ---- multi-token MoE over (expert, token) pairs.  Pair p runs the expert
// pair_expert[p] on token pair_token[p]; its unweighted down output lands in
// row pair_out[p] of v.  The row programs and layouts are those of the
// single-token launch, so every v row is bit-identical to the value the fused
// single-token combine multiplies by its routing weight.

__device__ __forceinline__ int checked_index(const int32_t* idx, int p, int n, unsigned* err) {
  int v = idx[p];
  if (v < 0 || v >= n) {
    if (err) atomicOr(err, 8u);  // out-of-range token / row index: clamped to 0, flagged
    v = 0;
  }
  return v;
}

// Rows per CTA for `total` rows over the grid: even, in whole 4-row batches.
__device__ __forceinline__ int split_rows(int total) {
  const int g = static_cast<int>(gridDim.x);
  return ((total + g - 1) / g + 3) / 4 * 4;
}

// gate/up: rows [c * R, (c + 1) * R) of the P * I rows of all pairs.
struct GateUpPairsProg {
  ExpertTables t;
  const int32_t* pair_expert;
  const int32_t* pair_token;
  const uint4* ximg;  // T token images, img_stride quads apart
  size_t img_stride;
  const float* xf = nullptr;  // float-quad rows: the T tokens, xf_stride floats apart
  size_t xf_stride = 0;
  const float* xd = nullptr;  // digit rows: the T tokens (wide-block terms), xf_stride floats apart
  float* act;  // [P][I]
  int P, I, T;
  int rows_per_cta;  // 0: derived in the kernel from *count
  const int32_t* count;  // pairs to run (device), nullptr: all P
  float swiglu_limit;
  unsigned* err;

  __device__ __forceinline__ int np() const { return count ? min(max(__ldg(count), 0), P) : P; }
  __device__ __forceinline__ int R() const { return rows_per_cta ? rows_per_cta : split_rows(np() * I); }
  __device__ __forceinline__ int first_p(int cta) const { return (cta * R()) / I; }
  __device__ __forceinline__ int njobs(int cta) const {
    const int a = cta * R();
    const int b = min(np() * I, a + R());
    if (a >= b) return 0;
    return (b - 1) / I - a / I + 1;
  }
  __device__ __forceinline__ Job job(int cta, int j) const {
    const int a = cta * R();
    const int b = min(np() * I, a + R());
    const int p = a / I + j;
    Job J;
    const int e = checked_expert(pair_expert, p, t.num_experts, err);
    const int tok = checked_index(pair_token, p, T, err);
    J.src.wa = t.gate[e];
    J.src.wb = t.up[e];
    J.src.sa = t.gate_scale ? t.gate_scale[e] : nullptr;
    J.src.sb = t.up_scale ? t.up_scale[e] : nullptr;
    J.ximg = ximg + static_cast<size_t>(tok) * img_stride;
    J.x = xf ? xf + static_cast<size_t>(tok) * xf_stride : nullptr;
    J.xd = xd ? xd + static_cast<size_t>(tok) * xf_stride : nullptr;
    J.row_begin = max(a, p * I) - p * I;
    J.row_end = min(b, (p + 1) * I) - p * I;
    return J;
  }
  __device__ __forceinline__ void epilogue(int cta, int j, int row, float va, float vb) const {
    const int p = first_p(cta) + j;
    act[static_cast<size_t>(p) * I + row] = swiglu(va, vb, swiglu_limit);
  }
  __device__ __forceinline__ void finalize(int, int, int) const {}
};

// down: rows [c * R, (c + 1) * R) of the P * O rows of all pairs; no combine.
struct DownPairsProg {
  ExpertTables t;
  const int32_t* pair_expert;
  const int32_t* pair_out;  // nullptr: row p
  const uint4* ximg;        // P activation images, img_stride quads apart
  size_t img_stride;
  const float* xf = nullptr;  // float-quad rows: the P activations, xf_stride floats apart
  size_t xf_stride = 0;
  const float* xd = nullptr;  // digit rows: the P activations (wide-block terms), xf_stride floats apart
  float* v;                 // [v_rows][O]
  int P, O, v_rows;
  int rows_per_cta;         // 0: derived in the kernel from *count
  const int32_t* count;     // pairs to run (device), nullptr: all P
  unsigned* err;

  __device__ __forceinline__ int np() const { return count ? min(max(__ldg(count), 0), P) : P; }
  __device__ __forceinline__ int R() const { return rows_per_cta ? rows_per_cta : split_rows(np() * O); }
  __device__ __forceinline__ int first_p(int cta) const { return (cta * R()) / O; }
  __device__ __forceinline__ int njobs(int cta) const {
    const int a = cta * R();
    const int b = min(np() * O, a + R());
    if (a >= b) return 0;
    return (b - 1) / O - a / O + 1;
  }
  __device__ __forceinline__ Job job(int cta, int j) const {
    const int a = cta * R();
    const int b = min(np() * O, a + R());
    const int p = a / O + j;
    Job J;
    const int e = checked_expert(pair_expert, p, t.num_experts, err);
    J.src.wa = t.down[e];
    J.src.sa = t.down_scale ? t.down_scale[e] : nullptr;
    J.src.wb = nullptr;
    J.src.sb = nullptr;
    J.ximg = ximg + static_cast<size_t>(p) * img_stride;
    J.x = xf ? xf + static_cast<size_t>(p) * xf_stride : nullptr;
    J.xd = xd ? xd + static_cast<size_t>(p) * xf_stride : nullptr;
    J.row_begin = max(a, p * O) - p * O;
    J.row_end = min(b, (p + 1) * O) - p * O;
    return J;
  }
  __device__ __forceinline__ void epilogue(int cta, int j, int row, float va, float) const {
    const int p = first_p(cta) + j;
    const int r = pair_out ? checked_index(pair_out, p, v_rows, err) : p;
    v[static_cast<size_t>(r) * O + row] = va;
  }
  __device__ __forceinline__ void finalize(int, int, int) const {}
};

// Weighted top-k combine of pair outputs, per token in slot order, with the
// arithmetic of the fused single-token combine (out = 0; out += w * down):
// out[t][i] = (((w0 * v[r0][i]) + w1 * v[r1][i]) + ...).  grid (ceil(O/256), T).
static __global__ void __launch_bounds__(256) combine_kernel(const float* __restrict__ v, const int32_t* __restrict__ slot_row,
                                                      const float* __restrict__ w, int K, int O, int v_rows,
                                                      float* __restrict__ out, unsigned* err) {
  const int t = blockIdx.y;
  const int i = blockIdx.x * blockDim.x + threadIdx.x;
  if (i >= O) return;
  float acc = 0.0f;
  for (int j = 0; j < K; ++j) {
    const int r = checked_index(slot_row + static_cast<size_t>(t) * K, j, v_rows, err);
    const float p = __fmul_rn(w[static_cast<size_t>(t) * K + j], v[static_cast<size_t>(r) * O + i]);
    acc = __fadd_rn(j == 0 ? 0.0f : acc, p);
  }
  out[static_cast<size_t>(t) * O + i] = acc;
}

// ---- one dense SwiGLU FFN (the shared expert): gate/up rows with SwiGLU in
// the epilogue, then down rows, optionally added onto out (routed + shared).
struct FfnGateUpProg {
  StageSource src;  // wa = gate, wb = up
  const uint4* ximg;
  const float* x = nullptr;  // != nullptr: the kernel forms the x registers itself (ximg unused)
  float* act;
  int I;
  int rows_per_cta;
  float swiglu_limit;
  unsigned* err;
  __device__ __forceinline__ int njobs(int cta) const { return cta * rows_per_cta < I ? 1 : 0; }
  __device__ __forceinline__ Job job(int cta, int) const {
    Job J;
    J.src = src;
    J.ximg = ximg;
    J.row_begin = cta * rows_per_cta;
    J.row_end = min(I, J.row_begin + rows_per_cta);
    return J;
  }
  __device__ __forceinline__ void epilogue(int, int, int row, float va, float vb) const {
    act[row] = swiglu(va, vb, swiglu_limit);
  }
  __device__ __forceinline__ void finalize(int, int, int) const {}
};

struct FfnDownProg {
  StageSource src;  // wa = down
  const uint4* ximg;
  const float* x = nullptr;  // != nullptr: the kernel forms the x registers itself (ximg unused)
  float* out;
  int O;
  int rows_per_cta;
  int accumulate;
  unsigned* err;
  __device__ __forceinline__ int njobs(int cta) const { return cta * rows_per_cta < O ? 1 : 0; }
  __device__ __forceinline__ Job job(int cta, int) const {
    Job J;
    J.src = src;
    J.ximg = ximg;
    J.row_begin = cta * rows_per_cta;
    J.row_end = min(O, J.row_begin + rows_per_cta);
    return J;
  }
  __device__ __forceinline__ void epilogue(int, int, int row, float va, float) const {
    out[row] = accumulate ? __fadd_rn(out[row], va) : va;
  }
  __device__ __forceinline__ void finalize(int, int, int) const {}
};

// Router (crates/objeta-cuda/src/bin/deepseek_single_layer_moe.rs:720-740):
// max-subtracted softmax, then the first top_k of a stable descending sort
// (ties keep the lower expert index); optional renormalisation of the kept
// weights by their sequential sum.  One CTA; the sequential f32 sum of the
// reference is kept (thread 0 sums in expert order).  exp is evaluated in
// double precision and rounded to f32.
static __global__ void __launch_bounds__(1024) router_topk_kernel(const float* __restrict__ logits, int n, int top_k,
                                                           int renorm, int32_t* __restrict__ ids,
                                                           float* __restrict__ weights) {
  // Launched with programmatic serialization: the next kernel may start its
  // prologue now; this one waits for the preceding grid (which may write the
  // logits, or still read ids / weights) before touching memory.
  asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
  asm volatile("griddepcontrol.wait;" ::: "memory");
  // CTA b routes token b (logits row b, ids / weights row b).
  logits += static_cast<size_t>(blockIdx.x) * n;
  ids += static_cast<size_t>(blockIdx.x) * top_k;
  weights += static_cast<size_t>(blockIdx.x) * top_k;
  extern __shared__ __align__(16) float sp[];  // [n] exp values, then probs
  __shared__ float s_max, s_sum;
  __shared__ float s_wmax[32];
  // the maximum is exact in any order: a block reduction
  float m = -__int_as_float(0x7F800000);
  for (int e = threadIdx.x; e < n; e += blockDim.x) m = fmaxf(m, logits[e]);
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) m = fmaxf(m, __shfl_xor_sync(0xFFFFFFFFu, m, o));
  if ((threadIdx.x & 31) == 0) s_wmax[threadIdx.x >> 5] = m;
  __syncthreads();
  if (threadIdx.x == 0) {
    float mm = s_wmax[0];
    for (int w = 1; w < static_cast<int>((blockDim.x + 31) >> 5); ++w) mm = fmaxf(mm, s_wmax[w]);
    s_max = mm;
  }
  __syncthreads();
  for (int e = threadIdx.x; e < n; e += blockDim.x)
    sp[e] = __double2float_rn(exp(static_cast<double>(__fsub_rn(logits[e], s_max))));
  __syncthreads();
  if (threadIdx.x == 0) {
    // the sum keeps the reference's sequential f32 order; the values come
    // from shared memory four at a time (the adds, not the loads, are the
    // dependent chain)
    float s = 0.0f;
    int e = 0;
    for (; e + 4 <= n; e += 4) {
      const float4 q = *reinterpret_cast<const float4*>(sp + e);
      s = __fadd_rn(s, q.x);
      s = __fadd_rn(s, q.y);
      s = __fadd_rn(s, q.z);
      s = __fadd_rn(s, q.w);
    }
    for (; e < n; ++e) s = __fadd_rn(s, sp[e]);
    s_sum = s;
  }
  __syncthreads();
  for (int e = threadIdx.x; e < n; e += blockDim.x) sp[e] = __fdiv_rn(sp[e], s_sum);
  __syncthreads();
  for (int e = threadIdx.x; e < n; e += blockDim.x) {
    const float pe = sp[e];
    int rank = 0, j = 0;
    for (; j + 4 <= n; j += 4) {  // four probabilities per shared load
      const float4 q = *reinterpret_cast<const float4*>(sp + j);
      rank += (q.x > pe) || (q.x == pe && j < e);
      rank += (q.y > pe) || (q.y == pe && j + 1 < e);
      rank += (q.z > pe) || (q.z == pe && j + 2 < e);
      rank += (q.w > pe) || (q.w == pe && j + 3 < e);
    }
    for (; j < n; ++j) {
      const float pj = sp[j];
      rank += (pj > pe) || (pj == pe && j < e);
    }
    if (rank < top_k) {
      ids[rank] = e;
      weights[rank] = pe;
    }
  }
  if (renorm) {
    __syncthreads();
    if (threadIdx.x == 0) {
      float s = 0.0f;
      for (int k = 0; k < top_k; ++k) s = __fadd_rn(s, weights[k]);
      if (s > 0.0f)
        for (int k = 0; k < top_k; ++k) weights[k] = __fdiv_rn(weights[k], s);
    }
  }
}

// Elementwise kernels of the generic (unaligned-shape) MoE path, same
// arithmetic as silu_mul / weighted_accum (moe.cu:2-34).
static __global__ void silu_mul_kernel(const float* __restrict__ gate, const float* __restrict__ up,
                                float* __restrict__ act, int n, float limit) {
  const int i = blockIdx.x * blockDim.x + threadIdx.x;
  if (i < n) act[i] = swiglu(gate[i], up[i], limit);
}

static __global__ void weighted_accum_kernel(const float* __restrict__ down, float* __restrict__ out,
                                      const float* __restrict__ weights, int k, int n) {
  const int i = blockIdx.x * blockDim.x + threadIdx.x;
  if (i < n) out[i] = __fadd_rn(k == 0 ? 0.0f : out[i], __fmul_rn(weights[k], down[i]));
}

}  // namespace dev
}  // namespace objb
