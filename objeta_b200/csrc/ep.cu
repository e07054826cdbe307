// ep.cu -- the device side of an expert-parallel MoE step with no host round
// trip: the pair list of this rank built from the all-gathered routing table,
// the per-rank partial combine, and the ordered sum of the partials on the
// token owner.  The collectives between them (all-gathers of ids / weights /
// token rows, one all-to-all of partials) are NCCL calls made by the host
// framework.  No counterpart in the reference (it has no expert parallelism).
#include <cuda_runtime.h>

#include <algorithm>

#include <string>

#include "objb_common.h"
#include "objb_launch.h"
#include "objb_host_launch.cuh"

namespace objb {
namespace dev {

// One CTA.  Entries i of ids_all [G*T*K] whose expert lives on `rank`
// (e / epr == rank) become pairs grouped by local expert: a count per local
// expert, an exclusive scan, then a scatter.  Within an expert the order is
// whatever the atomics give; it does not matter, as every pair writes its own
// output row (i) from its own token row (i / K).
//
// Layout: routing entry i = (s*T + t)*K + j sits at ids[s * ids_stride + i %
// (T*K)] (ids_stride = T*K: a plain [G][T][K] table; larger: the packed
// exchange buffer, where each rank's ids follow its token rows), and its
// token row is s * row_stride + t of the token rows (row_stride = T: plain
// [G*T][H] rows).
__device__ __forceinline__ int ep_entry(const int32_t* __restrict__ ids, int i, int TK, size_t ids_stride) {
  return ids[static_cast<size_t>(i / TK) * ids_stride + i % TK];
}

__global__ void __launch_bounds__(1024) ep_build_pairs_kernel(const int32_t* __restrict__ ids_all, int n, int K,
                                                              int TK, size_t ids_stride, int row_stride,
                                                              int num_experts, int epr, int rank,
                                                              int32_t* __restrict__ pair_expert,
                                                              int32_t* __restrict__ pair_token,
                                                              int32_t* __restrict__ pair_out,
                                                              int32_t* __restrict__ num_pairs, unsigned* err) {
  asm volatile("griddepcontrol.wait;" ::: "memory");
  extern __shared__ int bins[];  // [epr]
  __shared__ int warp_sums[32];
  const int tid = threadIdx.x, nt = blockDim.x;
  for (int b = tid; b < epr; b += nt) bins[b] = 0;
  __syncthreads();
  const int lo = rank * epr;
  for (int i = tid; i < n; i += nt) {
    const int e = ep_entry(ids_all, i, TK, ids_stride);
    if (e < 0 || e >= num_experts) {
      if (err) atomicOr(err, 8u);  // out-of-range expert id: dropped, flagged
      continue;
    }
    if (e >= lo && e < lo + epr) atomicAdd(&bins[e - lo], 1);
  }
  __syncthreads();
  // exclusive scan of bins: each thread a contiguous chunk, then a block scan
  const int chunk = (epr + nt - 1) / nt;
  const int b0 = min(epr, tid * chunk), b1 = min(epr, b0 + chunk);
  int local = 0;
  for (int b = b0; b < b1; ++b) local += bins[b];
  const int lane = tid & 31, wid = tid >> 5;
  int incl = local;
#pragma unroll
  for (int o = 1; o < 32; o <<= 1) {
    const int y = __shfl_up_sync(0xFFFFFFFFu, incl, o);
    if (lane >= o) incl += y;
  }
  if (lane == 31) warp_sums[wid] = incl;
  __syncthreads();
  if (wid == 0) {
    const int nw = (nt + 31) >> 5;
    int ws = lane < nw ? warp_sums[lane] : 0;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
      const int y = __shfl_up_sync(0xFFFFFFFFu, ws, o);
      if (lane >= o) ws += y;
    }
    if (lane < nw) warp_sums[lane] = ws;  // inclusive over warps
  }
  __syncthreads();
  int off = incl - local + (wid ? warp_sums[wid - 1] : 0);
  if (tid == nt - 1) *num_pairs = off + local;
  for (int b = b0; b < b1; ++b) {
    const int c = bins[b];
    bins[b] = off;  // becomes the write cursor of expert b
    off += c;
  }
  __syncthreads();
  for (int i = tid; i < n; i += nt) {
    const int e = ep_entry(ids_all, i, TK, ids_stride);
    if (e < lo || e >= lo + epr || e >= num_experts) continue;
    const int pos = atomicAdd(&bins[e - lo], 1);
    pair_expert[pos] = e - lo;
    pair_token[pos] = (i / TK) * row_stride + (i % TK) / K;
    pair_out[pos] = i;
  }
}

// partial[st][c] for routing row st = s*T + t: the slot-order fold of
// w * v over the slots whose expert lives on `rank` (0 when none), with the
// arithmetic of the single-token combine (0 + w0 v0, then + w v).
// (ids and weights in the layout of ep_build_pairs_kernel, one stride.)
__global__ void __launch_bounds__(256) ep_partial_combine_kernel(const int32_t* __restrict__ ids_all,
                                                                 const float* __restrict__ w_all,
                                                                 const float* __restrict__ v, int K, int TK,
                                                                 size_t ids_stride, int epr, int rank, int O,
                                                                 float* __restrict__ partial) {
  asm volatile("griddepcontrol.wait;" ::: "memory");
  const int st = blockIdx.y;
  const int c = blockIdx.x * blockDim.x + threadIdx.x;
  if (c >= O) return;
  const int lo = rank * epr;
  float acc = 0.0f;
  for (int j = 0; j < K; ++j) {
    const int i = st * K + j;
    const size_t at = static_cast<size_t>(i / TK) * ids_stride + i % TK;
    const int e = ids_all[at];
    if (e >= lo && e < lo + epr) acc = __fadd_rn(acc, __fmul_rn(w_all[at], v[static_cast<size_t>(i) * O + c]));
  }
  partial[static_cast<size_t>(st) * O + c] = acc;
}

// The packed exchange buffer of one rank: rows of H floats, the T token rows
// first, then the routing ids (int32 bits) and weights of its T*K entries in
// ceil(2*T*K / H) rows (zero-padded).  One all-gather of these buffers gives
// every rank the token rows, ids and weights of all ranks at once.
__global__ void __launch_bounds__(256) ep_pack_kernel(const float* __restrict__ x, const int32_t* __restrict__ ids,
                                                      const float* __restrict__ w, int T, int TK, int H,
                                                      size_t total, float* __restrict__ send) {
  asm volatile("griddepcontrol.wait;" ::: "memory");
  const size_t nx = static_cast<size_t>(T) * H;
  for (size_t i = blockIdx.x * static_cast<size_t>(blockDim.x) + threadIdx.x; i < total;
       i += static_cast<size_t>(gridDim.x) * blockDim.x) {
    float v = 0.0f;
    if (i < nx) v = x[i];
    else if (i < nx + TK) v = __int_as_float(ids[i - nx]);
    else if (i < nx + 2 * static_cast<size_t>(TK)) v = w[i - nx - TK];
    send[i] = v;
  }
}

// out[t][c] = sum over ranks r, in rank order from 0, of parts[r][t][c].
__global__ void __launch_bounds__(256) ep_sum_partials_kernel(const float* __restrict__ parts, int G, int T, int O,
                                                              float* __restrict__ out) {
  const int t = blockIdx.y;
  const int c = blockIdx.x * blockDim.x + threadIdx.x;
  if (c >= O) return;
  float acc = 0.0f;
  for (int r = 0; r < G; ++r) acc = __fadd_rn(acc, parts[(static_cast<size_t>(r) * T + t) * O + c]);
  out[static_cast<size_t>(t) * O + c] = acc;
}

}  // namespace dev
}  // namespace objb

extern "C" {

int objb_ep_build_pairs_device(const int32_t* d_ids_all, size_t world, size_t tokens, size_t top_k,
                               size_t num_experts, size_t rank, int32_t* d_pair_expert, int32_t* d_pair_token,
                               int32_t* d_pair_out, int32_t* d_num_pairs, objb_stream_t stream) {
  objb::clear_error();
  if (!d_ids_all || !d_pair_expert || !d_pair_token || !d_pair_out || !d_num_pairs)
    return OBJB_FAIL(OBJB_ERR_INVALID_INPUT, "objb_ep_build_pairs_device", "null device pointer");
  if (world == 0 || rank >= world || num_experts == 0 || num_experts % world || top_k == 0 || tokens == 0 ||
      num_experts > 65536 || world * tokens * top_k > (1u << 24))
    return OBJB_FAIL(OBJB_ERR_INVALID_INPUT, "objb_ep_build_pairs_device",
                     "need rank < world, num_experts divisible by world (<= 65536), and world*tokens*top_k <= 2^24");
  int device = 0;
  OBJB_TRY(objb::current_device(&device));
  unsigned* err = nullptr;
  OBJB_TRY(objb::device_error_word(device, &err));
  const int epr = static_cast<int>(num_experts / world);
  const size_t smem = static_cast<size_t>(epr) * sizeof(int);
  if (smem > 48 * 1024)
    OBJB_CUDA(cudaFuncSetAttribute(objb::dev::ep_build_pairs_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                   static_cast<int>(smem)),
              "opt the pair builder into large shared memory");
  objb::dev::ep_build_pairs_kernel<<<1, 1024, smem, static_cast<cudaStream_t>(stream)>>>(
      d_ids_all, static_cast<int>(world * tokens * top_k), static_cast<int>(top_k),
      static_cast<int>(tokens * top_k), tokens * top_k, static_cast<int>(tokens), static_cast<int>(num_experts),
      epr, static_cast<int>(rank), d_pair_expert, d_pair_token, d_pair_out, d_num_pairs, err);
  OBJB_CUDA(cudaGetLastError(), "launch the expert-parallel pair builder");
  return OBJB_OK;
}

int objb_ep_partial_combine_device(const int32_t* d_ids_all, const float* d_w_all, const float* d_v, size_t world,
                                   size_t tokens, size_t top_k, size_t num_experts, size_t rank, size_t out_dim,
                                   float* d_partial, objb_stream_t stream) {
  objb::clear_error();
  if (!d_ids_all || !d_w_all || !d_v || !d_partial)
    return OBJB_FAIL(OBJB_ERR_INVALID_INPUT, "objb_ep_partial_combine_device", "null device pointer");
  if (world == 0 || rank >= world || num_experts == 0 || num_experts % world || top_k == 0 || tokens == 0 ||
      out_dim == 0 || world * tokens > 65535 || out_dim > (1u << 24))
    return OBJB_FAIL(OBJB_ERR_INVALID_INPUT, "objb_ep_partial_combine_device", "shape out of range");
  const dim3 grid(static_cast<unsigned>((out_dim + 255) / 256), static_cast<unsigned>(world * tokens));
  objb::dev::ep_partial_combine_kernel<<<grid, 256, 0, static_cast<cudaStream_t>(stream)>>>(
      d_ids_all, d_w_all, d_v, static_cast<int>(top_k), static_cast<int>(tokens * top_k), tokens * top_k,
      static_cast<int>(num_experts / world), static_cast<int>(rank), static_cast<int>(out_dim), d_partial);
  OBJB_CUDA(cudaGetLastError(), "launch the expert-parallel partial combine");
  return OBJB_OK;
}

size_t objb_ep_packed_rows(size_t tokens, size_t top_k, size_t hidden) {
  if (hidden == 0) return 0;
  return tokens + (2 * tokens * top_k + hidden - 1) / hidden;
}

int objb_ep_pack_device(const float* d_x, const int32_t* d_ids, const float* d_w, size_t tokens, size_t top_k,
                        size_t hidden, float* d_send, objb_stream_t stream) {
  objb::clear_error();
  if (!d_x || !d_ids || !d_w || !d_send)
    return OBJB_FAIL(OBJB_ERR_INVALID_INPUT, "objb_ep_pack_device", "null device pointer");
  if (tokens == 0 || top_k == 0 || hidden == 0 || tokens * top_k > (1u << 24) || tokens * hidden > (1ull << 31))
    return OBJB_FAIL(OBJB_ERR_INVALID_INPUT, "objb_ep_pack_device", "shape out of range");
  const size_t total = objb_ep_packed_rows(tokens, top_k, hidden) * hidden;
  const int grid = static_cast<int>(std::min<size_t>((total + 255) / 256, 1024));
  OBJB_TRY(objb::launch_pdl(objb::dev::ep_pack_kernel, grid, 256, 0, static_cast<cudaStream_t>(stream), d_x, d_ids,
                            d_w, static_cast<int>(tokens), static_cast<int>(tokens * top_k),
                            static_cast<int>(hidden), total, d_send));
  return OBJB_OK;
}

int objb_ep_build_pairs_packed_device(const float* d_recv, size_t world, size_t tokens, size_t top_k,
                                      size_t hidden, size_t num_experts, size_t rank, int32_t* d_pair_expert,
                                      int32_t* d_pair_token, int32_t* d_pair_out, int32_t* d_num_pairs,
                                      objb_stream_t stream) {
  objb::clear_error();
  if (!d_recv || !d_pair_expert || !d_pair_token || !d_pair_out || !d_num_pairs)
    return OBJB_FAIL(OBJB_ERR_INVALID_INPUT, "objb_ep_build_pairs_packed_device", "null device pointer");
  if (world == 0 || rank >= world || num_experts == 0 || num_experts % world || top_k == 0 || tokens == 0 ||
      hidden == 0 || num_experts > 65536 || world * tokens * top_k > (1u << 24) ||
      world * objb_ep_packed_rows(tokens, top_k, hidden) > (1u << 30))
    return OBJB_FAIL(OBJB_ERR_INVALID_INPUT, "objb_ep_build_pairs_packed_device",
                     "need rank < world, num_experts divisible by world (<= 65536), and world*tokens*top_k <= 2^24");
  int device = 0;
  OBJB_TRY(objb::current_device(&device));
  unsigned* err = nullptr;
  OBJB_TRY(objb::device_error_word(device, &err));
  const int epr = static_cast<int>(num_experts / world);
  const size_t smem = static_cast<size_t>(epr) * sizeof(int);
  if (smem > 48 * 1024)
    OBJB_CUDA(cudaFuncSetAttribute(objb::dev::ep_build_pairs_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                   static_cast<int>(smem)),
              "opt the pair builder into large shared memory");
  const size_t rows = objb_ep_packed_rows(tokens, top_k, hidden);
  const int32_t* ids = reinterpret_cast<const int32_t*>(d_recv + tokens * hidden);
  OBJB_TRY(objb::launch_pdl(objb::dev::ep_build_pairs_kernel, 1, 1024, smem, static_cast<cudaStream_t>(stream), ids,
                            static_cast<int>(world * tokens * top_k), static_cast<int>(top_k),
                            static_cast<int>(tokens * top_k), rows * hidden, static_cast<int>(rows),
                            static_cast<int>(num_experts), epr, static_cast<int>(rank), d_pair_expert, d_pair_token,
                            d_pair_out, d_num_pairs, err));
  return OBJB_OK;
}

int objb_ep_partial_combine_packed_device(const float* d_recv, const float* d_v, size_t world, size_t tokens,
                                          size_t top_k, size_t hidden, size_t num_experts, size_t rank,
                                          size_t out_dim, float* d_partial, objb_stream_t stream) {
  objb::clear_error();
  if (!d_recv || !d_v || !d_partial)
    return OBJB_FAIL(OBJB_ERR_INVALID_INPUT, "objb_ep_partial_combine_packed_device", "null device pointer");
  if (world == 0 || rank >= world || num_experts == 0 || num_experts % world || top_k == 0 || tokens == 0 ||
      hidden == 0 || out_dim == 0 || world * tokens > 65535 || out_dim > (1u << 24) ||
      world * tokens * top_k > (1u << 24))
    return OBJB_FAIL(OBJB_ERR_INVALID_INPUT, "objb_ep_partial_combine_packed_device", "shape out of range");
  const size_t rows = objb_ep_packed_rows(tokens, top_k, hidden);
  const float* ids_f = d_recv + tokens * hidden;
  const dim3 grid(static_cast<unsigned>((out_dim + 255) / 256), static_cast<unsigned>(world * tokens));
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = grid;
  cfg.blockDim = dim3(256);
  cfg.stream = static_cast<cudaStream_t>(stream);
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  OBJB_CUDA(cudaLaunchKernelEx(&cfg, objb::dev::ep_partial_combine_kernel, reinterpret_cast<const int32_t*>(ids_f),
                               ids_f + tokens * top_k, d_v, static_cast<int>(top_k),
                               static_cast<int>(tokens * top_k), rows * hidden, static_cast<int>(num_experts / world),
                               static_cast<int>(rank), static_cast<int>(out_dim), d_partial),
            "launch the packed expert-parallel partial combine");
  return OBJB_OK;
}

int objb_ep_sum_partials_device(const float* d_parts, size_t world, size_t tokens, size_t out_dim, float* d_out,
                                objb_stream_t stream) {
  objb::clear_error();
  if (!d_parts || !d_out) return OBJB_FAIL(OBJB_ERR_INVALID_INPUT, "objb_ep_sum_partials_device", "null pointer");
  if (world == 0 || tokens == 0 || tokens > 65535 || out_dim == 0 || out_dim > (1u << 24))
    return OBJB_FAIL(OBJB_ERR_INVALID_INPUT, "objb_ep_sum_partials_device", "shape out of range");
  const dim3 grid(static_cast<unsigned>((out_dim + 255) / 256), static_cast<unsigned>(tokens));
  objb::dev::ep_sum_partials_kernel<<<grid, 256, 0, static_cast<cudaStream_t>(stream)>>>(
      d_parts, static_cast<int>(world), static_cast<int>(tokens), static_cast<int>(out_dim), d_out);
  OBJB_CUDA(cudaGetLastError(), "launch the expert-parallel partial sum");
  return OBJB_OK;
}

}  // extern "C"
