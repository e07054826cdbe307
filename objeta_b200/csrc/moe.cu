// moe.cu -- the selected-expert MoE layer on the device: router, fused
// gate/up + SwiGLU, fused down + weighted combine, and the C ABI for it.
#include <cuda_runtime.h>

#include <algorithm>
#include <cstring>
#include <string>

#include "objb_common.h"
#include "objb_host_launch.cuh"
#include "objb_moe.cuh"
#include "objb_moe_launch.h"
#include "objb_official.cuh"
#include "objb_official_launch.h"

namespace objb {
namespace dev {

// ---- generic path (any shape / alignment): one warp per (selected expert,
// row); blocks read straight from global memory.

// Block dot of the split FP4 layout (weight [rows, cols/2], scale [rows, cols/32]).
__device__ __forceinline__ float split_block_dot_global(const uint8_t* __restrict__ wrow,
                                                        const uint8_t* __restrict__ srow, int b,
                                                        const float* __restrict__ x32) {
  float a = 0.0f;
#pragma unroll
  for (int j = 0; j < 16; ++j) {
    const float2 v = e2m1x2_to_float2(wrow[b * 16 + j]);
    a = fmaf(v.x, __ldg(x32 + 2 * j), a);
    a = fmaf(v.y, __ldg(x32 + 2 * j + 1), a);
  }
  return a * e8m0_to_f32(srow[b]);
}

template <int FMT, bool SPLIT>
__device__ __forceinline__ float row_dot_global(const uint8_t* w, const uint8_t* s, int row, int cols,
                                                const float* x, int lane) {
  const int nb = cols / 32;
  float acc = 0.0f;
  if constexpr (SPLIT) {
    const uint8_t* rw = w + static_cast<size_t>(row) * (cols / 2);
    const uint8_t* rs = s + static_cast<size_t>(row) * nb;
    for (int b = lane; b < nb; b += 32) acc += split_block_dot_global(rw, rs, b, x + b * 32);
  } else {
    constexpr int BB = FMT == OBJB_Q4_0 ? 18 : FMT == OBJB_Q5_0 ? 22 : FMT == OBJB_IQ3_0 ? 14 : 17;
    const uint8_t* rw = w + static_cast<size_t>(row) * nb * BB;
    for (int b = lane; b < nb; b += 32) acc += block_dot_global<FMT>(rw + static_cast<size_t>(b) * BB, x + b * 32);
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) acc += __shfl_xor_sync(0xFFFFFFFFu, acc, o);
  return acc;
}

template <int FMT, bool SPLIT>
__global__ void __launch_bounds__(256) moe_generic_gateup_kernel(ExpertTables t, const int32_t* ids, int K, int I,
                                                                 int H, const float* __restrict__ x,
                                                                 float* __restrict__ act, float limit,
                                                                 unsigned* err) {
  const int wi = blockIdx.x * 8 + (threadIdx.x >> 5);
  if (wi >= K * I) return;
  const int k = wi / I, row = wi % I;
  const int e = checked_expert(ids, k, t.num_experts, err);
  const int lane = threadIdx.x & 31;
  const float g = row_dot_global<FMT, SPLIT>(t.gate[e], SPLIT ? t.gate_scale[e] : nullptr, row, H, x, lane);
  const float u = row_dot_global<FMT, SPLIT>(t.up[e], SPLIT ? t.up_scale[e] : nullptr, row, H, x, lane);
  if (lane == 0) act[static_cast<size_t>(k) * I + row] = swiglu(g, u, limit);
}

template <int FMT, bool SPLIT>
__global__ void __launch_bounds__(256) moe_generic_down_kernel(ExpertTables t, const int32_t* ids,
                                                               const float* __restrict__ weights, int K, int I,
                                                               int O, const float* __restrict__ act,
                                                               float* __restrict__ out, unsigned* err) {
  const int row = blockIdx.x * 8 + (threadIdx.x >> 5);
  if (row >= O) return;
  const int lane = threadIdx.x & 31;
  float acc = 0.0f;
  for (int k = 0; k < K; ++k) {
    const int e = checked_expert(ids, k, t.num_experts, err);
    const float d = row_dot_global<FMT, SPLIT>(t.down[e], SPLIT ? t.down_scale[e] : nullptr, row, I,
                                               act + static_cast<size_t>(k) * I, lane);
    acc = __fadd_rn(acc, __fmul_rn(weights[k], d));
  }
  if (lane == 0) out[row] = acc;
}

// Generic pair kernels: one warp per (pair, row).
template <int FMT, bool SPLIT>
__global__ void __launch_bounds__(256) moe_generic_pairs_gateup_kernel(ExpertTables t, const int32_t* pair_expert,
                                                                       const int32_t* pair_token, int P, int I,
                                                                       int H, int T, const float* __restrict__ x,
                                                                       float* __restrict__ act, float limit,
                                                                       unsigned* err) {
  const int wi = blockIdx.x * 8 + (threadIdx.x >> 5);
  if (wi >= P * I) return;
  const int p = wi / I, row = wi % I;
  const int e = checked_expert(pair_expert, p, t.num_experts, err);
  const float* xp = x + static_cast<size_t>(checked_index(pair_token, p, T, err)) * H;
  const int lane = threadIdx.x & 31;
  const float g = row_dot_global<FMT, SPLIT>(t.gate[e], SPLIT ? t.gate_scale[e] : nullptr, row, H, xp, lane);
  const float u = row_dot_global<FMT, SPLIT>(t.up[e], SPLIT ? t.up_scale[e] : nullptr, row, H, xp, lane);
  if (lane == 0) act[static_cast<size_t>(p) * I + row] = swiglu(g, u, limit);
}

template <int FMT, bool SPLIT>
__global__ void __launch_bounds__(256) moe_generic_pairs_down_kernel(ExpertTables t, const int32_t* pair_expert,
                                                                     const int32_t* pair_out, int P, int I, int O,
                                                                     int v_rows, const float* __restrict__ act,
                                                                     float* __restrict__ v, unsigned* err) {
  const int wi = blockIdx.x * 8 + (threadIdx.x >> 5);
  if (wi >= P * O) return;
  const int p = wi / O, row = wi % O;
  const int e = checked_expert(pair_expert, p, t.num_experts, err);
  const int lane = threadIdx.x & 31;
  const float d = row_dot_global<FMT, SPLIT>(t.down[e], SPLIT ? t.down_scale[e] : nullptr, row, I,
                                             act + static_cast<size_t>(p) * I, lane);
  if (lane == 0) {
    const int r = pair_out ? checked_index(pair_out, p, v_rows, err) : p;
    v[static_cast<size_t>(r) * O + row] = d;
  }
}

}  // namespace dev

namespace {

struct MoeShape {
  int H, I, O, E, K;
};

dev::ExpertTables tables_of(const objb_moe_layer& l) {
  dev::ExpertTables t;
  t.gate = reinterpret_cast<const uint8_t* const*>(l.d_gate);
  t.up = reinterpret_cast<const uint8_t* const*>(l.d_up);
  t.down = reinterpret_cast<const uint8_t* const*>(l.d_down);
  t.gate_scale = reinterpret_cast<const uint8_t* const*>(l.d_gate_scale);
  t.up_scale = reinterpret_cast<const uint8_t* const*>(l.d_up_scale);
  t.down_scale = reinterpret_cast<const uint8_t* const*>(l.d_down_scale);
  t.num_experts = static_cast<int>(l.num_experts);
  return t;
}

// Row byte sizes of one matrix with `cols` columns.
void row_bytes(int fmt, bool split, int cols, int* rb, int* srb) {
  if (split) {
    *rb = cols / 2;
    *srb = cols / 32;
  } else {
    *rb = cols / 32 * block_bytes(fmt);
    *srb = 0;
  }
}

// Row format of the down matrix.  Split FP4 down rows take one block per
// lane: the CTAs of the down launch own few rows per expert (O / SMs), and one
// block per lane puts two warps on each row, so every consumer warp has a
// batch in every stage instead of half of them idling at the stage barrier.
template <class RD>
struct DownRowFormat {
  using type = RD;
  static constexpr int kBlocksPerLane = 2;
};
template <>
struct DownRowFormat<dev::RowDotSplitFp4Digit> {
  using type = dev::RowDotSplitFp4DigitT<1>;
  static constexpr int kBlocksPerLane = 1;
};

template <class RD>
struct MoePlan {
  bool fast = false;
  RowLayoutHost lg, ld;
  size_t act_bytes = 0, imgx_quads = 0, imga_quads = 0;
  size_t scratch_bytes() const {
    return fast ? act_bytes + (imgx_quads + imga_quads) * 16 + 256 : act_bytes;
  }
};

template <class RD>
MoePlan<RD> plan_moe(const MoeShape& s, int fmt, bool split, bool aligned) {
  MoePlan<RD> p;
  p.act_bytes = (static_cast<size_t>(s.K) * s.I * 4 + 255) / 256 * 256;
  int rbh, srbh, rbi, srbi;
  row_bytes(fmt, split, s.H, &rbh, &srbh);
  row_bytes(fmt, split, s.I, &rbi, &srbi);
  const int P = 2, Pd = DownRowFormat<RD>::kBlocksPerLane;
  const bool blocks_ok = split || ((s.H / 32) % P == 0 && (s.I / 32) % P == 0);
  p.fast = aligned && blocks_ok &&
           plan_rows(s.I, s.H, rbh, srbh, P, true, dev::kMaxConsumerWarps, &p.lg, kMoeSmemBudget) &&
           plan_rows(s.O, s.I, rbi, srbi, Pd, false, dev::kMaxConsumerWarps, &p.ld, kMoeSmemBudget);
  if (p.fast) {
    p.imgx_quads = ximage_quads<RD>(p.lg);
    p.imga_quads = ximage_quads<typename DownRowFormat<RD>::type>(p.ld);  // per vector
  }
  return p;
}

template <class RD, int FMT, bool SPLIT>
int run_moe(const objb_moe_layer& l, const MoeShape& s, const int32_t* ids, const float* weights,
            const float* x, float* out, float limit, cudaStream_t stream, void* scratch, size_t scratch_bytes,
            bool aligned, cudaEvent_t mid, unsigned* err_word) {
  int device = 0;
  OBJB_TRY(current_device(&device));
  DeviceProps props;
  OBJB_TRY(device_props(device, &props));
  unsigned* err = err_word;
  if (!err) OBJB_TRY(device_error_word(device, &err));
  MoePlan<RD> p = plan_moe<RD>(s, FMT, SPLIT, aligned);
  const size_t need = p.fast ? p.act_bytes + (p.imgx_quads + p.imga_quads * s.K) * 16 + 256 : p.act_bytes;
  if (scratch_bytes < need)
    return OBJB_FAIL(OBJB_ERR_INVALID_INPUT, "run selected-expert MoE",
                     "scratch of " + std::to_string(scratch_bytes) + " bytes < needed " + std::to_string(need));
  uint8_t* sc = static_cast<uint8_t*>(scratch);
  float* act = reinterpret_cast<float*>(sc);
  const dev::ExpertTables t = tables_of(l);
  if (!p.fast) {
    const int g1 = (s.K * s.I + 7) / 8;
    dev::moe_generic_gateup_kernel<FMT, SPLIT><<<g1, 256, 0, stream>>>(t, ids, s.K, s.I, s.H, x, act, limit, err);
    OBJB_CUDA(cudaGetLastError(), "launch generic gate/up kernel");
    if (mid) OBJB_CUDA(cudaEventRecord(mid, stream), "record gate/up end");
    dev::moe_generic_down_kernel<FMT, SPLIT><<<(s.O + 7) / 8, 256, 0, stream>>>(t, ids, weights, s.K, s.I, s.O, act,
                                                                               out, err);
    OBJB_CUDA(cudaGetLastError(), "launch generic down kernel");
    return OBJB_OK;
  }
  uint4* imgx = reinterpret_cast<uint4*>(sc + p.act_bytes);
  uint4* imga = imgx + p.imgx_quads;
  // gate/up (the kernel forms the x registers itself where that pays)
  const bool x_inline = inline_x_ok<RD>(p.lg, x);
  if (!x_inline) OBJB_TRY(launch_ximage<RD>(p.lg, x, 0, 1, imgx, 0, stream));
  {
    const int total = s.K * s.I;
    const int T = p.lg.tstage;
    int R = (total + props.sm_count - 1) / props.sm_count;
    R = (R + 3) / 4 * 4;  // whole 4-row batches; stages may end short
    const int grid = (total + R - 1) / R;
    dev::GateUpProg prog;
    prog.t = t;
    prog.ids = ids;
    prog.ximg = imgx;
    prog.x = x_inline ? x : nullptr;
    prog.xd = x;
    prog.act = act;
    prog.K = s.K;
    prog.I = s.I;
    prog.rows_per_cta = R;
    prog.swiglu_limit = limit;
    prog.err = err;
    const size_t smem = pipe_smem_bytes(p.lg);
    auto kernel = dev::pipe_kernel<RD, dev::GateUpProg, true>;
    OBJB_TRY(ensure_smem_attr(kernel, device, smem));
    dev::RowLayout dl;
    std::memcpy(&dl, &p.lg, sizeof(dl));
    OBJB_TRY(launch_pdl(kernel, grid, (p.lg.nseg * p.lg.ngrp + 1) * 32, smem, stream, dl, prog));
  }
  if (mid) OBJB_CUDA(cudaEventRecord(mid, stream), "record gate/up end");
  // down + combine (float-quad rows read the activations directly)
  using RDd = typename DownRowFormat<RD>::type;
  const bool act_direct = direct_x_ok<RDd>(act, static_cast<size_t>(s.I));
  if (!act_direct) OBJB_TRY(launch_ximage<RDd>(p.ld, act, static_cast<size_t>(s.I), s.K, imga, p.imga_quads, stream));
  {
    const int T = p.ld.tstage;
    int R = (s.O + props.sm_count - 1) / props.sm_count;
    R = (R + 3) / 4 * 4;  // whole 4-row batches; stages may end short
    const int grid = (s.O + R - 1) / R;
    dev::DownProg prog;
    prog.t = t;
    prog.ids = ids;
    prog.weights = weights;
    prog.ximg = imga;
    prog.img_stride = p.imga_quads;
    prog.xf = act_direct ? act : nullptr;
    prog.xf_stride = static_cast<size_t>(s.I);
    prog.xd = act;
    prog.out = out;
    prog.K = s.K;
    prog.O = s.O;
    prog.rows_per_cta = R;
    prog.err = err;
    const size_t smem = pipe_smem_bytes(p.ld);
    auto kernel = dev::pipe_kernel<RDd, dev::DownProg, false>;
    OBJB_TRY(ensure_smem_attr(kernel, device, smem));
    dev::RowLayout dl;
    std::memcpy(&dl, &p.ld, sizeof(dl));
    OBJB_TRY(launch_pdl(kernel, grid, (p.ld.nseg * p.ld.ngrp + 1) * 32, smem, stream, dl, prog));
  }
  return OBJB_OK;
}

// Pairs: s.K is the pair count P; T token vectors of H floats.
template <class RD>
size_t pairs_need(const MoePlan<RD>& p, const MoeShape& s, int T) {
  return p.fast ? p.act_bytes + (p.imgx_quads * T + p.imga_quads * s.K) * 16 + 256 : p.act_bytes;
}

template <class RD, int FMT, bool SPLIT>
int run_pairs(const objb_moe_layer& l, const MoeShape& s, int T, const int32_t* pair_expert,
              const int32_t* pair_token, const int32_t* pair_out, const int32_t* d_count, const float* x, float* v,
              int v_rows, float limit, cudaStream_t stream, void* scratch, size_t scratch_bytes, bool aligned,
              unsigned* err_word) {
  int device = 0;
  OBJB_TRY(current_device(&device));
  DeviceProps props;
  OBJB_TRY(device_props(device, &props));
  unsigned* err = err_word;
  if (!err) OBJB_TRY(device_error_word(device, &err));
  MoePlan<RD> p = plan_moe<RD>(s, FMT, SPLIT, aligned);
  const size_t need = pairs_need(p, s, T);
  if (scratch_bytes < need)
    return OBJB_FAIL(OBJB_ERR_INVALID_INPUT, "run multi-token MoE pairs",
                     "scratch of " + std::to_string(scratch_bytes) + " bytes < needed " + std::to_string(need));
  uint8_t* sc = static_cast<uint8_t*>(scratch);
  float* act = reinterpret_cast<float*>(sc);
  const dev::ExpertTables t = tables_of(l);
  const int P = s.K;
  if (!p.fast) {
    if (d_count)
      return OBJB_FAIL(OBJB_ERR_UNSUPPORTED, "run multi-token MoE pairs",
                       "a device-side pair count needs 16-byte aligned experts and aligned shapes");
    dev::moe_generic_pairs_gateup_kernel<FMT, SPLIT><<<(P * s.I + 7) / 8, 256, 0, stream>>>(
        t, pair_expert, pair_token, P, s.I, s.H, T, x, act, limit, err);
    OBJB_CUDA(cudaGetLastError(), "launch generic pair gate/up kernel");
    dev::moe_generic_pairs_down_kernel<FMT, SPLIT><<<(P * s.O + 7) / 8, 256, 0, stream>>>(
        t, pair_expert, pair_out, P, s.I, s.O, v_rows, act, v, err);
    OBJB_CUDA(cudaGetLastError(), "launch generic pair down kernel");
    return OBJB_OK;
  }
  uint4* imgx = reinterpret_cast<uint4*>(sc + p.act_bytes);
  uint4* imga = imgx + p.imgx_quads * T;
  // float-quad rows read the token and activation rows directly
  const bool x_direct = direct_x_ok<RD>(x, static_cast<size_t>(s.H));
  using RDd = typename DownRowFormat<RD>::type;
  const bool act_direct = direct_x_ok<RDd>(act, static_cast<size_t>(s.I));
  if (!x_direct) OBJB_TRY(launch_ximage<RD>(p.lg, x, static_cast<size_t>(s.H), T, imgx, p.imgx_quads, stream));
  {
    const int total = P * s.I;
    int R = (total + props.sm_count - 1) / props.sm_count;
    R = (R + 3) / 4 * 4;  // whole 4-row batches; stages may end short
    // with a device-side count the split is made in the kernel over all SMs
    const int grid = d_count ? props.sm_count : (total + R - 1) / R;
    dev::GateUpPairsProg prog;
    prog.t = t;
    prog.pair_expert = pair_expert;
    prog.pair_token = pair_token;
    prog.ximg = imgx;
    prog.img_stride = p.imgx_quads;
    prog.xf = x_direct ? x : nullptr;
    prog.xf_stride = static_cast<size_t>(s.H);
    prog.xd = x;
    prog.act = act;
    prog.P = P;
    prog.I = s.I;
    prog.T = T;
    prog.rows_per_cta = d_count ? 0 : R;
    prog.count = d_count;
    prog.swiglu_limit = limit;
    prog.err = err;
    const size_t smem = pipe_smem_bytes(p.lg);
    auto kernel = dev::pipe_kernel<RD, dev::GateUpPairsProg, true>;
    OBJB_TRY(ensure_smem_attr(kernel, device, smem));
    dev::RowLayout dl;
    std::memcpy(&dl, &p.lg, sizeof(dl));
    OBJB_TRY(launch_pdl(kernel, grid, (p.lg.nseg * p.lg.ngrp + 1) * 32, smem, stream, dl, prog));
  }
  if (!act_direct)
    OBJB_TRY(launch_ximage<RDd>(p.ld, act, static_cast<size_t>(s.I), P, imga, p.imga_quads, stream, d_count));
  {
    const int total = P * s.O;
    int R = (total + props.sm_count - 1) / props.sm_count;
    R = (R + 3) / 4 * 4;  // whole 4-row batches; stages may end short
    const int grid = d_count ? props.sm_count : (total + R - 1) / R;
    dev::DownPairsProg prog;
    prog.t = t;
    prog.pair_expert = pair_expert;
    prog.pair_out = pair_out;
    prog.ximg = imga;
    prog.img_stride = p.imga_quads;
    prog.xf = act_direct ? act : nullptr;
    prog.xf_stride = static_cast<size_t>(s.I);
    prog.xd = act;
    prog.v = v;
    prog.P = P;
    prog.O = s.O;
    prog.v_rows = v_rows;
    prog.rows_per_cta = d_count ? 0 : R;
    prog.count = d_count;
    prog.err = err;
    const size_t smem = pipe_smem_bytes(p.ld);
    auto kernel = dev::pipe_kernel<RDd, dev::DownPairsProg, false>;
    OBJB_TRY(ensure_smem_attr(kernel, device, smem));
    dev::RowLayout dl;
    std::memcpy(&dl, &p.ld, sizeof(dl));
    OBJB_TRY(launch_pdl(kernel, grid, (p.ld.nseg * p.ld.ngrp + 1) * 32, smem, stream, dl, prog));
  }
  return OBJB_OK;
}

int validate_layer(const objb_moe_layer* l, size_t top_k, MoeShape* s, bool* split) {
  if (!l) return OBJB_FAIL(OBJB_ERR_INVALID_INPUT, "validate MoE layer", "null layer descriptor");
  if (!valid_format(l->fmt))
    return OBJB_FAIL(OBJB_ERR_INVALID_INPUT, "validate MoE layer", "unknown QuantFormat ordinal " + std::to_string(l->fmt));
  if (l->hidden % 32 || l->intermediate % 32)
    return OBJB_FAIL(OBJB_ERR_INVALID_INPUT, "validate MoE layer",
                     "hidden " + std::to_string(l->hidden) + " and intermediate " + std::to_string(l->intermediate) +
                         " must be multiples of block_size 32");
  if (!l->d_gate || !l->d_up || !l->d_down)
    return OBJB_FAIL(OBJB_ERR_INVALID_INPUT, "validate MoE layer", "null expert pointer table");
  *split = l->fmt == OBJB_FP4_E2M1 && l->d_gate_scale && l->d_up_scale && l->d_down_scale;
  if (l->fmt == OBJB_FP4_E2M1 && !*split && (l->d_gate_scale || l->d_up_scale || l->d_down_scale))
    return OBJB_FAIL(OBJB_ERR_INVALID_INPUT, "validate MoE layer", "split FP4 needs all three scale tables");
  if (top_k == 0 || top_k > 1024)
    return OBJB_FAIL(OBJB_ERR_INVALID_INPUT, "validate MoE layer", "top_k must be in 1..1024");
  if (l->num_experts == 0 || l->num_experts > (1u << 20))
    return OBJB_FAIL(OBJB_ERR_INVALID_INPUT, "validate MoE layer", "num_experts must be in 1..2^20");
  if (l->hidden > (1u << 20) || l->intermediate > (1u << 20) || l->out_dim > (1u << 24) || l->out_dim == 0)
    return OBJB_FAIL(OBJB_ERR_INVALID_INPUT, "validate MoE layer", "shape exceeds the supported range");
  if (static_cast<size_t>(top_k) * l->intermediate > (1u << 30))
    return OBJB_FAIL(OBJB_ERR_INVALID_INPUT, "validate MoE layer", "top_k * intermediate too large");
  s->H = static_cast<int>(l->hidden);
  s->I = static_cast<int>(l->intermediate);
  s->O = static_cast<int>(l->out_dim);
  s->E = static_cast<int>(l->num_experts);
  s->K = static_cast<int>(top_k);
  return OBJB_OK;
}

}  // namespace

int moe_scratch_bytes(const objb_moe_layer* l, size_t top_k, size_t* out) {
  MoeShape s;
  bool split = false;
  OBJB_TRY(validate_layer(l, top_k, &s, &split));
  size_t need = 0;
  auto calc = [&](auto tag) {
    using RD = decltype(tag);
    // planned as moe_selected plans it: an unaligned layer runs the generic
    // path, which needs only the activations
    MoePlan<RD> p = plan_moe<RD>(s, l->fmt, split, (l->flags & OBJB_MOE_UNALIGNED) == 0);
    need = p.fast ? p.act_bytes + (p.imgx_quads + p.imga_quads * s.K) * 16 + 256 : p.act_bytes;
  };
  if (split) calc(dev::RowDotSplitFp4Digit{});
  else if (l->fmt == OBJB_Q4_0) calc(dev::RowDot<OBJB_Q4_0>{});
  else if (l->fmt == OBJB_Q5_0) calc(dev::RowDot<OBJB_Q5_0>{});
  else if (l->fmt == OBJB_IQ3_0) calc(dev::RowDot<OBJB_IQ3_0>{});
  else calc(dev::RowDot<OBJB_FP4_E2M1>{});
  *out = need;
  return OBJB_OK;
}

// Alignment of every expert pointer is not visible to the host (the tables
// live in device memory); the caller states it.  Unaligned layers run the
// generic path.
int moe_selected(const objb_moe_layer* l, const int32_t* ids, const float* weights, size_t top_k,
                 const float* x, float* out, float limit, cudaStream_t stream, void* scratch,
                 size_t scratch_bytes, cudaEvent_t mid, unsigned* err_word) {
  MoeShape s;
  bool split = false;
  OBJB_TRY(validate_layer(l, top_k, &s, &split));
  if (!ids || !weights || !x || !out)
    return OBJB_FAIL(OBJB_ERR_INVALID_INPUT, "run selected-expert MoE", "null device pointer");
  const bool aligned = (l->flags & OBJB_MOE_UNALIGNED) == 0;
  if (split)
    return run_moe<dev::RowDotSplitFp4Digit, OBJB_FP4_E2M1, true>(*l, s, ids, weights, x, out, limit, stream, scratch,
                                                              scratch_bytes, aligned, mid, err_word);
  switch (l->fmt) {
    case OBJB_Q4_0:
      return run_moe<dev::RowDot<OBJB_Q4_0>, OBJB_Q4_0, false>(*l, s, ids, weights, x, out, limit, stream, scratch,
                                                                scratch_bytes, aligned, mid, err_word);
    case OBJB_Q5_0:
      return run_moe<dev::RowDot<OBJB_Q5_0>, OBJB_Q5_0, false>(*l, s, ids, weights, x, out, limit, stream, scratch,
                                                                scratch_bytes, aligned, mid, err_word);
    case OBJB_IQ3_0:
      return run_moe<dev::RowDot<OBJB_IQ3_0>, OBJB_IQ3_0, false>(*l, s, ids, weights, x, out, limit, stream,
                                                                  scratch, scratch_bytes, aligned, mid, err_word);
    default:
      return run_moe<dev::RowDot<OBJB_FP4_E2M1>, OBJB_FP4_E2M1, false>(*l, s, ids, weights, x, out, limit, stream,
                                                                        scratch, scratch_bytes, aligned, mid, err_word);
  }
}

namespace {

int validate_pairs(const objb_moe_layer* l, size_t num_pairs, size_t num_tokens, MoeShape* s, bool* split) {
  OBJB_TRY(validate_layer(l, 1, s, split));
  if (num_pairs == 0 || num_pairs > (1u << 20) || num_tokens == 0 || num_tokens > (1u << 20))
    return OBJB_FAIL(OBJB_ERR_INVALID_INPUT, "validate MoE pairs",
                     "need 1 <= num_pairs, num_tokens <= 2^20 (got " + std::to_string(num_pairs) + ", " +
                         std::to_string(num_tokens) + ")");
  if (num_pairs * std::max(l->intermediate, l->out_dim) > (1u << 30) || num_tokens * l->hidden > (1ull << 34))
    return OBJB_FAIL(OBJB_ERR_INVALID_INPUT, "validate MoE pairs", "num_pairs * rows too large");
  s->K = static_cast<int>(num_pairs);
  return OBJB_OK;
}

}  // namespace

int moe_pairs_scratch_bytes(const objb_moe_layer* l, size_t num_pairs, size_t num_tokens, size_t* out) {
  MoeShape s;
  bool split = false;
  OBJB_TRY(validate_pairs(l, num_pairs, num_tokens, &s, &split));
  const int T = static_cast<int>(num_tokens);
  auto calc = [&](auto tag) {
    using RD = decltype(tag);
    *out = pairs_need(plan_moe<RD>(s, l->fmt, split, true), s, T);
  };
  if (split) calc(dev::RowDotSplitFp4Digit{});
  else if (l->fmt == OBJB_Q4_0) calc(dev::RowDot<OBJB_Q4_0>{});
  else if (l->fmt == OBJB_Q5_0) calc(dev::RowDot<OBJB_Q5_0>{});
  else if (l->fmt == OBJB_IQ3_0) calc(dev::RowDot<OBJB_IQ3_0>{});
  else calc(dev::RowDot<OBJB_FP4_E2M1>{});
  return OBJB_OK;
}

int moe_pairs(const objb_moe_layer* l, size_t num_pairs, const int32_t* pair_expert, const int32_t* pair_token,
              const int32_t* pair_out, size_t num_tokens, const float* x, float* v, size_t v_rows, float limit,
              cudaStream_t stream, void* scratch, size_t scratch_bytes, unsigned* err_word,
              const int32_t* d_num_pairs) {
  MoeShape s;
  bool split = false;
  OBJB_TRY(validate_pairs(l, num_pairs, num_tokens, &s, &split));
  if (!pair_expert || !pair_token || !x || !v)
    return OBJB_FAIL(OBJB_ERR_INVALID_INPUT, "run multi-token MoE pairs", "null device pointer");
  if (v_rows < (pair_out ? 1 : num_pairs) || v_rows > (1u << 30))
    return OBJB_FAIL(OBJB_ERR_INVALID_INPUT, "run multi-token MoE pairs",
                     "v_rows " + std::to_string(v_rows) + " cannot hold the pair outputs");
  const bool aligned = (l->flags & OBJB_MOE_UNALIGNED) == 0;
  const int T = static_cast<int>(num_tokens);
  const int VR = static_cast<int>(v_rows);
#define OBJB_PAIRS(RDT, F, SP)                                                                                   \
  return run_pairs<RDT, F, SP>(*l, s, T, pair_expert, pair_token, pair_out, d_num_pairs, x, v, VR, limit, stream, \
                               scratch, scratch_bytes, aligned, err_word)
  if (split) OBJB_PAIRS(dev::RowDotSplitFp4Digit, OBJB_FP4_E2M1, true);
  switch (l->fmt) {
    case OBJB_Q4_0: OBJB_PAIRS(dev::RowDot<OBJB_Q4_0>, OBJB_Q4_0, false);
    case OBJB_Q5_0: OBJB_PAIRS(dev::RowDot<OBJB_Q5_0>, OBJB_Q5_0, false);
    case OBJB_IQ3_0: OBJB_PAIRS(dev::RowDot<OBJB_IQ3_0>, OBJB_IQ3_0, false);
    default: OBJB_PAIRS(dev::RowDot<OBJB_FP4_E2M1>, OBJB_FP4_E2M1, false);
  }
#undef OBJB_PAIRS
}

int moe_combine(const float* v, size_t v_rows, const int32_t* slot_row, const float* weights, size_t num_tokens,
                size_t top_k, size_t out_dim, float* out, cudaStream_t stream, unsigned* err_word) {
  if (!v || !slot_row || !weights || !out)
    return OBJB_FAIL(OBJB_ERR_INVALID_INPUT, "objb_moe_combine_device", "null device pointer");
  if (num_tokens == 0 || num_tokens > 65535 || top_k == 0 || top_k > 1024 || out_dim == 0 ||
      out_dim > (1u << 24) || v_rows == 0 || v_rows > (1u << 30))
    return OBJB_FAIL(OBJB_ERR_INVALID_INPUT, "objb_moe_combine_device",
                     "need 1 <= num_tokens <= 65535, 1 <= top_k <= 1024, 1 <= out_dim <= 2^24");
  unsigned* err = err_word;
  if (!err) {
    int device = 0;
    OBJB_TRY(current_device(&device));
    OBJB_TRY(device_error_word(device, &err));
  }
  const dim3 grid(static_cast<unsigned>((out_dim + 255) / 256), static_cast<unsigned>(num_tokens));
  dev::combine_kernel<<<grid, 256, 0, stream>>>(v, slot_row, weights, static_cast<int>(top_k),
                                                 static_cast<int>(out_dim), static_cast<int>(v_rows), out, err);
  OBJB_CUDA(cudaGetLastError(), "launch combine kernel");
  return OBJB_OK;
}

int router_topk_batched(const float* logits, size_t num_tokens, size_t n, size_t top_k, int renorm, int32_t* ids,
                        float* weights, cudaStream_t stream) {
  if (!logits || !ids || !weights)
    return OBJB_FAIL(OBJB_ERR_INVALID_INPUT, "objb_router_topk_batched_device", "null device pointer");
  if (num_tokens == 0 || num_tokens > 65535 || n == 0 || n > 8192 || top_k == 0 || top_k > n)
    return OBJB_FAIL(OBJB_ERR_INVALID_INPUT, "objb_router_topk_batched_device",
                     "need 1 <= num_tokens <= 65535 and 1 <= top_k <= num_experts <= 8192 (got top_k " +
                         std::to_string(top_k) + ", num_experts " + std::to_string(n) + ")");
  const int threads = static_cast<int>(std::min<size_t>(1024, (n + 31) / 32 * 32));
  return launch_pdl(dev::router_topk_kernel, static_cast<int>(num_tokens), threads, n * sizeof(float), stream, logits,
                    static_cast<int>(n), static_cast<int>(top_k), renorm, ids, weights);
}

// ---- official DeepSeek routed experts (execute_selected_moe_official_routed_fp4_cuda,
// moe.rs:1393-1548): act_quant(x) -> FP8 x FP4 gate/up with SwiGLU -> act_quant(act)
// -> FP8 x FP4 down with the weighted combine.  Split-FP4 layers only.
namespace {

struct OfficialPlan {
  RowLayoutHost lg, ld;
  size_t codes_x = 0, scales_x = 0, act = 0, codes_a = 0, scales_a = 0, imgx = 0, imga = 0, total = 0;
};

int plan_official(const MoeShape& s, OfficialPlan* p) {
  if (s.H % 512 || s.I % 512)
    return OBJB_FAIL(OBJB_ERR_UNSUPPORTED, "plan official MoE", "hidden and intermediate must be multiples of 512");
  if (!plan_fp8_fp4(s.I, s.H, true, &p->lg) || !plan_fp8_fp4(s.O, s.I, false, &p->ld))
    return OBJB_FAIL(OBJB_ERR_UNSUPPORTED, "plan official MoE", "shape does not fit the row pipeline");
  auto r256 = [](size_t b) { return (b + 255) / 256 * 256; };
  p->codes_x = r256(s.H);
  p->scales_x = r256(s.H / 128);
  p->act = r256(static_cast<size_t>(s.K) * s.I * 4);
  p->codes_a = r256(static_cast<size_t>(s.K) * s.I);
  p->scales_a = r256(static_cast<size_t>(s.K) * s.I / 128);
  p->imgx = fp8_image_quads(p->lg) * 16;
  p->imga = fp8_image_quads(p->ld) * 16 * s.K;
  p->total = p->codes_x + p->scales_x + p->act + p->codes_a + p->scales_a + p->imgx + p->imga + 256;
  return OBJB_OK;
}

}  // namespace

int moe_official_scratch_bytes(const objb_moe_layer* l, size_t top_k, size_t* out) {
  MoeShape s;
  bool split = false;
  OBJB_TRY(validate_layer(l, top_k, &s, &split));
  if (!split) return OBJB_FAIL(OBJB_ERR_INVALID_INPUT, "plan official MoE", "needs a split FP4 layer (scale tables)");
  OfficialPlan p;
  OBJB_TRY(plan_official(s, &p));
  *out = p.total;
  return OBJB_OK;
}

int moe_official_selected(const objb_moe_layer* l, const int32_t* ids, const float* weights, size_t top_k,
                          const float* x, float* out, float limit, cudaStream_t stream, void* scratch,
                          size_t scratch_bytes, cudaEvent_t mid, unsigned* err_word) {
  MoeShape s;
  bool split = false;
  OBJB_TRY(validate_layer(l, top_k, &s, &split));
  if (!split) return OBJB_FAIL(OBJB_ERR_INVALID_INPUT, "run official MoE", "needs a split FP4 layer (scale tables)");
  if (!ids || !weights || !x || !out) return OBJB_FAIL(OBJB_ERR_INVALID_INPUT, "run official MoE", "null device pointer");
  if (l->flags & OBJB_MOE_UNALIGNED)
    return OBJB_FAIL(OBJB_ERR_UNSUPPORTED, "run official MoE", "expert tensors must be 16-byte aligned");
  OfficialPlan p;
  OBJB_TRY(plan_official(s, &p));
  if (scratch_bytes < p.total)
    return OBJB_FAIL(OBJB_ERR_INVALID_INPUT, "run official MoE",
                     "scratch of " + std::to_string(scratch_bytes) + " bytes < needed " + std::to_string(p.total));
  int device = 0;
  OBJB_TRY(current_device(&device));
  DeviceProps props;
  OBJB_TRY(device_props(device, &props));
  unsigned* err = err_word;
  if (!err) OBJB_TRY(device_error_word(device, &err));
  uint8_t* sc = static_cast<uint8_t*>(scratch);
  uint8_t* codes_x = sc;
  uint8_t* scales_x = codes_x + p.codes_x;
  float* act = reinterpret_cast<float*>(scales_x + p.scales_x);
  uint8_t* codes_a = reinterpret_cast<uint8_t*>(act) + p.act;
  uint8_t* scales_a = codes_a + p.codes_a;
  uint4* imgx = reinterpret_cast<uint4*>(scales_a + p.scales_a);
  uint4* imga = reinterpret_cast<uint4*>(reinterpret_cast<uint8_t*>(imgx) + p.imgx);
  const dev::ExpertTables t = tables_of(*l);
  OBJB_TRY(act_quant(x, 1, s.H, codes_x, scales_x, stream, "act_quant hidden"));
  OBJB_TRY(launch_ximage_fp8(p.lg, codes_x, scales_x, 1, imgx, 0, stream));
  {
    const int total = s.K * s.I;
    int R = (total + props.sm_count - 1) / props.sm_count;
    R = (R + 3) / 4 * 4;
    dev::GateUpProg prog;
    prog.t = t;
    prog.ids = ids;
    prog.ximg = imgx;
    prog.act = act;
    prog.K = s.K;
    prog.I = s.I;
    prog.rows_per_cta = R;
    prog.swiglu_limit = limit;
    prog.err = err;
    prog.clamp_gate = false;
    const size_t smem = pipe_smem_bytes(p.lg);
    auto kernel = dev::pipe_kernel<dev::RowDotFp8Fp4, dev::GateUpProg, true>;
    OBJB_TRY(ensure_smem_attr(kernel, device, smem));
    dev::RowLayout dl;
    std::memcpy(&dl, &p.lg, sizeof(dl));
    OBJB_TRY(launch_pdl(kernel, (total + R - 1) / R, (p.lg.nseg * p.lg.ngrp + 1) * 32, smem, stream, dl, prog));
  }
  if (mid) OBJB_CUDA(cudaEventRecord(mid, stream), "record gate/up end");
  OBJB_TRY(act_quant(act, s.K, s.I, codes_a, scales_a, stream, "act_quant intermediate"));
  const size_t qa = fp8_image_quads(p.ld);
  OBJB_TRY(launch_ximage_fp8(p.ld, codes_a, scales_a, s.K, imga, qa, stream));
  {
    int R = (s.O + props.sm_count - 1) / props.sm_count;
    R = (R + 3) / 4 * 4;
    dev::DownProg prog;
    prog.t = t;
    prog.ids = ids;
    prog.weights = weights;
    prog.ximg = imga;
    prog.img_stride = qa;
    prog.out = out;
    prog.K = s.K;
    prog.O = s.O;
    prog.rows_per_cta = R;
    prog.err = err;
    const size_t smem = pipe_smem_bytes(p.ld);
    auto kernel = dev::pipe_kernel<dev::RowDotFp8Fp4, dev::DownProg, false>;
    OBJB_TRY(ensure_smem_attr(kernel, device, smem));
    dev::RowLayout dl;
    std::memcpy(&dl, &p.ld, sizeof(dl));
    OBJB_TRY(launch_pdl(kernel, (s.O + R - 1) / R, (p.ld.nseg * p.ld.ngrp + 1) * 32, smem, stream, dl, prog));
  }
  return OBJB_OK;
}

int router_topk(const float* logits, size_t n, size_t top_k, int renorm, int32_t* ids, float* weights,
                cudaStream_t stream) {
  if (!logits || !ids || !weights)
    return OBJB_FAIL(OBJB_ERR_INVALID_INPUT, "objb_router_topk_device", "null device pointer");
  if (n == 0 || n > 8192 || top_k == 0 || top_k > n)
    return OBJB_FAIL(OBJB_ERR_INVALID_INPUT, "objb_router_topk_device",
                     "need 1 <= top_k <= num_experts <= 8192 (got top_k " + std::to_string(top_k) +
                         ", num_experts " + std::to_string(n) + ")");
  const int threads = static_cast<int>(std::min<size_t>(1024, (n + 31) / 32 * 32));
  return launch_pdl(dev::router_topk_kernel, 1, threads, n * sizeof(float), stream, logits, static_cast<int>(n),
                    static_cast<int>(top_k), renorm, ids, weights);
}

}  // namespace objb

extern "C" {

int objb_moe_scratch_bytes(const objb_moe_layer* layer, size_t top_k, size_t* bytes) {
  objb::clear_error();
  if (!bytes) return OBJB_FAIL(OBJB_ERR_INVALID_INPUT, "objb_moe_scratch_bytes", "null output pointer");
  return objb::moe_scratch_bytes(layer, top_k, bytes);
}

int objb_router_topk_device(const float* d_logits, size_t num_experts, size_t top_k, int renormalize,
                            int32_t* d_ids, float* d_weights, objb_stream_t stream) {
  objb::clear_error();
  return objb::router_topk(d_logits, num_experts, top_k, renormalize, d_ids, d_weights,
                           static_cast<cudaStream_t>(stream));
}

int objb_moe_selected_device(const objb_moe_layer* layer, const int32_t* d_ids, const float* d_weights,
                             size_t top_k, const float* d_x, float* d_out, float swiglu_limit,
                             objb_stream_t stream_) {
  objb::clear_error();
  cudaStream_t stream = static_cast<cudaStream_t>(stream_);
  size_t need = 0;
  OBJB_TRY(objb::moe_scratch_bytes(layer, top_k, &need));
  int device = 0;
  OBJB_TRY(objb::current_device(&device));
  void* ws = nullptr;
  OBJB_TRY(objb::workspace_get(device, stream, need, &ws));
  return objb::moe_selected(layer, d_ids, d_weights, top_k, d_x, d_out, swiglu_limit, stream, ws, need, nullptr);
}

int objb_moe_forward_device(const objb_moe_layer* layer, const float* d_logits, size_t top_k, int renormalize,
                            int32_t* d_ids, float* d_weights, const float* d_x, float* d_out, float swiglu_limit,
                            objb_stream_t stream) {
  objb::clear_error();
  if (!layer) return OBJB_FAIL(OBJB_ERR_INVALID_INPUT, "objb_moe_forward_device", "null layer descriptor");
  OBJB_TRY(objb::router_topk(d_logits, layer->num_experts, top_k, renormalize, d_ids, d_weights,
                             static_cast<cudaStream_t>(stream)));
  return objb_moe_selected_device(layer, d_ids, d_weights, top_k, d_x, d_out, swiglu_limit, stream);
}

int objb_moe_pairs_scratch_bytes(const objb_moe_layer* layer, size_t num_pairs, size_t num_tokens, size_t* bytes) {
  objb::clear_error();
  if (!bytes) return OBJB_FAIL(OBJB_ERR_INVALID_INPUT, "objb_moe_pairs_scratch_bytes", "null output pointer");
  return objb::moe_pairs_scratch_bytes(layer, num_pairs, num_tokens, bytes);
}

int objb_moe_pairs_device(const objb_moe_layer* layer, size_t num_pairs, const int32_t* d_num_pairs,
                          const int32_t* d_pair_expert, const int32_t* d_pair_token, const int32_t* d_pair_out,
                          size_t num_tokens, const float* d_x, float* d_v, size_t v_rows, float swiglu_limit,
                          objb_stream_t stream_) {
  objb::clear_error();
  cudaStream_t stream = static_cast<cudaStream_t>(stream_);
  size_t need = 0;
  OBJB_TRY(objb::moe_pairs_scratch_bytes(layer, num_pairs, num_tokens, &need));
  int device = 0;
  OBJB_TRY(objb::current_device(&device));
  void* ws = nullptr;
  OBJB_TRY(objb::workspace_get(device, stream, need, &ws));
  return objb::moe_pairs(layer, num_pairs, d_pair_expert, d_pair_token, d_pair_out, num_tokens, d_x, d_v, v_rows,
                         swiglu_limit, stream, ws, need, nullptr, d_num_pairs);
}

int objb_moe_combine_device(const float* d_v, size_t v_rows, const int32_t* d_slot_row, const float* d_weights,
                            size_t num_tokens, size_t top_k, size_t out_dim, float* d_out, objb_stream_t stream) {
  objb::clear_error();
  return objb::moe_combine(d_v, v_rows, d_slot_row, d_weights, num_tokens, top_k, out_dim, d_out,
                           static_cast<cudaStream_t>(stream), nullptr);
}

int objb_router_topk_batched_device(const float* d_logits, size_t num_tokens, size_t num_experts, size_t top_k,
                                    int renormalize, int32_t* d_ids, float* d_weights, objb_stream_t stream) {
  objb::clear_error();
  return objb::router_topk_batched(d_logits, num_tokens, num_experts, top_k, renormalize, d_ids, d_weights,
                                   static_cast<cudaStream_t>(stream));
}

int objb_moe_official_scratch_bytes(const objb_moe_layer* layer, size_t top_k, size_t* bytes) {
  objb::clear_error();
  if (!bytes) return OBJB_FAIL(OBJB_ERR_INVALID_INPUT, "objb_moe_official_scratch_bytes", "null output pointer");
  return objb::moe_official_scratch_bytes(layer, top_k, bytes);
}

int objb_moe_official_selected_device(const objb_moe_layer* layer, const int32_t* d_ids, const float* d_weights,
                                      size_t top_k, const float* d_x, float* d_out, float swiglu_limit,
                                      objb_stream_t stream_) {
  objb::clear_error();
  cudaStream_t stream = static_cast<cudaStream_t>(stream_);
  size_t need = 0;
  OBJB_TRY(objb::moe_official_scratch_bytes(layer, top_k, &need));
  int device = 0;
  OBJB_TRY(objb::current_device(&device));
  void* ws = nullptr;
  OBJB_TRY(objb::workspace_get(device, stream, need, &ws));
  return objb::moe_official_selected(layer, d_ids, d_weights, top_k, d_x, d_out, swiglu_limit, stream, ws, need,
                                     nullptr, nullptr);
}

}  // extern "C"
