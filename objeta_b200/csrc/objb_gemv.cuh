// objb_gemv.cuh -- the batch-1 block-dequant GEMV pipeline for sm_100a.
//
// One persistent CTA per SM streams a contiguous range of rows through a ring
// of shared-memory stages with 1-D bulk TMA copies (cp.async.bulk, one
// elected producer thread, mbarrier completion, L2 evict-first policy).  The
// consumer warps keep the x values of their lane tiles in registers for the
// whole kernel, decode each row's blocks in registers, reduce the row across
// the lanes that share it with warp shuffles and across column segments in
// shared memory, in a fixed order, so results are bit-stable run to run.
//
// The same pipeline runs the MoE kernels: a "job" is one matrix (plus an
// optional second matrix with identical shape whose rows are consumed in the
// same pass) and an epilogue that receives finished row values.
#pragma once

#include <cstdint>

#include "objb_decode.cuh"
#include "objb_pipe.cuh"

namespace objb {
namespace dev {

constexpr int kMaxSlots = 4;
constexpr int kMaxConsumerWarps = 16;
constexpr int kMaxRowsPerStage = 64;

// Geometry of one streamed matrix, decided on the host.
struct RowLayout {
  int rows, cols;
  int nblocks;      // cols / 32
  int row_bytes;    // packed bytes per row (weights)
  int srow_bytes;   // split-FP4 scale bytes per row (0 otherwise)
  int nseg;         // column segments (warps per row)
  int lpr;          // lanes per row slot (power of two, <= 32)
  int rpw;          // rows per warp step = 32 / lpr
  int ngrp;         // row groups; consumer warps = nseg * ngrp
  int tstage;       // rows per pipeline stage
  int nslots;       // ring depth
  int stage_bytes;  // bytes of one ring slot (weights + scales of tstage rows)
};

struct SmemPlan {
  uint64_t* full;
  uint64_t* empty;
  float* red;      // [nslots][tstage][nseg][2]
  uint8_t* stage;  // [nslots][stage_bytes]
};

__device__ __forceinline__ SmemPlan carve_smem(uint8_t* base, const RowLayout& L, int nred) {
  SmemPlan p;
  p.full = reinterpret_cast<uint64_t*>(base);
  p.empty = p.full + kMaxSlots;
  p.red = reinterpret_cast<float*>(base + 2 * kMaxSlots * sizeof(uint64_t));
  size_t red_bytes = static_cast<size_t>(L.nslots) * L.tstage * L.nseg * nred * sizeof(float);
  size_t off = 2 * kMaxSlots * sizeof(uint64_t) + red_bytes;
  off = (off + 127) & ~static_cast<size_t>(127);
  p.stage = base + off;
  return p;
}

// Per-format adapter: x registers and the lane-partial dot of one row.
template <int FMT>
struct RowDot {
  using T = Tile<FMT>;
  static constexpr int XR = T::XR;
  int tile_off;  // byte offset of this lane's tile inside a row
  bool active;
  __device__ __forceinline__ void init(const RowLayout& L, int seg, int ll, const float* x,
                                       float (&xr)[XR]) {
    const int lt = seg * L.lpr + ll;
    active = (lt * T::P) < L.nblocks;
    tile_off = lt * T::TB;
    T::load_x(x, lt * T::P * 32, active, xr);
  }
  __device__ __forceinline__ float dot(const uint8_t* wrow, const uint8_t*,
                                       const float (&xr)[XR]) const {
    return active ? T::dot(wrow + tile_off, xr) : 0.0f;
  }
};

struct RowDotSplitFp4 {
  static constexpr int XR = SplitFp4::XR;
  int b0, stride, nblocks;
  __device__ __forceinline__ void init(const RowLayout& L, int seg, int ll, const float* x,
                                       float (&xr)[XR]) {
    b0 = seg * L.lpr * SplitFp4::P + ll;
    stride = L.lpr;
    nblocks = L.nblocks;
    SplitFp4::load_x(x, b0, stride, nblocks, xr);
  }
  __device__ __forceinline__ float dot(const uint8_t* wrow, const uint8_t* srow,
                                       const float (&xr)[XR]) const {
    return SplitFp4::dot(wrow, srow, b0, stride, nblocks, xr);
  }
};

// The producer side: issues the bulk copies of `nst` stages of up to two
// matrices (A and, when dual, B) into the ring.  Stage i covers rows
// [row0 + i*tstage, ...).  Weights of A land at slot offset 0, scales of A
// after tstage weight rows; B's weights and scales follow A's.
struct StageSource {
  const uint8_t* wa;
  const uint8_t* sa;
  const uint8_t* wb;
  const uint8_t* sb;
};

__device__ __forceinline__ int slot_part_bytes(const RowLayout& L) {
  return L.tstage * (L.row_bytes + L.srow_bytes);
}

// Issues stage `i` (row range [r0, r0 + nr)) into `slot`.
__device__ __forceinline__ void issue_stage(const RowLayout& L, const SmemPlan& sp, int slot,
                                            const StageSource& src, bool dual, int r0, int nr,
                                            uint64_t pol) {
  uint8_t* dst = sp.stage + static_cast<size_t>(slot) * L.stage_bytes;
  const uint32_t wbytes = static_cast<uint32_t>(nr) * L.row_bytes;
  const uint32_t sbytes = static_cast<uint32_t>(nr) * L.srow_bytes;
  const uint32_t per = wbytes + sbytes;
  mbar_arrive_expect_tx(&sp.full[slot], dual ? 2 * per : per);
  bulk_g2s(dst, src.wa + static_cast<size_t>(r0) * L.row_bytes, wbytes, &sp.full[slot], pol);
  if (sbytes)
    bulk_g2s(dst + static_cast<size_t>(L.tstage) * L.row_bytes,
             src.sa + static_cast<size_t>(r0) * L.srow_bytes, sbytes, &sp.full[slot], pol);
  if (dual) {
    uint8_t* dstb = dst + slot_part_bytes(L);
    bulk_g2s(dstb, src.wb + static_cast<size_t>(r0) * L.row_bytes, wbytes, &sp.full[slot], pol);
    if (sbytes)
      bulk_g2s(dstb + static_cast<size_t>(L.tstage) * L.row_bytes,
               src.sb + static_cast<size_t>(r0) * L.srow_bytes, sbytes, &sp.full[slot], pol);
  }
}


// One job = a row range of one matrix (or a matching pair) against one x.
struct Job {
  StageSource src;
  const float* x;
  int row_begin, row_end;
};

// Consumer warps: nseg * ngrp (<= kMaxConsumerWarps); one producer warp more.
constexpr int kPipeThreads = (8 + 1) * 32;

// The pipelined kernel.  `Prog` supplies, for this CTA, a list of jobs and an
// epilogue that receives each finished row (va for matrix A, vb for B):
//   int njobs(int cta) const;   Job job(int cta, int j) const;
//   void epilogue(int cta, int j, int row, float va, float vb) const;
//   void finalize(int cta, int tid, int nthreads) const;   // after all jobs
//   bool dual;  unsigned* err;
template <class RD, class Prog>
__global__ void __launch_bounds__(kPipeThreads, 1) pipe_kernel(const RowLayout L, const Prog prog) {
  extern __shared__ __align__(128) uint8_t smem_raw[];
  const SmemPlan sp = carve_smem(smem_raw, L, 2);
  const int ncw = L.nseg * L.ngrp;
  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const int cta = blockIdx.x;
  const int S = L.nslots;
  const int T = L.tstage;
  unsigned* err = prog.err;

  if (threadIdx.x == 0) {
    for (int i = 0; i < S; ++i) {
      mbar_init(&sp.full[i], 1);
      mbar_init(&sp.empty[i], ncw);
    }
    fence_mbar_init();
  }
  __syncthreads();

  const int njobs = prog.njobs(cta);

  if (warp == ncw) {
    // ---------------- producer: one elected thread issues every stage.
    if (lane == 0) {
      const uint64_t pol = l2_policy_evict_first();
      uint32_t it = 0;
      bool ok = true;
      for (int j = 0; j < njobs && ok; ++j) {
        const Job J = prog.job(cta, j);
        for (int r0 = J.row_begin; r0 < J.row_end; r0 += T) {
          const int slot = static_cast<int>(it % S);
          if (it >= static_cast<uint32_t>(S)) {
            if (!mbar_wait_bounded(&sp.empty[slot], ((it / S) - 1) & 1u, err, kErrEmptyWaitTimeout)) {
              ok = false;
              break;
            }
          }
          const int nr = min(T, J.row_end - r0);
          issue_stage(L, sp, slot, J.src, prog.dual, r0, nr, pol);
          ++it;
        }
      }
      // Never leave while this CTA's own copies may still be landing.
      const uint32_t first = it > static_cast<uint32_t>(S) ? it - S : 0u;
      for (uint32_t k = first; k < it; ++k)
        mbar_wait_bounded(&sp.full[k % S], (k / S) & 1u, nullptr, 0u);
    }
    return;
  }

  // ---------------- consumers
  const int seg = warp % L.nseg;
  const int grp = warp / L.nseg;
  const int sub = lane / L.lpr;
  const int ll = lane % L.lpr;
  const int nthr = ncw * 32;
  const uint32_t shfl_mask = 0xFFFFFFFFu;
  bool ok = true;
  uint32_t it = 0;
  RD rd;
  float xr[RD::XR];
  const int part = slot_part_bytes(L);

  for (int j = 0; j < njobs; ++j) {
    const Job J = prog.job(cta, j);
    rd.init(L, seg, ll, J.x, xr);
    for (int r0 = J.row_begin; r0 < J.row_end; r0 += T) {
      const int slot = static_cast<int>(it % S);
      if (ok) ok = mbar_wait_bounded(&sp.full[slot], (it / S) & 1u, err, kErrFullWaitTimeout);
      const int nr = min(T, J.row_end - r0);
      const uint8_t* stg = sp.stage + static_cast<size_t>(slot) * L.stage_bytes;
      const uint8_t* sca = stg + static_cast<size_t>(T) * L.row_bytes;
      float* red = sp.red + static_cast<size_t>(slot) * T * L.nseg * 2;
      for (int step = grp; step * L.rpw < nr; step += L.ngrp) {
        const int t = step * L.rpw + sub;
        const bool have = t < nr;
        const int tt = have ? t : 0;
        float pa = have ? rd.dot(stg + tt * L.row_bytes, sca + tt * L.srow_bytes, xr) : 0.0f;
        float pb = 0.0f;
        if (prog.dual)
          pb = have ? rd.dot(stg + part + tt * L.row_bytes, stg + part + static_cast<size_t>(T) * L.row_bytes + tt * L.srow_bytes, xr)
                    : 0.0f;
        for (int o = L.lpr >> 1; o > 0; o >>= 1) {
          pa += __shfl_xor_sync(shfl_mask, pa, o);
          if (prog.dual) pb += __shfl_xor_sync(shfl_mask, pb, o);
        }
        if (ll == 0 && have) {
          red[(t * L.nseg + seg) * 2] = pa;
          red[(t * L.nseg + seg) * 2 + 1] = pb;
        }
      }
      __syncwarp();
      if (lane == 0) mbar_arrive(&sp.empty[slot]);
      named_bar_sync(1, nthr);
      for (int t = threadIdx.x; t < nr; t += nthr) {
        float va = 0.0f, vb = 0.0f;
        for (int s2 = 0; s2 < L.nseg; ++s2) {
          va += red[(t * L.nseg + s2) * 2];
          vb += red[(t * L.nseg + s2) * 2 + 1];
        }
        prog.epilogue(cta, j, r0 + t, va, vb);
      }
      ++it;
    }
  }
  named_bar_sync(1, nthr);
  prog.finalize(cta, threadIdx.x, nthr);
}

// Plain GEMV: each CTA owns `rows_per_cta` consecutive rows.
struct GemvProg {
  StageSource src;
  const float* x;
  float* y;
  int rows;
  int rows_per_cta;
  bool dual;
  unsigned* err;
  __device__ __forceinline__ int njobs(int) const { return 1; }
  __device__ __forceinline__ Job job(int cta, int) const {
    Job J;
    J.src = src;
    J.x = x;
    J.row_begin = cta * rows_per_cta;
    J.row_end = min(rows, J.row_begin + rows_per_cta);
    return J;
  }
  __device__ __forceinline__ void epilogue(int, int, int row, float va, float) const { y[row] = va; }
  __device__ __forceinline__ void finalize(int, int, int) const {}
};

// Fallback for shapes / pointers the bulk-copy path cannot take: one warp
// per row, blocks read straight from global memory with byte loads.
template <int FMT>
__global__ void __launch_bounds__(256) gemv_fallback_kernel(const uint8_t* __restrict__ w,
                                                            const float* __restrict__ x,
                                                            float* __restrict__ y, int rows,
                                                            int cols, size_t row_bytes) {
  const int row = blockIdx.x * 8 + (threadIdx.x >> 5);
  const int lane = threadIdx.x & 31;
  if (row >= rows) return;
  constexpr int BB = FMT == OBJB_Q4_0 ? 18 : FMT == OBJB_Q5_0 ? 22 : FMT == OBJB_IQ3_0 ? 14 : 17;
  const int nb = cols / 32;
  const uint8_t* rw = w + static_cast<size_t>(row) * row_bytes;
  float acc = 0.0f;
  for (int b = lane; b < nb; b += 32) acc += block_dot_global<FMT>(rw + static_cast<size_t>(b) * BB, x + b * 32);
  for (int o = 16; o > 0; o >>= 1) acc += __shfl_xor_sync(0xFFFFFFFFu, acc, o);
  if (lane == 0) y[row] = acc;
}

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
}  // namespace objb
