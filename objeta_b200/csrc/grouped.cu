// grouped.cu -- the multi-token ("grouped expert") MoE contraction on the
// tensor cores: for Q4_0 experts, each 128-row tile of an expert's matrix is
// multiplied with the digit planes of up to 32 vectors routed to that expert
// by tcgen05 kind::i8 MMAs (signed codes q - 8 x signed 7-bit digits, both
// s8, S32 in tensor memory), one MMA per 32-column block; the epilogue
// combines the three digit products into the exact integer block sum and
// applies the block's f16 row scale and the vector's block scale in f32:
//   y[v][r] = sum_b d[r][b] * 2^(E[v][b]-20) * sum_i (q[r][b][i] - 8) X[v][b][i]
// -- the arithmetic of the CUDA-core row programs, summed in another order.
// Wide blocks of a vector (objb_decode.cuh) have zero digits here and are
// added in fp32 by the SwiGLU and wide-down kernels.
//
// A launch works on pairs sorted by expert: "slices" (pieces of at most 32
// pairs of one expert) are found on the device (no host round trip), and
// each (slice, 128-row tile) is one work item of a persistent grid.  Before
// the contraction, the digit planes and block scales of every slice are
// gathered into a slice image laid out exactly as the MMA reads its B
// operand (16 or 32 vectors wide).  A work item walks its K in steps of 8
// blocks (256 columns):
//   * one producer thread stages a step with one 2-D TMA copy of the raw
//     Q4_0 tile (128 rows x 144 bytes, rows past the matrix end zero-filled;
//     every slice's tensor maps are written once per call by
//     tc_maps_kernel) and two bulk copies of the slice image;
//   * four unpack warps turn the raw rows into signed code bytes q - 8 in
//     core-matrix order (K-major, no swizzle) and the row block scales;
//   * one warp issues one MMA per block into one of five tensor-memory
//     slots (N = 3 x 16 or 3 x 32 columns each);
//   * sixteen epilogue warps (tensor-memory lanes = tile rows; a quarter of
//     the slice's vectors each) fold the exact block sums into f32 row sums
//     and store them at the item's end.
// Every hand-off is an mbarrier with a bounded wait.
#include <cuda.h>
#include <cudaTypedefs.h>
#include <cuda_runtime.h>

#include <algorithm>
#include <map>
#include <mutex>
#include <string>
#include <utility>

#include "objb_common.h"
#include "objb_decode.cuh"
#include "objb_host_launch.cuh"
#include "objb_launch.h"
#include "objb_moe.cuh"
#include "objb_official_launch.h"
#include "objb_tc.cuh"

namespace objb {
namespace dev {

constexpr int kTcRows = 128;                   // rows per CTA of a 256-row pair tile (M 256 per MMA)
constexpr int kTcNvp = 32;                     // pairs per slice (at most)
constexpr int kTcUnit = 16;                    // vectors per slice-image unit; a slice is 1 or 2 units wide
constexpr int kTcNp = 3 * kTcNvp;              // widest MMA N: three digit planes of kTcNvp vectors
constexpr int kTcKB = 8;                       // 32-column blocks per step
constexpr int kTcStages = 4;                   // ring of raw tiles + slice-image steps
constexpr int kTcAbuf = 2;                     // unpacked code buffers
constexpr int kTcQ = 4;                        // ring of a step's scales for the epilogue
constexpr int kTcItemRing = 16;                // ring of work items (read once, by the producer warp)
constexpr int kTcRawRow = kTcKB * 18;          // raw Q4_0 bytes of one row per step
constexpr int kTcKch = 2 * kTcKB;              // 16-byte K columns of a staged operand
constexpr int kTcSlotCols = 512;              // tensor-memory columns of one MMA group
constexpr int kTcSlots = 1;                    // one slot: a whole step (or half of one) per hand-off
// A group (one wait, one commit) is 8 blocks of a 16-vector slice (48 of 64
// columns each: a whole step) or 4 blocks of a 32-vector slice (96 of 128
// columns each: half a step).
__device__ __forceinline__ int tc_group_blocks(int nv) { return nv > kTcUnit ? 4 : 8; }
constexpr uint32_t kTcTmemCols = 512;
constexpr int kTcUnitBBytes = 3 * kTcUnit * kTcKB * 32;  // digit planes of one unit, one step
constexpr int kTcUnitXFloats = kTcKB * kTcUnit;          // block scales of one unit, one step
// warp roles
constexpr int kTcProducerWarp = 0;
constexpr int kTcMmaWarp = 1;
constexpr int kTcUnpackWarp0 = 2, kTcUnpackWarps = 4;
constexpr int kTcEpiWarp0 = 6, kTcEpiWarps = 16;
constexpr int kTcThreads = 32 * (kTcEpiWarp0 + kTcEpiWarps);

// A work item as the MMA and epilogue warps need it, written by the producer
// warp after its empty[st] wait for the item's first step.  That wait means
// the epilogue has finished step s - kTcStages - kTcQ (unpack waited its
// q_empty before releasing the stage), so with items of one step or more the
// entry being overwritten (item n - kTcItemRing) has been read.
struct TcItemSlot {
  int tile, s0, ns, nv, mat;
  int orow[kTcNvp];  // output row of the slice's vector i (-1 past its length)
};
static_assert(kTcItemRing >= kTcStages + kTcQ, "item ring outlives the producer's lead");

struct TcSmem {
  TcItemSlot items[kTcItemRing];
  alignas(1024) uint8_t a[kTcAbuf][kTcRows * kTcKB * 32];   // signed codes q - 8, core-matrix order
  alignas(1024) uint8_t b[kTcStages][kTcNp / 2 * kTcKB * 32];  // this CTA's half of a slice-image step
  alignas(128) uint8_t raw[kTcStages][kTcRows * kTcRawRow]; // raw Q4_0 rows of a step (bulk copies)
  alignas(16) float xs[kTcStages][kTcKB * kTcNvp];          // vector block scales [block][vector] (bulk copy)
  // the epilogue's copy of a step's scales (written by unpack), so that a
  // stage is free once unpacked and multiplied
  alignas(16) float q_xs[kTcQ][kTcKB * kTcNvp];
  alignas(16) float q_d[kTcQ][kTcKB][kTcRows];              // row block scales
  alignas(8) uint64_t full[kTcStages], empty[kTcStages], a_full[kTcAbuf], a_empty[kTcAbuf];
  uint64_t q_full[kTcQ], q_empty[kTcQ];
  uint64_t t_full[kTcSlots], t_empty[kTcSlots];
  uint32_t tmem_base;
  uint32_t abort;  // a wait of this CTA timed out
};
static_assert(sizeof(TcSmem) <= 227 * 1024, "grouped kernel shared memory");
static_assert(kTcSlots == 1 && kTcSlotCols == 512 && kTcSlots * kTcSlotCols <= static_cast<int>(kTcTmemCols) &&
                  kTcNp <= 128 && kTcKB == 8,
              "tensor-memory slot: 8 blocks x 64 columns or 2 x 4 blocks x 128 columns per step");
static_assert(kTcUnpackWarps * 32 == kTcRows && kTcEpiWarps == 16 && kTcNvp == 2 * kTcUnit, "warp roles");

// Arrival counts of the pipeline barriers.
constexpr uint32_t kTcFullCount = 1;                                  // producer (arrive + transaction bytes)
constexpr uint32_t kTcEmptyCount = 1 + kTcUnpackWarps;               // MMA commit, unpack
constexpr uint32_t kTcQFullCount = kTcUnpackWarps;                    // a step's scales written
constexpr uint32_t kTcQEmptyCount = kTcEpiWarps;                      // a step's scales read
constexpr uint32_t kTcAFullCount = 32 * kTcUnpackWarps;               // every unpack thread
constexpr uint32_t kTcAEmptyCount = 1;                                // MMA commit
constexpr uint32_t kTcTEmptyCount = 2 * kTcEpiWarps;  // the epilogue warps of both CTAs of the pair
constexpr uint32_t kTcPeerCount = kTcUnpackWarps;     // the other CTA's unpack warps, codes of a step written

// 1-D bulk copy (both addresses 16-byte aligned, bytes a multiple of 16).
__device__ __forceinline__ void tc_bulk(void* smem_dst, const void* gsrc, uint32_t bytes, uint64_t* bar) {
  asm volatile("cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(
                   smem_addr(smem_dst)),
               "l"(gsrc), "r"(bytes), "r"(smem_addr(bar))
               : "memory");
}
// 2-D tiled TMA load of the box at (x, y) of the tensor map (no multicast).
__device__ __forceinline__ void tc_tma_2d(void* smem_dst, const CUtensorMap* map, int x, int y, uint64_t* bar) {
  asm volatile(
      "cp.async.bulk.tensor.2d.shared::cluster.global.tile.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3}], [%4];" ::
          "r"(smem_addr(smem_dst)),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(x), "r"(y), "r"(smem_addr(bar))
      : "memory");
}
// Tensor map in global memory: new global address (generic proxy), and the
// release fence that makes such writes visible to the tensor-map proxy.
__device__ __forceinline__ void tc_tmap_set_addr_global(CUtensorMap* gmem_map, const void* addr) {
  asm volatile("tensormap.replace.tile.global_address.global.b1024.b64 [%0], %1;" ::"l"(
                   reinterpret_cast<uint64_t>(gmem_map)),
               "l"(reinterpret_cast<uint64_t>(addr))
               : "memory");
}
__device__ __forceinline__ void tc_tmap_release() {
  asm volatile("fence.proxy.tensormap::generic.release.gpu;" ::: "memory");
}
__device__ __forceinline__ void tc_tmap_acquire(const CUtensorMap* gmem_map) {
  asm volatile("fence.proxy.tensormap::generic.acquire.gpu [%0], 128;" ::"l"(reinterpret_cast<uint64_t>(gmem_map))
               : "memory");
}

// Bounded wait.  On timeout it records kErrFullWaitTimeout in the device
// error word and raises the CTA's abort word (shared memory); it gives up
// early only when another wait of this CTA already raised it (the device
// word keeps codes of earlier launches, and other codes such as a flagged
// index, so it never cuts a wait short).
__device__ __forceinline__ void tc_raise(unsigned* err, uint32_t* abort) {
  if (err) atomicOr(err, kErrFullWaitTimeout);
  *reinterpret_cast<volatile uint32_t*>(abort) = 1u;
}
__device__ __forceinline__ bool tc_wait(uint64_t* bar, uint32_t parity, unsigned* err, uint32_t* abort) {
  for (uint32_t i = 0; i < kMaxSpins; ++i) {
    if (mbar_try_wait(bar, parity)) return true;
    if ((i & 1023u) == 1023u && *reinterpret_cast<volatile uint32_t*>(abort) != 0u) return false;
  }
  tc_raise(err, abort);
  return false;
}

// Bounded wait without suspending the thread between polls (lowest wake-up
// latency; for the MMA-issuing warp, every lane of which polls so that the
// lane elect.sync picks has itself observed the phase).
__device__ __forceinline__ bool tc_spin(uint64_t* bar, uint32_t parity, unsigned* err, uint32_t* abort) {
  for (uint32_t i = 0; i < 64u * kMaxSpins; ++i) {
    uint32_t done;
    asm volatile(
        "{\n\t.reg .pred p;\n\tmbarrier.test_wait.parity.shared::cta.b64 p, [%1], %2;\n\tselp.u32 %0, 1, 0, p;\n\t}"
        : "=r"(done)
        : "r"(smem_addr(bar)), "r"(parity)
        : "memory");
    if (done) return true;
    if ((i & 4095u) == 4095u && *reinterpret_cast<volatile uint32_t*>(abort) != 0u) return false;
  }
  tc_raise(err, abort);
  return false;
}
__device__ __forceinline__ bool tc_spin_warp(uint64_t* bar, uint32_t parity, unsigned* err, uint32_t* abort) {
  return __all_sync(0xFFFFFFFFu, tc_spin(bar, parity, err, abort));
}
// The same for a barrier the other CTA of the pair arrives on (acquire at
// cluster scope).
__device__ __forceinline__ bool tc_spin_cluster(uint64_t* bar, uint32_t parity, unsigned* err, uint32_t* abort) {
  for (uint32_t i = 0; i < 64u * kMaxSpins; ++i) {
    uint32_t done;
    asm volatile(
        "{\n\t.reg .pred p;\n\tmbarrier.test_wait.parity.acquire.cluster.shared::cta.b64 p, [%1], %2;\n\t"
        "selp.u32 %0, 1, 0, p;\n\t}"
        : "=r"(done)
        : "r"(smem_addr(bar)), "r"(parity)
        : "memory");
    if (done) return true;
    if ((i & 4095u) == 4095u && *reinterpret_cast<volatile uint32_t*>(abort) != 0u) return false;
  }
  tc_raise(err, abort);
  return false;
}
__device__ __forceinline__ bool tc_spin_cluster_warp(uint64_t* bar, uint32_t parity, unsigned* err, uint32_t* abort) {
  return __all_sync(0xFFFFFFFFu, tc_spin_cluster(bar, parity, err, abort));
}

// Instruction descriptor of kind::i8 with both operands signed.
__host__ __device__ constexpr uint32_t umma_idesc_s8s8(int m, int n) {
  return (2u << 4) | (1u << 7) | (1u << 10) | ((static_cast<uint32_t>(n) >> 3) << 17) |
         ((static_cast<uint32_t>(m) >> 4) << 24);
}

// Digit planes of one 32-value block of vector v (one warp, one value per
// lane): X = rint(x * 2^(20-E)), E the block's frexp exponent, split in three
// signed 7-bit digits; plane k at planes[(v * 3 + k) * C + col]; per block
// 2^(E-20) (NaN when the block is not finite).  A wide block (block_is_wide:
// its largest value dwarfs the others) gets zero digits, so the MMAs
// add nothing for it, and wflag[v * C/32 + b] = 1: its terms are added in
// fp32 by tc_add_wide_rows (gate / up) and tc_wide_down_kernel (down), and
// wany[v] = 1 (zeroed by tc_slices_kernel).  Returns whether it is wide.
__device__ __forceinline__ bool tc_block_digits(float xe, int v, int b, int C, int8_t* planes, float* xsc,
                                                uint8_t* wflag, uint8_t* wany) {
  const int lane = threadIdx.x & 31, nb = C / 32;
  float m = fabsf(xe);
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) m = fmaxf(m, __shfl_xor_sync(0xFFFFFFFFu, m, o));
  int E = 0;
  frexpf(m, &E);
  const float y = ldexpf(xe, 20 - E);
  const int X0 = __float2int_rn(y);
  const int cnt = __popc(__ballot_sync(0xFFFFFFFFu, fabsf(y) >= kWideFloor));
  const int capped = __reduce_add_sync(0xFFFFFFFFu, min(abs(X0), kWideCap));
  const bool wide = isfinite(m) && block_is_wide(cnt, capped);
  const int X = wide ? 0 : X0;
  const int d0 = ((X + 64) & 127) - 64;
  const int X1 = (X - d0) / 128;
  const int d1 = ((X1 + 64) & 127) - 64;
  const int d2 = (X1 - d1) / 128;
  int8_t* p = planes + static_cast<size_t>(v) * 3 * C + b * 32 + lane;
  p[0] = static_cast<int8_t>(d0);
  p[C] = static_cast<int8_t>(d1);
  p[2 * C] = static_cast<int8_t>(d2);
  if (lane == 0) {
    xsc[static_cast<size_t>(v) * nb + b] = isfinite(m) ? ldexpf(1.0f, E - 20) : __int_as_float(0x7FC00000);
    wflag[static_cast<size_t>(v) * nb + b] = wide ? 1 : 0;
    if (wide) wany[v] = 1;
  }
  return wide;
}

// Digit planes of `nvec` vectors (rows of x, x_stride apart); one warp per
// (vector, block).
__global__ void __launch_bounds__(256) tc_planes_kernel(const float* __restrict__ x, size_t x_stride, int nvec,
                                                        const int32_t* count, int C, int8_t* __restrict__ planes,
                                                        float* __restrict__ xsc, uint8_t* __restrict__ wflag,
                                                        uint8_t* __restrict__ wany) {
  asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
  asm volatile("griddepcontrol.wait;" ::: "memory");
  if (count) nvec = min(max(*count, 0), nvec);
  const int nb = C / 32, lane = threadIdx.x & 31;
  const int warps = (gridDim.x * blockDim.x) >> 5;
  for (int wi = (blockIdx.x * blockDim.x + threadIdx.x) >> 5; wi < nvec * nb; wi += warps) {
    const int v = wi / nb, b = wi % nb;
    tc_block_digits(x[static_cast<size_t>(v) * x_stride + b * 32 + lane], v, b, C, planes, xsc, wflag, wany);
  }
}

// Adds to `acc` (this lane's row r of a Q4_0 matrix, row_bytes apart) the
// fp32 terms of the wide blocks of vector xv (flags wf[0 .. nb)), rounded as
// the reference's dot rows round them (quant.rs:950-970):
// ((q - 8) * scale) * x per element, in element order.  Warp-uniform loop
// over the flagged blocks; x is read once per block (one value per lane) and
// broadcast by shuffles.  `row` must point at a readable row for every lane
// (a lane that is not `live` keeps acc).
__device__ __forceinline__ float tc_add_wide_rows(float acc, const uint8_t* __restrict__ row,
                                                  const float* __restrict__ xv, const uint8_t* __restrict__ wf,
                                                  int nb, bool live) {
  const int lane = threadIdx.x & 31;
  for (int b0 = 0; b0 < nb; b0 += 32) {
    uint32_t m = __ballot_sync(0xFFFFFFFFu, b0 + lane < nb && wf[b0 + lane] != 0);
    while (m) {
      const int b = b0 + __ffs(m) - 1;
      m &= m - 1;
      // every lane runs the shuffles; `row` is a valid row even for a lane
      // that is not live, whose sum is dropped
      const float xl = __ldg(xv + b * 32 + lane);
      const uint8_t* blk = row + static_cast<size_t>(b) * 18;
      const float sc = f16_bits_to_f32(blk[0] | (static_cast<uint32_t>(blk[1]) << 8));
      float t = 0.0f;
      for (int k = 0; k < 32; ++k) {
        const float xk = __shfl_sync(0xFFFFFFFFu, xl, k);
        t = __fadd_rn(t, __fmul_rn(__fmul_rn(qf(block_code<OBJB_Q4_0>(blk, k), 8.0f), sc), xk));
      }
      if (live) acc = __fadd_rn(acc, t);
    }
  }
  return acc;
}

// act = SwiGLU(g, u) of every pair (rows of I floats) straight into digit
// planes; one warp per (pair, block).  First the gate / up rows get the fp32
// terms of their token's wide blocks (the grouped launch added nothing for
// them; a token with none, wany_x[t] == 0, costs one byte read); an
// activation block that is itself wide is also stored over g, for the down
// rows' wide-block terms.
__global__ void __launch_bounds__(256) tc_swiglu_planes_kernel(float* __restrict__ g,
                                                               const float* __restrict__ u, int P,
                                                               const int32_t* count, int I, float limit,
                                                               int8_t* __restrict__ planes, float* __restrict__ xsc,
                                                               uint8_t* __restrict__ wflag_a,
                                                               uint8_t* __restrict__ wany_a, const int32_t* pe,
                                                               const int32_t* pt, int T, const float* __restrict__ x,
                                                               int H, const uint8_t* __restrict__ wflag_x,
                                                               const uint8_t* __restrict__ wany_x,
                                                               const uint8_t* const* gate_w,
                                                               const uint8_t* const* up_w, int num_experts) {
  asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
  asm volatile("griddepcontrol.wait;" ::: "memory");
  if (count) P = min(max(*count, 0), P);
  const int nb = I / 32, nbh = H / 32, lane = threadIdx.x & 31;
  const size_t row_bytes = static_cast<size_t>(nbh) * 18;
  const int warps = (gridDim.x * blockDim.x) >> 5;
  for (int wi = (blockIdx.x * blockDim.x + threadIdx.x) >> 5; wi < P * nb; wi += warps) {
    const int p = wi / nb, b = wi % nb;
    const size_t i = static_cast<size_t>(p) * I + b * 32 + lane;
    float gv = g[i], uv = u[i];
    int t = pt[p], e = pe[p];
    const bool ok = t >= 0 && t < T && e >= 0 && e < num_experts;
    if (!ok) {  // the grouped launch flagged it already; no wide terms
      t = 0;
      e = 0;
    }
    if (ok && wany_x[t]) {
      const uint8_t* wf = wflag_x + static_cast<size_t>(t) * nbh;
      const float* xv = x + static_cast<size_t>(t) * H;
      const size_t roff = static_cast<size_t>(b * 32 + lane) * row_bytes;
      gv = tc_add_wide_rows(gv, gate_w[e] + roff, xv, wf, nbh, true);
      uv = tc_add_wide_rows(uv, up_w[e] + roff, xv, wf, nbh, true);
    }
    const float a = swiglu(gv, uv, limit);
    if (tc_block_digits(a, p, b, I, planes, xsc, wflag_a, wany_a)) g[i] = a;
  }
}

// The down rows' terms of the activations' wide blocks: v[slot(p)][r] +=
// sum over the wide blocks of pair p's activation (act rows of I floats; the
// wide blocks' values were stored there) of ((q - 8) * scale) * act.  One
// warp per pair; a pair with no wide block (wany_a[p] == 0) costs one byte
// read, one with some walks every 32 output rows.
__global__ void __launch_bounds__(256) tc_wide_down_kernel(const float* __restrict__ act, int P, const int32_t* count,
                                                           int I, int O, const uint8_t* __restrict__ wflag_a,
                                                           const uint8_t* __restrict__ wany_a, const int32_t* pe,
                                                           const int32_t* po, int v_rows,
                                                           const uint8_t* const* down_w, int num_experts,
                                                           const int32_t* nslices, float* __restrict__ v) {
  asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
  asm volatile("griddepcontrol.wait;" ::: "memory");
  if (*nslices <= 0) return;  // the launch ran nothing (a pair list not grouped by expert): v stays as it was
  if (count) P = min(max(*count, 0), P);
  const int nb = I / 32, lane = threadIdx.x & 31;
  const size_t row_bytes = static_cast<size_t>(nb) * 18;
  const int warps = (gridDim.x * blockDim.x) >> 5;
  for (int p = (blockIdx.x * blockDim.x + threadIdx.x) >> 5; p < P; p += warps) {
    if (!wany_a[p]) continue;
    const int e = pe[p], o = po ? po[p] : p;
    if (e < 0 || e >= num_experts || o < 0 || o >= v_rows) continue;  // flagged by the grouped launch
    const uint8_t* wf = wflag_a + static_cast<size_t>(p) * nb;
    for (int r0 = 0; r0 < O; r0 += 32) {
      const int r = r0 + lane;
      const bool live = r < O;
      const size_t roff = static_cast<size_t>(live ? r : 0) * row_bytes;
      const float add = tc_add_wide_rows(0.0f, down_w[e] + roff, act + static_cast<size_t>(p) * I, wf, nb, live);
      if (live) {
        float* dst = v + static_cast<size_t>(o) * O + r;
        *dst = __fadd_rn(*dst, add);
      }
    }
  }
}

// Work slices of the expert-sorted pair list: runs of equal experts cut into
// pieces of at most `nvp` pairs -> slice_start / slice_len [0..n), n in
// *nslices.  One CTA; each thread scans a contiguous slice of the pairs.
// With slice_order (and nslices of two entries) it also lists the slices
// widest first, for the grouped kernels' item assignment.
__device__ __forceinline__ int block_exclusive_scan(int v, int* total, int* warp_tot) {
  const int lane = threadIdx.x & 31, wid = threadIdx.x >> 5, nt = blockDim.x;
  int incl = v;
#pragma unroll
  for (int o = 1; o < 32; o <<= 1) {
    const int y = __shfl_up_sync(0xFFFFFFFFu, incl, o);
    if (lane >= o) incl += y;
  }
  __syncthreads();
  if (lane == 31) warp_tot[wid] = incl;
  __syncthreads();
  if (wid == 0) {
    const int nw = (nt + 31) >> 5;
    int w = lane < nw ? warp_tot[lane] : 0;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
      const int y = __shfl_up_sync(0xFFFFFFFFu, w, o);
      if (lane >= o) w += y;
    }
    if (lane < nw) warp_tot[lane] = w;
  }
  __syncthreads();
  *total = warp_tot[((nt + 31) >> 5) - 1];
  return incl - v + (wid ? warp_tot[wid - 1] : 0);
}

__global__ void __launch_bounds__(1024) tc_slices_kernel(const int32_t* __restrict__ pe, int P, const int32_t* count,
                                                         int nvp, int unit, int32_t* __restrict__ run_start,
                                                         int32_t* __restrict__ slice_start,
                                                         int32_t* __restrict__ slice_len,
                                                         int32_t* __restrict__ slice_unit,
                                                         int32_t* __restrict__ nslices, int unit_cap,
                                                         unsigned* err, uint8_t* __restrict__ wany_x, int T,
                                                         uint8_t* __restrict__ wany_a,
                                                         int32_t* __restrict__ slice_order) {
  asm volatile("griddepcontrol.wait;" ::: "memory");
  __shared__ int warp_tot[32];
  // the any-wide bytes of this call start clear (the planes kernels set them)
  if (wany_x)
    for (int i = threadIdx.x; i < T; i += blockDim.x) wany_x[i] = 0;
  if (wany_a)
    for (int i = threadIdx.x; i < P; i += blockDim.x) wany_a[i] = 0;
  if (count) P = min(max(*count, 0), P);
  const int nt = blockDim.x, tid = threadIdx.x;
  // 1. run starts
  int per = (P + nt - 1) / nt;
  int a = min(P, tid * per), b = min(P, a + per);
  int local = 0;
  for (int p = a; p < b; ++p) local += (p == 0 || pe[p] != pe[p - 1]);
  int nruns = 0;
  int pos = block_exclusive_scan(local, &nruns, warp_tot);
  for (int p = a; p < b; ++p)
    if (p == 0 || pe[p] != pe[p - 1]) run_start[pos++] = p;
  __syncthreads();
  // 2. slices of each run, and their offsets in slice-image units
  per = (nruns + nt - 1) / nt;
  a = min(nruns, tid * per);
  b = min(nruns, a + per);
  local = 0;
  int lunits = 0;
  for (int r = a; r < b; ++r) {
    const int s0 = run_start[r], s1 = r + 1 < nruns ? run_start[r + 1] : P;
    for (int q = s0; q < s1; q += nvp) {
      ++local;
      lunits += (min(nvp, s1 - q) + unit - 1) / unit;
    }
  }
  int total = 0, total_units = 0;
  pos = block_exclusive_scan(local, &total, warp_tot);
  int upos = block_exclusive_scan(lunits, &total_units, warp_tot);
  for (int r = a; r < b; ++r) {
    const int s0 = run_start[r], s1 = r + 1 < nruns ? run_start[r + 1] : P;
    for (int q = s0; q < s1; q += nvp) {
      const int len = min(nvp, s1 - q);
      slice_start[pos] = q;
      slice_len[pos] = len;
      slice_unit[pos] = upos;
      upos += (len + unit - 1) / unit;
      ++pos;
    }
  }
  // 3. (optional) the slices by width in units, widest first, each width in
  // slice order (a counting sort); nslices[1] = how many are wider than one
  // unit
  if (slice_order) {
    __syncthreads();  // every slice length written
    per = (total + nt - 1) / nt;
    a = min(total, tid * per);
    b = min(total, a + per);
    int base = 0, nwide = 0;
    for (int c = (nvp + unit - 1) / unit; c >= 1; --c) {
      local = 0;
      for (int q = a; q < b; ++q) local += (slice_len[q] + unit - 1) / unit == c;
      int cnt = 0;
      int at = base + block_exclusive_scan(local, &cnt, warp_tot);
      for (int q = a; q < b; ++q)
        if ((slice_len[q] + unit - 1) / unit == c) slice_order[at++] = q;
      base += cnt;
      if (c == 2) nwide = base;
    }
    if (tid == 0) nslices[1] = nwide;
  }
  // a pair list not grouped by expert can need more image space than sized
  // for: run nothing and flag it
  if (tid == 0) {
    *nslices = total_units <= unit_cap ? total : 0;
    if (total_units > unit_cap && err) atomicOr(err, kErrBadExpertId);
  }
}

// The slice images of one contraction: for slice sl, step c, the B operand
// rows 3 i + k (plane k of the slice's vector i, nv = 16 or 32) in
// core-matrix order, then the block scales [block][vector]; unit offsets
// from tc_slices_kernel.  Rows and scales past the slice's length are not
// written: the MMAs multiply them into columns that the epilogue never reads
// or stores.  One warp per (slice, vector): one id lookup, then the vector's
// three digit planes for every step, read contiguously (several loads in
// flight per lane) and scattered as 16-byte core-matrix rows.
__global__ void __launch_bounds__(256) tc_image_kernel(const int32_t* __restrict__ slice_start,
                                                       const int32_t* __restrict__ slice_len,
                                                       const int32_t* __restrict__ slice_unit,
                                                       const int32_t* __restrict__ nslices,
                                                       const int8_t* __restrict__ planes,
                                                       const float* __restrict__ xsc,
                                                       const int32_t* __restrict__ slot_vec, int nvec, int C,
                                                       uint8_t* __restrict__ bimg, float* __restrict__ ximg) {
  asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
  asm volatile("griddepcontrol.wait;" ::: "memory");
  constexpr int kBatch = 4;  // steps per plane in flight per lane before their stores
  const int lane = threadIdx.x & 31;
  const int nchunks = C / (kTcKB * 32), nb = C / 32, kc = C / 16;  // steps, blocks, 16-byte columns
  const int nsl = *nslices, total = nsl * kTcNvp;
  const int nwarps = static_cast<int>(gridDim.x * blockDim.x) >> 5;
  // vector-major order: the live items (small i, present in most slices)
  // spread over every block instead of a quarter of them
  for (int w = static_cast<int>((blockIdx.x * blockDim.x + threadIdx.x) >> 5); w < total; w += nwarps) {
    const int sl = w % nsl, i = w / nsl;
    const int ns = slice_len[sl];
    if (i >= ns) continue;
    const int s0 = slice_start[sl];
    const int nv = ns > kTcUnit ? 2 * kTcUnit : kTcUnit, units = nv / kTcUnit;
    const size_t ubase = static_cast<size_t>(slice_unit[sl]) * nchunks;
    int v = slot_vec ? slot_vec[s0 + i] : s0 + i;
    v = (v < 0 || v >= nvec) ? 0 : v;
    // a lane copies the 16-byte column pk of steps c = cl, cl + 2, ... of the
    // three planes: contiguous reads across lanes, and a store address that
    // is a fixed per-plane row offset plus c times the step's image size
    const uint4* src = reinterpret_cast<const uint4*>(planes + static_cast<size_t>(v) * 3 * C);
    const int cl = lane >> 4, pk = lane & 15;
    const size_t step_bytes = static_cast<size_t>(units) * kTcUnitBBytes;
    uint8_t* base = bimg + ubase * kTcUnitBBytes;
    size_t rowoff[3];
#pragma unroll
    for (int k = 0; k < 3; ++k) {
      const int brow = 3 * i + k;
      rowoff[k] = static_cast<size_t>(((brow >> 3) * kTcKch + pk) * 128 + (brow & 7) * 16);
    }
    for (int c0 = cl; c0 < nchunks; c0 += 2 * kBatch) {
      uint4 t[3][kBatch];
#pragma unroll
      for (int k = 0; k < 3; ++k)
#pragma unroll
        for (int u = 0; u < kBatch; ++u) {
          const int c = c0 + 2 * u;
          if (c < nchunks) t[k][u] = src[k * kc + c * kTcKch + pk];
        }
#pragma unroll
      for (int k = 0; k < 3; ++k)
#pragma unroll
        for (int u = 0; u < kBatch; ++u) {
          const int c = c0 + 2 * u;
          if (c < nchunks) *reinterpret_cast<uint4*>(base + rowoff[k] + static_cast<size_t>(c) * step_bytes) = t[k][u];
        }
    }
    for (int q = lane; q < nb; q += 32) {
      const int c = q / kTcKB, j = q % kTcKB;
      ximg[(ubase + static_cast<size_t>(c) * units) * kTcUnitXFloats + j * nv + i] =
          xsc[static_cast<size_t>(v) * nb + q];
    }
  }
}

// The tensor maps of every slice's gate, up and down matrices: maps[3 sl + k]
// = template k (gate / up share one) with the global address of expert
// pe[slice_start[sl]]'s matrix.  Written once per call, so the grouped
// kernels only acquire a map when an item starts (no per-item rewrite).
__global__ void __launch_bounds__(256) tc_maps_kernel(const __grid_constant__ CUtensorMap t_gu,
                                                      const __grid_constant__ CUtensorMap t_dn,
                                                      const int32_t* __restrict__ slice_start,
                                                      const int32_t* __restrict__ nslices, int max_slices,
                                                      const int32_t* __restrict__ pe, const uint8_t* const* Wg,
                                                      const uint8_t* const* Wu, const uint8_t* const* Wd, int E,
                                                      CUtensorMap* __restrict__ maps) {
  asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
  asm volatile("griddepcontrol.wait;" ::: "memory");
  const int n = min(*nslices, max_slices);
  for (int i = blockIdx.x * blockDim.x + threadIdx.x; i < 3 * n; i += gridDim.x * blockDim.x) {
    const int sl = i / 3, k = i % 3;
    int e = pe[slice_start[sl]];
    if (e < 0 || e >= E) e = 0;  // flagged by the grouped kernel
    const uint8_t* w = k == 0 ? Wg[e] : (k == 1 ? Wu[e] : Wd[e]);
    const uint4* src = reinterpret_cast<const uint4*>(k == 2 ? &t_dn : &t_gu);
    uint4* dst = reinterpret_cast<uint4*>(&maps[i]);
#pragma unroll
    for (int q = 0; q < 8; ++q) dst[q] = src[q];
    tc_tmap_set_addr_global(&maps[i], w);
  }
  tc_tmap_release();
}

// Operands of one launch of the grouped kernel.
struct TcArgs {
  const uint8_t* const* W;   // expert matrices [R][C/32 blocks of 18 bytes]
  const uint8_t* const* W2;  // second matrix of the same experts (gate + up in one launch), or null
  int num_experts, R, C;
  const int32_t* pe;         // expert of each pair (sorted)
  const int32_t* slot_vec;   // vector of each pair (null: the pair index)
  const int32_t* slot_out;   // output row of each pair (null: the pair index)
  const int32_t* slice_start;
  const int32_t* slice_len;
  const int32_t* slice_unit;
  const int32_t* nslices;      // [0] slices, [1] slices wider than one unit
  const int32_t* slice_order;  // the wide slices first (tc_slices_kernel)
  const uint8_t* bimg;       // slice images (tc_image_kernel)
  const float* ximg;
  const CUtensorMap* maps;   // tensor maps of every slice's matrices (tc_maps_kernel): [slice][gate, up, down]
  int map0;                  // 0: gate (+ up), 2: down
  int box_rows;              // rows of the maps' box (min(128, R))
  int nvec;
  float* out;                // [out_rows][R]
  float* out2;               // for W2
  int out_rows;
  unsigned* err;
};

struct TcItem {
  const CUtensorMap* map;
  float* dst;
  int tile, s0, ns, nv, unit;
};

// Item o of the launch's ordered list: (slice slice_order[o / (tiles mats)],
// tile, matrix), the matrix fastest.
__device__ __forceinline__ TcItem tc_item(const TcArgs& A, int o, int tiles, int mats) {
  TcItem it;
  const int mat = o % mats, rest = o / mats;
  const int sl = A.slice_order[rest / tiles];
  it.tile = rest % tiles;
  it.s0 = A.slice_start[sl];
  it.ns = min(max(A.slice_len[sl], 1), kTcNvp);
  it.nv = it.ns > kTcUnit ? 2 * kTcUnit : kTcUnit;
  it.unit = A.slice_unit[sl];
  it.map = A.maps + 3 * sl + A.map0 + mat;
  it.dst = mat ? A.out2 : A.out;
  return it;
}

// Unpack (four warps, thread = tile row): raw row of ring slot `st` -> signed
// codes q - 8 in core-matrix order (A buffer `ab`) and the row's block scales
// (beside the stage, so that the A buffer is free once the MMAs have read it).
__device__ __forceinline__ void tc_unpack(TcSmem& sm, int st, int ab, int q, int r) {
  uint32_t w[kTcRawRow / 4];
  const uint8_t* src = sm.raw[st] + r * kTcRawRow;
#pragma unroll
  for (int q = 0; q < kTcRawRow / 16; ++q) {
    const uint4 x = *reinterpret_cast<const uint4*>(src + 16 * q);
    w[4 * q] = x.x, w[4 * q + 1] = x.y, w[4 * q + 2] = x.z, w[4 * q + 3] = x.w;
  }
#pragma unroll
  for (int b = 0; b < kTcKB; ++b) {
    // block b occupies bytes [18 b, 18 b + 18): f16 scale, 16 code bytes
    const int wi = 18 * b / 4;
    uint32_t d16, qs[4];
    if ((18 * b) % 4 == 0) {
      d16 = w[wi] & 0xFFFFu;
#pragma unroll
      for (int m = 0; m < 4; ++m) qs[m] = __funnelshift_r(w[wi + m], w[wi + m + 1], 16);
    } else {
      d16 = w[wi] >> 16;
#pragma unroll
      for (int m = 0; m < 4; ++m) qs[m] = w[wi + 1 + m];
    }
    uint32_t c[8];
#pragma unroll
    for (int m = 0; m < 4; ++m) {
      // bytes q in [0, 15] -> q - 8 as int8: (q + 0x78) ^ 0x80, no carry between bytes
      const uint32_t lo = (qs[m] & 0x0F0F0F0Fu) + 0x78787878u, hi = ((qs[m] >> 4) & 0x0F0F0F0Fu) + 0x78787878u;
      c[2 * m] = __byte_perm(lo, hi, 0x5140) ^ 0x80808080u;      // codes 8m .. 8m+3
      c[2 * m + 1] = __byte_perm(lo, hi, 0x7362) ^ 0x80808080u;  // codes 8m+4 .. 8m+7
    }
    uint8_t* dst = sm.a[ab] + ((r >> 3) * kTcKch + 2 * b) * 128 + (r & 7) * 16;
    *reinterpret_cast<uint4*>(dst) = make_uint4(c[0], c[1], c[2], c[3]);
    *reinterpret_cast<uint4*>(dst + 128) = make_uint4(c[4], c[5], c[6], c[7]);
    sm.q_d[q][b][r] = f16_bits_to_f32(d16);
  }
}

// The grouped contraction of Q4_0 matrices: out[slot_out[p]][r] = y[vector
// slot_vec[p]][r] of expert pe[p]'s matrix for every pair p.  Needs C a
// multiple of 256, 16-byte aligned matrices and the slice images of this
// launch.
//
// A 2-CTA cluster (a CTA pair on two SMs) works one 256-row tile at a time:
// each CTA stages its 128 rows and half of the slice image, and the even
// CTA issues M256 cta_group::2 MMAs (about 35 cycles of issue each, against
// 170 to 230 for an M128 MMA of one CTA) whose sums land in each CTA's own
// tensor memory.  Commits are multicast to both CTAs' barriers; the odd
// CTA's unpack and epilogue warps arrive on the even CTA's barriers.
//
// Roles and hand-offs (every wait bounded):
//   producer   empty[st] -> raw tile (2-D TMA) + slice-image half + block scales -> full[st]
//   unpack     full[st], a_empty[ab], q_empty[q] -> codes a[ab], scales q_d/q_xs[q] -> a_full[ab], q_full[q],
//              empty[st]
//              (odd CTA: also a_full[ab] of the even CTA, one arrival per warp)
//   MMA        (even CTA) a_full[ab]; per group t_empty -> 4 or 8 MMAs -> t_full
//              (both CTAs); then a_empty[ab], empty[st] (both CTAs)
//   epilogue   q_full[q]; per group t_full -> tensor-memory loads -> t_empty (even CTA); q_empty[q]
// A code buffer is released by the MMAs alone, so the unpack of step s + 2
// overlaps the epilogue of step s.  One 512-column tensor-memory slot holds
// a whole step of a 16-vector slice (half a step of a 32-vector one), so a
// step crosses between the SMs once: the epilogue loads it in one batch of
// packed 16-bit loads and releases the slot before folding.  The releases are
// relaxed cluster arrivals (the tcgen05 fences order the tensor-memory
// accesses; a release at cluster scope costs the arriving warp hundreds of
// cycles).  Epilogue warp (quarter q, set w) owns tile rows 32 q .. 32 q + 31
// of its CTA and vectors w * nv/4 .. (w + 1) * nv/4 - 1 of every block, so its
// sums need no exchange with other warps; a warp whose vectors are all past
// the slice's length still waits and arrives, without loading.
// A block's columns hold, per vector i and digit plane k, the int32 sum
// r_k(i) = sum over the block's 32 elements of (q - 8) * digit_k at column
// 3 i + k.  |r_k| <= 32 * 8 * 64 = 16384, so the low 16 bits hold it: the
// loads take two columns per register (.pack::16b), the 3 NVW columns of a
// warp's NVW vectors in 3 NVW / 2 registers, in column order.
template <int NVW>
__device__ __forceinline__ void tc_epi_load(uint32_t taddr, uint32_t (&r)[3 * NVW / 2]) {
#pragma unroll
  for (int m = 0; m < 3; ++m) {
    if constexpr (NVW == 8)
      tmem_ld4_pack16(taddr + m * 8, r[4 * m], r[4 * m + 1], r[4 * m + 2], r[4 * m + 3]);
    else
      tmem_ld2_pack16(taddr + m * 4, r[2 * m], r[2 * m + 1]);
  }
}
// d = lo16(a) * byte0(b) + hi16(a) * byte1(b) + c, a's halves signed, b's bytes unsigned.
__device__ __forceinline__ int dp2a_lo_su(uint32_t a, uint32_t b, int c) {
  int d;
  asm("dp2a.lo.s32.u32 %0, %1, %2, %3;" : "=r"(d) : "r"(a), "r"(b), "r"(c));
  return d;
}
// Block sums of a vector pair (2p, 2p + 1) from its three registers
// ra = [r0 | r1], rb = [r2 | r0'], rc = [r1' | r2']:
//   S = r0 + 128 r1 + 16384 r2,  S' = r0' + 128 (r1' + 128 r2'),
// then acc += f32(S) * (d * xv) as in the block epilogue before.
template <int NVW>
__device__ __forceinline__ void tc_epi_fold(const uint32_t (&r)[3 * NVW / 2], float dr, const float* xsv,
                                            float (&acc)[8]) {
  float xv[NVW];
#pragma unroll
  for (int q = 0; q < NVW / 4; ++q) {
    const float4 t = *reinterpret_cast<const float4*>(xsv + 4 * q);
    xv[4 * q] = t.x, xv[4 * q + 1] = t.y, xv[4 * q + 2] = t.z, xv[4 * q + 3] = t.w;
  }
  constexpr uint32_t kRadix = 0x8001u;  // bytes 1, 128
#pragma unroll
  for (int u = 0; u < NVW; u += 2) {
    const uint32_t ra = r[3 * (u / 2)], rb = r[3 * (u / 2) + 1], rc = r[3 * (u / 2) + 2];
    const int S0 = dp2a_lo_su(ra, kRadix, static_cast<int>(rb << 16) >> 2);
    const int S1 = (static_cast<int>(rb) >> 16) + dp2a_lo_su(rc, kRadix, 0) * 128;
    const float2 sc = __fmul2_rn(make_float2(dr, dr), make_float2(xv[u], xv[u + 1]));
    const float2 a = __ffma2_rn(make_float2(__int2float_rn(S0), __int2float_rn(S1)), sc, make_float2(acc[u], acc[u + 1]));
    acc[u] = a.x, acc[u + 1] = a.y;
  }
}
// One MMA group of an epilogue warp: tensor-memory loads of its GB blocks
// (column stride BS) in one batch, the slot released to the pair's MMA warp
// (in CTA 0), then the folds.
template <int NVW, int GB, int BS>
__device__ __forceinline__ void tc_epi_group(uint32_t taddr, int nv, const float* dcol, const float* xsv,
                                             uint64_t* t_empty, float (&acc)[8]) {
  uint32_t r[GB][3 * NVW / 2];
#pragma unroll
  for (int b = 0; b < GB; ++b) tc_epi_load<NVW>(taddr + b * BS, r[b]);
  tmem_wait_ld();
  tc_fence_before_sync();
  __syncwarp();
  if ((threadIdx.x & 31) == 0) mbar_arrive_cta_relaxed(t_empty, 0);  // the pair's MMAs are issued by CTA 0
#pragma unroll
  for (int b = 0; b < GB; ++b) tc_epi_fold<NVW>(r[b], dcol[b * kTcRows], xsv + b * nv, acc);
}

__global__ void __cluster_dims__(2, 1, 1) __launch_bounds__(kTcThreads, 1) tc_q4_grouped_kernel(const TcArgs A) {
  extern __shared__ __align__(1024) uint8_t tc_smem_raw[];
  TcSmem& sm = *reinterpret_cast<TcSmem*>(tc_smem_raw);
  asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  if (tid == 0) {
    for (int i = 0; i < kTcStages; ++i) {
      mbar_init(&sm.full[i], kTcFullCount);
      mbar_init(&sm.empty[i], kTcEmptyCount);
    }
    for (int i = 0; i < kTcQ; ++i) {
      mbar_init(&sm.q_full[i], kTcQFullCount);
      mbar_init(&sm.q_empty[i], kTcQEmptyCount);
    }
    for (int i = 0; i < kTcAbuf; ++i) {
      // the even CTA's also counts the odd CTA's unpack warps (its codes and
      // slice-image half of the step are in place)
      mbar_init(&sm.a_full[i], kTcAFullCount + (cluster_ctarank() == 0 ? kTcPeerCount : 0u));
      mbar_init(&sm.a_empty[i], kTcAEmptyCount);
    }
    for (int i = 0; i < kTcSlots; ++i) {
      mbar_init(&sm.t_full[i], 1);
      mbar_init(&sm.t_empty[i], kTcTEmptyCount);
    }
    sm.abort = 0u;
    fence_mbar_init();
  }
  if (warp == kTcMmaWarp) tmem_alloc_pair(&sm.tmem_base, kTcTmemCols);
  __syncthreads();
  cluster_sync_all();  // both CTAs' barriers exist before either arrives on the other's
  tc_fence_after_sync();
  const uint32_t tmem = sm.tmem_base;
  const uint32_t rank = cluster_ctarank();  // 0: issues the MMAs of the pair
  const int pair = static_cast<int>(blockIdx.x) >> 1, npairs = static_cast<int>(gridDim.x) >> 1;
  asm volatile("griddepcontrol.wait;" ::: "memory");

  const int nb = A.C / 32, nchunks = nb / kTcKB;
  const int tiles = (A.R + 2 * kTcRows - 1) / (2 * kTcRows);  // 256-row tiles of the pair
  const int mats = A.W2 ? 2 : 1;
  // Static item assignment balanced for cost: a wide slice's item (32
  // vectors: two tensor-memory hand-offs a step) costs about two narrow
  // ones.  The wide items go round-robin over the pairs; the narrow ones
  // round-robin from the first pair that got one fewer wide item.  A pair
  // takes its wide items first.
  const int per_slice = tiles * mats;
  const int total = *A.nslices * per_slice, wide_items = A.nslices[1] * per_slice;
  const int narrow_items = total - wide_items;
  const int my_wide = wide_items / npairs + (pair < wide_items % npairs ? 1 : 0);
  const int nfirst = (pair - wide_items % npairs + npairs) % npairs;  // this pair's first narrow item
  const int my_items = my_wide + narrow_items / npairs + (nfirst < narrow_items % npairs ? 1 : 0);
  const int nsteps = my_items * nchunks;
  auto item_at = [&](int s) {
    const int i = s / nchunks;
    const int o = i < my_wide ? pair + i * npairs : wide_items + nfirst + (i - my_wide) * npairs;
    return tc_item(A, o, tiles, mats);
  };
  const int row0 = static_cast<int>(rank) * kTcRows;  // this CTA's rows within a pair tile

  if (warp == kTcProducerWarp) {
    // the whole warp reads each item (its fields, the slice's output rows,
    // the pair ids checked); lane 0 issues the copies
    TcItem it{};
#pragma unroll 1
    for (int s = 0; s < nsteps; ++s) {
      const int st = s % kTcStages, chunk = s % nchunks;
      bool okw = true;
      if (lane == 0 && s >= kTcStages) okw = tc_wait(&sm.empty[st], ((s / kTcStages) - 1) & 1, A.err, &sm.abort);
      if (!__shfl_sync(0xFFFFFFFFu, okw, 0)) break;
      __syncwarp();  // lane 0's wait orders the other lanes' entry writes below
      if (chunk == 0) {
        it = item_at(s);
        TcItemSlot& e = sm.items[(s / nchunks) % kTcItemRing];
        int o = -1;
        if (lane < it.ns) {
          const int p = it.s0 + lane;
          o = A.slot_out ? A.slot_out[p] : p;
          const int v = A.slot_vec ? A.slot_vec[p] : p;
          const int x = A.pe[p];
          if ((o < 0 || o >= A.out_rows || v < 0 || v >= A.nvec || x < 0 || x >= A.num_experts) && A.err)
            atomicOr(A.err, kErrBadExpertId);
        }
        e.orow[lane] = o;
        if (lane == 0) {
          e.tile = it.tile, e.s0 = it.s0, e.ns = it.ns, e.nv = it.nv;
          e.mat = it.dst == A.out ? 0 : 1;
        }
        __syncwarp();  // the entry is published by lane 0's arrival on full[st]
        if (lane == 0) tc_tmap_acquire(it.map);
      }
      if (lane == 0) {
        const int units = it.nv / kTcUnit;
        // this CTA's half of the slice image (B rows N/2 * rank ..), all the block scales
        const uint32_t bhalf = units * kTcUnitBBytes / 2, xbytes = units * kTcUnitXFloats * 4;
        const size_t uoff = static_cast<size_t>(it.unit) * nchunks + static_cast<size_t>(chunk) * units;
        mbar_arrive_expect_tx(&sm.full[st], A.box_rows * kTcRawRow + bhalf + xbytes);
        tc_tma_2d(sm.raw[st], it.map, chunk * kTcRawRow, it.tile * 2 * kTcRows + row0, &sm.full[st]);
        tc_bulk(sm.b[st], A.bimg + uoff * kTcUnitBBytes + rank * bhalf, bhalf, &sm.full[st]);
        tc_bulk(sm.xs[st], A.ximg + uoff * kTcUnitXFloats, xbytes, &sm.full[st]);
      }
    }
  } else if (warp == kTcMmaWarp) {
    // the even CTA's whole warp walks the steps (warp-uniform operands); one
    // lane issues the pair's MMAs; the odd CTA's MMA warp has no steps
    if (rank != 0) goto tc_done;
    // Operand descriptors of block j of code buffer ab / image stage st: the
    // address field (bits 0-13, byte address >> 4; shared memory stays below
    // 256 KB, so no carry leaves it) of the buffer's base plus 16 per block.
    const uint64_t da0 = umma_desc_kmajor(smem_addr(sm.a[0]), 128, kTcKch * 128);
    const uint64_t db0 = umma_desc_kmajor(smem_addr(sm.b[0]), 128, kTcKch * 128);
    constexpr uint64_t kADesc = sizeof(sm.a[0]) >> 4, kBDesc = sizeof(sm.b[0]) >> 4;
    int st = 0, ab = 0, G = 0;  // image stage, code buffer, groups issued
    uint32_t apar = 0;          // a_full parity of buffer ab
    uint32_t idesc = 0;
    bool wide = false;
#pragma unroll 1
    for (int i = 0; i < my_items; ++i) {
#pragma unroll 1
      for (int c = 0; c < nchunks; ++c) {
        // One wait covers both CTAs' operands of the step: the unpack
        // threads of both arrive on this a_full after their own full[st]
        // wait (the slice-image halves landed, the item entry published)
        // and after fencing their code stores to the async proxy.
        if (!tc_spin_cluster_warp(&sm.a_full[ab], apar, A.err, &sm.abort)) goto tc_mma_out;
        tc_fence_after_sync();
        if (c == 0) {
          const int nv = sm.items[i % kTcItemRing].nv;
          idesc = umma_idesc_s8s8(2 * kTcRows, 3 * nv);
          wide = nv > kTcUnit;
        }
        const uint64_t da = da0 + ab * kADesc, db = db0 + st * kBDesc;
        if (wide) {  // two groups of 4 blocks, 128 columns each
#pragma unroll
          for (int h = 0; h < 2; ++h, ++G) {
            if (G > 0 && !tc_spin_cluster_warp(&sm.t_empty[0], (G - 1) & 1, A.err, &sm.abort)) goto tc_mma_out;
            tc_fence_after_sync();
#pragma unroll
            for (int jj = 0; jj < 4; ++jj)
              umma_i8_pair(tmem + jj * 128, da + 16 * (4 * h + jj), db + 16 * (4 * h + jj), idesc);
            umma_commit_pair(&sm.t_full[0]);
          }
        } else {  // one group of 8 blocks, 64 columns each
          if (G > 0 && !tc_spin_cluster_warp(&sm.t_empty[0], (G - 1) & 1, A.err, &sm.abort)) goto tc_mma_out;
          tc_fence_after_sync();
#pragma unroll
          for (int jj = 0; jj < 8; ++jj) umma_i8_pair(tmem + jj * 64, da + 16 * jj, db + 16 * jj, idesc);
          umma_commit_pair(&sm.t_full[0]);
          ++G;
        }
        umma_commit_pair(&sm.a_empty[ab]);
        umma_commit_pair(&sm.empty[st]);
        ab = ab == kTcAbuf - 1 ? 0 : ab + 1;
        apar ^= static_cast<uint32_t>(ab == 0);
        st = st == kTcStages - 1 ? 0 : st + 1;
      }
    }
  tc_mma_out:;
  } else if (warp < kTcEpiWarp0) {
    const int r = tid - 32 * kTcUnpackWarp0;
#pragma unroll 1
    for (int s = 0; s < nsteps; ++s) {
      const int st = s % kTcStages, ab = s % kTcAbuf, q = s % kTcQ;
      if (!tc_wait(&sm.full[st], (s / kTcStages) & 1, A.err, &sm.abort)) break;
      if (s >= kTcAbuf && !tc_wait(&sm.a_empty[ab], ((s / kTcAbuf) - 1) & 1, A.err, &sm.abort)) break;
      if (s >= kTcQ && !tc_wait(&sm.q_empty[q], ((s / kTcQ) - 1) & 1, A.err, &sm.abort)) break;
      tc_unpack(sm, st, ab, q, r);
      {  // the block scales: 2 of the step's 256 per thread
        static_assert(kTcKB * kTcNvp == 2 * kTcRows, "block scales per unpack thread");
        reinterpret_cast<float2*>(sm.q_xs[q])[r] = reinterpret_cast<const float2*>(sm.xs[st])[r];
      }
      fence_async_shared();  // codes written here, read by the MMAs
      mbar_arrive(&sm.a_full[ab]);
      __syncwarp();
      if (lane == 0) {
        mbar_arrive(&sm.q_full[q]);
        mbar_arrive(&sm.empty[st]);
        // the even CTA issues the MMAs that read these codes and this CTA's
        // slice-image half (landed: full[st] was waited above)
        if (rank != 0) mbar_arrive_cta(&sm.a_full[ab], 0);
      }
      __syncwarp();  // the warp unpacks the next step converged
    }
  } else {
    const int ew = warp - kTcEpiWarp0;
    const int quarter = warp & 3;  // tensor-memory lanes 32*quarter ..
    const int vset = ew >> 2;      // vectors vset * nv/4 ..
    const int trow = 32 * quarter + lane;
    const uint32_t lane_addr = static_cast<uint32_t>(32 * quarter) << 16;
    float acc[8];
#pragma unroll
    for (int i = 0; i < 8; ++i) acc[i] = 0.0f;
    int nv = kTcUnit, ns = 0, tile = 0, nvw = 4, v0 = 0, orow = -1, G = 0;
    float* dst = A.out;
    bool live = false;
#pragma unroll 1
    for (int s = 0; s < nsteps; ++s) {
      const int q = s % kTcQ, chunk = s % nchunks;
      // the step's block and row scales (copied and written by unpack) are
      // read below, and at an item's first step its entry
      bool ok = tc_wait(&sm.q_full[q], (s / kTcQ) & 1, A.err, &sm.abort);
      if (chunk == 0) {
        const TcItemSlot& e = sm.items[(s / nchunks) % kTcItemRing];
        nv = e.nv, ns = e.ns, tile = e.tile;
        dst = e.mat ? A.out2 : A.out;
        nvw = nv / 4;
        v0 = vset * nvw;
        live = v0 < ns;
        orow = live && lane < nvw ? e.orow[v0 + lane] : -1;  // this lane's vector's output row
      }
      const int gb = tc_group_blocks(nv);
#pragma unroll 1
      for (int j = 0; j < kTcKB && ok; j += gb, ++G) {
        const int slot = G % kTcSlots;
        if (!tc_wait(&sm.t_full[slot], (G / kTcSlots) & 1, A.err, &sm.abort)) {
          ok = false;
          break;
        }
        tc_fence_after_sync();
        if (live) {
          const uint32_t taddr = tmem + lane_addr + slot * kTcSlotCols + 3 * v0;
          const float* dcol = &sm.q_d[q][j][trow];
          const float* xsv = &sm.q_xs[q][j * nv + v0];
          if (nvw == 8)
            tc_epi_group<8, 4, 128>(taddr, nv, dcol, xsv, &sm.t_empty[slot], acc);
          else
            tc_epi_group<4, 8, 64>(taddr, nv, dcol, xsv, &sm.t_empty[slot], acc);
        } else {
          tc_fence_before_sync();
          __syncwarp();
          if (lane == 0) mbar_arrive_cta_relaxed(&sm.t_empty[slot], 0);
        }
      }
      if (!ok) break;
      __syncwarp();
      if (lane == 0) mbar_arrive(&sm.q_empty[q]);
      if (chunk == nchunks - 1) {
        const int grow = tile * 2 * kTcRows + row0 + trow;
        if (live) {
#pragma unroll
          for (int i = 0; i < 8; ++i) {
            const int o = __shfl_sync(0xFFFFFFFFu, orow, i);
            if (i < nvw && v0 + i < ns && o >= 0 && o < A.out_rows && grow < A.R)
              dst[static_cast<size_t>(o) * A.R + grow] = acc[i];
          }
        }
#pragma unroll
        for (int i = 0; i < 8; ++i) acc[i] = 0.0f;
      }
    }
  }
tc_done:
  tc_fence_before_sync();
  __syncthreads();
  cluster_sync_all();  // neither CTA leaves while the other may still read or arrive on its memory
  if (warp == kTcMmaWarp) {
    tc_fence_after_sync();
    tmem_dealloc_pair(tmem, kTcTmemCols);
  }
}


// ======================================================================
// The official DeepSeek FP8 x FP4 contraction on block-scaled MMAs.
// Weights are split FP4 E2M1 [R][C/2] with E8M0 scales per 32 columns;
// activations are act_quant output: E4M3 codes [nvec][C] with E8M0 scales per
// 128 columns.  tcgen05.mma.kind::mxf8f6f4.block_scale multiplies them
// directly: A = the weight tile (E2M1; under this kind a 16-value group sits
// in 16 bytes of shared memory: 8 packed bytes, then 8 bytes of padding),
// B = the slice's activation codes (E4M3), the UE8M0 scale factors of both
// in tensor memory (CUTLASS's K-major scale atom: 128 rows x 4 blocks in 512
// bytes, row m = m0 + 32 m1 at byte m0 * 16 + m1 * 4 + block, copied with
// tcgen05.cp 32x128b.warpx4).  The products are exact and the f32 sum of a
// whole row stays in tensor memory: one epilogue per work item, none per
// block.  Work item = (slice of up to 128 pairs of one expert, 128-row tile);
// a step is 128 columns (4 MMAs, one scale atom).
constexpr int kMxKB = 4;                           // 32-column blocks per step
constexpr int kMxStepCols = kMxKB * 32;            // 128
constexpr int kMxNvp = 128;                        // pairs per slice (at most)
constexpr int kMxRawRow = kMxStepCols / 2;         // packed FP4 bytes of one row per step
constexpr int kMxKch = kMxStepCols / 16;           // 16-byte K columns of a staged operand
constexpr int kMxStages = 6, kMxAbuf = 2, kMxDslots = 2;  // six steps in flight cover the DRAM latency
constexpr int kMxUnitBBytes = kTcUnit * kMxStepCols;  // 16 activation rows of one step
constexpr int kMxSfAtom = 512;
constexpr int kMxDCols = 128;                      // tensor-memory columns of one accumulator slot
constexpr int kMxSfaCol = 256, kMxSfbCol = 272;    // scale-factor columns (4 per buffer)
constexpr int kMxProducerWarp = 0, kMxMmaWarp = 1, kMxUnpackWarp0 = 2, kMxEpiWarp0 = 6, kMxEpiWarps = 4;
constexpr int kMxThreads = 32 * (kMxEpiWarp0 + kMxEpiWarps);

struct MxSmem {
  alignas(1024) uint8_t a[kMxAbuf][kTcRows * kMxStepCols];
  alignas(1024) uint8_t b[kMxStages][kMxNvp * kMxStepCols];
  alignas(128) uint8_t raw[kMxStages][kTcRows * kMxRawRow];
  alignas(128) uint8_t sfa[kMxAbuf][kMxSfAtom];
  alignas(128) uint8_t sfb[kMxStages][kMxSfAtom];
  alignas(8) uint64_t full[kMxStages], empty[kMxStages], a_full[kMxAbuf], a_empty[kMxAbuf];
  uint64_t d_full[kMxDslots], d_empty[kMxDslots];
  uint32_t tmem_base;
  uint32_t abort;  // a wait of this CTA timed out
};
static_assert(sizeof(MxSmem) <= 227 * 1024, "block-scaled kernel shared memory");
static_assert(kMxDslots * kMxDCols <= kMxSfaCol && kMxSfbCol + 4 * kMxStages <= 512, "tensor-memory columns");

// Block-scaled instruction descriptor: A E2M1, B E4M3, UE8M0 scales, M 128,
// K 32; scale-factor byte `kb` of both operands.
__device__ __forceinline__ uint32_t mx_idesc(int n, int kb) {
  return (static_cast<uint32_t>(kb) << 4) | (5u << 7) | (0u << 10) | ((static_cast<uint32_t>(n) >> 3) << 17) |
         (1u << 23) | ((static_cast<uint32_t>(kTcRows) >> 4) << 24) | (static_cast<uint32_t>(kb) << 29);
}
__device__ __forceinline__ void umma_mx(uint32_t d_tmem, uint64_t a_desc, uint64_t b_desc, uint32_t idesc,
                                        uint32_t sfa_tmem, uint32_t sfb_tmem, bool accumulate) {
  asm volatile(
      "{\n\t.reg .pred p, e;\n\telect.sync _|e, 0xffffffff;\n\tsetp.ne.b32 p, %4, 0;\n\t"
      "@e tcgen05.mma.cta_group::1.kind::mxf8f6f4.block_scale [%0], %1, %2, %3, [%5], [%6], p;\n\t}\n" ::"r"(d_tmem),
      "l"(a_desc), "l"(b_desc), "r"(idesc), "r"(accumulate ? 1u : 0u), "r"(sfa_tmem), "r"(sfb_tmem));
}
// 32 rows x 16 bytes of shared memory -> 4 tensor-memory columns of every lane
// quarter (a converged warp executes it; the elected lane issues).
__device__ __forceinline__ void tmem_cp_sf(uint32_t taddr, const void* smem_atom) {
  asm volatile("{\n\t.reg .pred e;\n\telect.sync _|e, 0xffffffff;\n\t"
               "@e tcgen05.cp.cta_group::1.32x128b.warpx4 [%0], %1;\n\t}" ::"r"(taddr),
               "l"(umma_desc_kmajor(smem_addr(smem_atom), 128, 128)));
}

// Slice images of the block-scaled path: for slice sl, step c, the B rows i
// (activation codes of the slice's vector i; zero past the slice's length)
// in core-matrix order, nv = 16 * ceil(len / 16) rows, and the B scale atom
// (vector i's E8M0 scale of the step's 128 columns in all four blocks).
__global__ void __launch_bounds__(256) mx_image_kernel(const int32_t* __restrict__ slice_start,
                                                       const int32_t* __restrict__ slice_len,
                                                       const int32_t* __restrict__ slice_unit,
                                                       const int32_t* __restrict__ nslices,
                                                       const uint8_t* __restrict__ codes,
                                                       const uint8_t* __restrict__ scales,
                                                       const int32_t* __restrict__ slot_vec, int nvec, int C,
                                                       uint8_t* __restrict__ bimg, uint8_t* __restrict__ sfimg) {
  asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
  asm volatile("griddepcontrol.wait;" ::: "memory");
  const int nchunks = C / kMxStepCols;
  const int total = *nslices * nchunks;
  for (int w = blockIdx.x; w < total; w += gridDim.x) {
    const int sl = w / nchunks, c = w % nchunks;
    const int s0 = slice_start[sl], ns = min(slice_len[sl], kMxNvp);
    const int units = (ns + kTcUnit - 1) / kTcUnit, nv = units * kTcUnit;
    uint8_t* bdst = bimg + (static_cast<size_t>(slice_unit[sl]) * nchunks + static_cast<size_t>(c) * units) * kMxUnitBBytes;
    for (int q = threadIdx.x; q < nv * kMxKch; q += blockDim.x) {
      const int cm = q >> 3, r = q & 7;  // core matrix (row group, K column), row within it
      const int row = 8 * (cm / kMxKch) + r, p = cm % kMxKch;
      uint4 val = make_uint4(0u, 0u, 0u, 0u);
      if (row < ns) {
        int v = slot_vec ? slot_vec[s0 + row] : s0 + row;
        v = (v < 0 || v >= nvec) ? 0 : v;
        val = *reinterpret_cast<const uint4*>(codes + static_cast<size_t>(v) * C + c * kMxStepCols + p * 16);
      }
      *reinterpret_cast<uint4*>(bdst + static_cast<size_t>(q) * 16) = val;
    }
    uint32_t* sdst = reinterpret_cast<uint32_t*>(sfimg + (static_cast<size_t>(sl) * nchunks + c) * kMxSfAtom);
    for (int q = threadIdx.x; q < kMxSfAtom / 4; q += blockDim.x) {
      // word q = row (q / 4) % 32 + 32 * (q % 4), all four blocks
      const int row = (q >> 2) + 32 * (q & 3);
      uint32_t val = 0u;
      if (row < ns) {
        int v = slot_vec ? slot_vec[s0 + row] : s0 + row;
        v = (v < 0 || v >= nvec) ? 0 : v;
        val = static_cast<uint32_t>(scales[static_cast<size_t>(v) * (C / 128) + c]) * 0x01010101u;
      }
      sdst[q] = val;
    }
  }
}

// SwiGLU of the official path (only the up value clamped, deepseek.rs:1707-1711)
// over the pairs' gate / up rows, in place into the gate rows.
__global__ void __launch_bounds__(256) mx_swiglu_kernel(float* __restrict__ g, const float* __restrict__ u, size_t n,
                                                        const int32_t* count, int I, float limit) {
  asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
  asm volatile("griddepcontrol.wait;" ::: "memory");
  if (count) n = min(n, static_cast<size_t>(max(*count, 0)) * I);
  for (size_t i = blockIdx.x * static_cast<size_t>(blockDim.x) + threadIdx.x; i < n;
       i += static_cast<size_t>(gridDim.x) * blockDim.x)
    g[i] = swiglu(g[i], u[i], limit, false);
}

struct MxArgs {
  const uint8_t* const* W;    // packed E2M1 weights [R][C/2]
  const uint8_t* const* WS;   // E8M0 scales [R][C/32]
  const uint8_t* const* W2;   // second matrix (gate + up in one launch), or null
  const uint8_t* const* WS2;
  int num_experts, R, C;
  const int32_t* pe;
  const int32_t* slot_vec;
  const int32_t* slot_out;
  const int32_t* slice_start;
  const int32_t* slice_len;
  const int32_t* slice_unit;
  const int32_t* nslices;
  const int32_t* slice_order;  // slices widest first (tc_slices_kernel)
  const uint8_t* bimg;
  const uint8_t* sfimg;
  const CUtensorMap* maps;   // tensor maps of every slice's weight matrices (tc_maps_kernel): [slice][gate, up, down]
  int map0;                  // 0: gate (+ up), 2: down
  int box_rows;
  int nvec;
  float* out;
  float* out2;
  int out_rows;
  unsigned* err;
};

struct MxItem {
  const CUtensorMap* map;
  const uint8_t* ws;
  float* dst;
  int tile, s0, ns, units, unit, sl;
};

// Item o of the launch's ordered list (slices widest first; tile, matrix
// within a slice, the matrix fastest).
__device__ __forceinline__ MxItem mx_item(const MxArgs& A, int o, int tiles, int mats) {
  MxItem it;
  const int mat = o % mats, rest = o / mats;
  it.sl = A.slice_order[rest / tiles];
  it.tile = rest % tiles;
  it.s0 = A.slice_start[it.sl];
  it.ns = min(max(A.slice_len[it.sl], 1), kMxNvp);
  it.units = (it.ns + kTcUnit - 1) / kTcUnit;
  it.unit = A.slice_unit[it.sl];
  int e = A.pe[it.s0];
  if (e < 0 || e >= A.num_experts) e = 0;  // flagged by the epilogue
  it.map = A.maps + 3 * it.sl + A.map0 + mat;
  it.ws = mat ? A.WS2[e] : A.WS[e];
  it.dst = mat ? A.out2 : A.out;
  return it;
}

__global__ void __launch_bounds__(kMxThreads, 1) mx_grouped_kernel(const MxArgs A) {
  extern __shared__ __align__(1024) uint8_t mx_smem_raw[];
  MxSmem& sm = *reinterpret_cast<MxSmem*>(mx_smem_raw);
  asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  if (tid == 0) {
    for (int i = 0; i < kMxStages; ++i) {
      mbar_init(&sm.full[i], 1);
      mbar_init(&sm.empty[i], 1 + kTcUnpackWarps);
    }
    for (int i = 0; i < kMxAbuf; ++i) {
      mbar_init(&sm.a_full[i], 32 * kTcUnpackWarps);
      mbar_init(&sm.a_empty[i], 1);
    }
    for (int i = 0; i < kMxDslots; ++i) {
      mbar_init(&sm.d_full[i], 1);
      mbar_init(&sm.d_empty[i], kMxEpiWarps);
    }
    sm.abort = 0u;
    fence_mbar_init();
  }
  if (warp == kMxMmaWarp) tmem_alloc(&sm.tmem_base, kTcTmemCols);
  __syncthreads();
  tc_fence_after_sync();
  const uint32_t tmem = sm.tmem_base;
  asm volatile("griddepcontrol.wait;" ::: "memory");

  const int nchunks = A.C / kMxStepCols;
  const int tiles = (A.R + kTcRows - 1) / kTcRows;
  const int mats = A.W2 ? 2 : 1;
  // Items widest first, dealt in snake order (round r goes over the CTAs
  // forward when r is even, backward when odd), so each CTA's share of the
  // costly wide items and of the cheap narrow ones evens out.
  const int total = *A.nslices * tiles * mats, G = static_cast<int>(gridDim.x), cta = static_cast<int>(blockIdx.x);
  auto item_o = [&](int r) { return r * G + ((r & 1) ? G - 1 - cta : cta); };
  const int rounds = (total + G - 1) / G;
  const int my_items = rounds > 0 && item_o(rounds - 1) >= total ? rounds - 1 : rounds;
  const int nsteps = my_items * nchunks;
  auto item_at = [&](int s) { return mx_item(A, item_o(s / nchunks), tiles, mats); };

  if (warp == kMxProducerWarp) {
    if (lane == 0) {
      MxItem it{};
#pragma unroll 1
      for (int s = 0; s < nsteps; ++s) {
        const int st = s % kMxStages, chunk = s % nchunks;
        if (chunk == 0) {
          it = item_at(s);
          tc_tmap_acquire(it.map);
        }
        if (s >= kMxStages && !tc_wait(&sm.empty[st], ((s / kMxStages) - 1) & 1, A.err, &sm.abort)) break;
        const uint32_t bbytes = it.units * kMxUnitBBytes;
        const size_t uoff = static_cast<size_t>(it.unit) * nchunks + static_cast<size_t>(chunk) * it.units;
        mbar_arrive_expect_tx(&sm.full[st], A.box_rows * kMxRawRow + bbytes + kMxSfAtom);
        tc_tma_2d(sm.raw[st], it.map, chunk * kMxRawRow, it.tile * kTcRows, &sm.full[st]);
        tc_bulk(sm.b[st], A.bimg + uoff * kMxUnitBBytes, bbytes, &sm.full[st]);
        tc_bulk(sm.sfb[st], A.sfimg + (static_cast<size_t>(it.sl) * nchunks + chunk) * kMxSfAtom, kMxSfAtom,
                &sm.full[st]);
      }
    }
  } else if (warp == kMxMmaWarp) {
    // the whole warp walks the steps (warp-uniform operands); one lane issues
    int n = kTcUnit, item = -1, slot = 0;
#pragma unroll 1
    for (int s = 0; s < nsteps; ++s) {
      const int st = s % kMxStages, ab = s % kMxAbuf, chunk = s % nchunks;
      if (chunk == 0) {
        n = item_at(s).units * kTcUnit;
        ++item;
        slot = item % kMxDslots;
        if (item >= kMxDslots && !tc_spin_warp(&sm.d_empty[slot], ((item / kMxDslots) - 1) & 1, A.err, &sm.abort)) break;
      }
      if (!tc_spin_warp(&sm.a_full[ab], (s / kMxAbuf) & 1, A.err, &sm.abort) || !tc_spin_warp(&sm.full[st], (s / kMxStages) & 1, A.err, &sm.abort))
        break;
      fence_async_shared();  // codes and weight scales written by the unpack threads
      tc_fence_after_sync();
      const uint32_t t_sfa = tmem + kMxSfaCol + 4 * ab, t_sfb = tmem + kMxSfbCol + 4 * st;
      tmem_cp_sf(t_sfa, sm.sfa[ab]);
      tmem_cp_sf(t_sfb, sm.sfb[st]);
#pragma unroll
      for (int kb = 0; kb < kMxKB; ++kb) {
        const uint64_t da = umma_desc_kmajor(smem_addr(sm.a[ab] + 2 * kb * 128), 128, kMxKch * 128);
        const uint64_t db = umma_desc_kmajor(smem_addr(sm.b[st] + 2 * kb * 128), 128, kMxKch * 128);
        umma_mx(tmem + slot * kMxDCols, da, db, mx_idesc(n, kb), t_sfa, t_sfb, chunk > 0 || kb > 0);
      }
      umma_commit(&sm.a_empty[ab]);
      umma_commit(&sm.empty[st]);
      if (chunk == nchunks - 1) umma_commit(&sm.d_full[slot]);
    }
  } else if (warp < kMxEpiWarp0) {
    const int r = tid - 32 * kMxUnpackWarp0;
    MxItem it{};
#pragma unroll 1
    for (int s = 0; s < nsteps; ++s) {
      const int st = s % kMxStages, ab = s % kMxAbuf, chunk = s % nchunks;
      if (chunk == 0) it = item_at(s);
      const int row = it.tile * kTcRows + r;
      // this row's four E8M0 block scales of the step (rows past the matrix: 2^-127, zero weights)
      const uint32_t wsc = row < A.R ? *reinterpret_cast<const uint32_t*>(
                                           it.ws + static_cast<size_t>(row) * (A.C / 32) + chunk * kMxKB)
                                     : 0u;
      if (!tc_wait(&sm.full[st], (s / kMxStages) & 1, A.err, &sm.abort)) break;
      if (s >= kMxAbuf && !tc_wait(&sm.a_empty[ab], ((s / kMxAbuf) - 1) & 1, A.err, &sm.abort)) break;
      const uint8_t* src = sm.raw[st] + r * kMxRawRow;
      uint8_t* dst = sm.a[ab] + (r >> 3) * kMxKch * 128 + (r & 7) * 16;
#pragma unroll
      for (int q = 0; q < kMxRawRow / 16; ++q) {
        const uint4 x = *reinterpret_cast<const uint4*>(src + 16 * q);
        // 16 values = 8 packed bytes, then 8 bytes of padding
        *reinterpret_cast<uint4*>(dst + (2 * q) * 128) = make_uint4(x.x, x.y, 0u, 0u);
        *reinterpret_cast<uint4*>(dst + (2 * q + 1) * 128) = make_uint4(x.z, x.w, 0u, 0u);
      }
      *reinterpret_cast<uint32_t*>(sm.sfa[ab] + (r & 31) * 16 + (r >> 5) * 4) = wsc;
      fence_async_shared();  // read by the MMAs and the scale copy
      mbar_arrive(&sm.a_full[ab]);
      __syncwarp();
      if (lane == 0) mbar_arrive(&sm.empty[st]);
    }
  } else {
    const int quarter = warp & 3;
    const int trow = 32 * quarter + lane;
    const uint32_t lane_addr = static_cast<uint32_t>(32 * quarter) << 16;
#pragma unroll 1
    for (int i = 0; i < my_items; ++i) {
      const MxItem it = item_at(i * nchunks);
      const int slot = i % kMxDslots;
      if (!tc_wait(&sm.d_full[slot], (i / kMxDslots) & 1, A.err, &sm.abort)) break;
      tc_fence_after_sync();
      const int grow = it.tile * kTcRows + trow;
#pragma unroll 1
      for (int c0 = 0; c0 < it.units * kTcUnit; c0 += 16) {
        uint32_t rv[16];
        tmem_ld16(tmem + lane_addr + slot * kMxDCols + c0, rv);
        tmem_wait_ld();
#pragma unroll
        for (int j = 0; j < 16; ++j) {
          const int vi = c0 + j;
          if (vi < it.ns && grow < A.R) {
            const int p = it.s0 + vi;
            const int o = A.slot_out ? A.slot_out[p] : p;
            if (o >= 0 && o < A.out_rows) it.dst[static_cast<size_t>(o) * A.R + grow] = __uint_as_float(rv[j]);
          }
        }
      }
      if (quarter == 0) {
        for (int vi = lane; vi < it.ns; vi += 32) {
          const int p = it.s0 + vi;
          const int o = A.slot_out ? A.slot_out[p] : p;
          const int v = A.slot_vec ? A.slot_vec[p] : p;
          const int e = A.pe[p];
          if ((o < 0 || o >= A.out_rows || v < 0 || v >= A.nvec || e < 0 || e >= A.num_experts) && A.err)
            atomicOr(A.err, kErrBadExpertId);
        }
      }
      tc_fence_before_sync();
      __syncwarp();
      if (lane == 0) mbar_arrive(&sm.d_empty[slot]);
    }
  }
  tc_fence_before_sync();
  __syncthreads();
  if (warp == kMxMmaWarp) {
    tc_fence_after_sync();
    tmem_dealloc(tmem, kTcTmemCols);
  }
}

}  // namespace dev

namespace {

struct TcLayout {
  size_t planes_x, xsc_x, wflag_x, wflag_a, wany_x, wany_a, g, u, planes_a, xsc_a, run_start, slice_start, slice_len, slice_unit,
      slice_order, nslices, bimg, ximg, maps, total;
};

size_t align256(size_t b) { return (b + 255) / 256 * 256; }

// Slice-image units (16 vectors) a pair list grouped by expert can need:
// slices are runs cut at 32 pairs, so sum ceil(len / 16) <= P / 16 + slices
// and slices <= P / 32 + runs, runs <= distinct experts.  (A list that is not
// grouped may need more; the slices kernel then runs nothing and flags it.)
size_t tc_max_units(size_t P, size_t E) { return 3 * P / 32 + std::min(P, E) + 2; }

TcLayout tc_layout(size_t P, size_t T, size_t H, size_t I, size_t E, int sm_count) {
  TcLayout L;
  size_t off = 0;
  auto take = [&](size_t bytes) {
    const size_t at = off;
    off += align256(bytes);
    return at;
  };
  const size_t units = tc_max_units(P, E), nchunks = std::max(H, I) / (dev::kTcKB * 32);
  L.planes_x = take(T * 3 * H);
  L.xsc_x = take(T * (H / 32) * 4);
  L.wflag_x = take(T * (H / 32));
  L.wflag_a = take(P * (I / 32));
  L.wany_x = take(T);
  L.wany_a = take(P);
  L.g = take(P * I * 4);
  L.u = take(P * I * 4);
  L.planes_a = take(P * 3 * I);
  L.xsc_a = take(P * (I / 32) * 4);
  L.run_start = take(P * 4);
  L.slice_start = take(P * 4);
  L.slice_len = take(P * 4);
  L.slice_unit = take(P * 4);
  L.slice_order = take(P * 4);
  L.nslices = take(8);
  L.bimg = take(units * nchunks * dev::kTcUnitBBytes);
  L.ximg = take(units * nchunks * dev::kTcUnitXFloats * 4);
  L.maps = take(3 * units * sizeof(CUtensorMap));  // slices <= units
  L.total = off;
  return L;
}

int validate_tc(const objb_moe_layer* l, size_t num_pairs, size_t num_tokens) {
  if (!l) return OBJB_FAIL(OBJB_ERR_INVALID_INPUT, "grouped Q4_0 MoE pairs", "null layer");
  if (l->fmt != OBJB_Q4_0 || l->d_gate_scale || l->d_up_scale || l->d_down_scale)
    return OBJB_FAIL(OBJB_ERR_UNSUPPORTED, "grouped Q4_0 MoE pairs", "the tensor-core pair path takes Q4_0 experts");
  if ((l->flags & OBJB_MOE_UNALIGNED) != 0)
    return OBJB_FAIL(OBJB_ERR_UNSUPPORTED, "grouped Q4_0 MoE pairs", "expert tensors must be 16-byte aligned");
  if (!l->d_gate || !l->d_up || !l->d_down || l->num_experts == 0 || l->num_experts > (1u << 20))
    return OBJB_FAIL(OBJB_ERR_INVALID_INPUT, "grouped Q4_0 MoE pairs", "missing expert tables");
  if (l->hidden == 0 || l->intermediate == 0 || l->out_dim == 0 || l->hidden > (1u << 20) ||
      l->intermediate > (1u << 20) || l->out_dim > (1u << 20))
    return OBJB_FAIL(OBJB_ERR_INVALID_INPUT, "grouped Q4_0 MoE pairs", "shape out of range");
  if (l->hidden % 256 || l->intermediate % 256)
    return OBJB_FAIL(OBJB_ERR_UNSUPPORTED, "grouped Q4_0 MoE pairs",
                     "hidden and intermediate must be multiples of 256 (rows staged in 16-byte pieces)");
  if (num_pairs == 0 || num_pairs > (1u << 20) || num_tokens == 0 || num_tokens > (1u << 20))
    return OBJB_FAIL(OBJB_ERR_INVALID_INPUT, "grouped Q4_0 MoE pairs", "need 1 <= num_pairs, num_tokens <= 2^20");
  if (num_pairs * std::max(l->intermediate, l->out_dim) > (1u << 30) || num_tokens * l->hidden > (1ull << 34))
    return OBJB_FAIL(OBJB_ERR_INVALID_INPUT, "grouped Q4_0 MoE pairs", "num_pairs * rows too large");
  return OBJB_OK;
}

// cuTensorMapEncodeTiled through the runtime's driver entry point (no link
// against the driver library).
int tc_encode_tiled(CUtensorMap* map, void* base, size_t row_bytes, size_t rows, int box_rows,
                    int box_inner = dev::kTcRawRow) {
  static PFN_cuTensorMapEncodeTiled_v12000 fn = nullptr;
  static std::once_flag once;
  std::call_once(once, [] {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q = cudaDriverEntryPointSymbolNotFound;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(p);
  });
  if (!fn) return OBJB_FAIL(OBJB_ERR_DRIVER, "grouped Q4_0 MoE pairs", "cuTensorMapEncodeTiled is not available");
  const cuuint64_t dims[2] = {static_cast<cuuint64_t>(row_bytes), static_cast<cuuint64_t>(rows)};
  const cuuint64_t strides[1] = {static_cast<cuuint64_t>(row_bytes)};
  const cuuint32_t box[2] = {static_cast<cuuint32_t>(box_inner), static_cast<cuuint32_t>(box_rows)};
  const cuuint32_t estr[2] = {1, 1};
  const CUresult r = fn(map, CU_TENSOR_MAP_DATA_TYPE_UINT8, 2, base, dims, strides, box, estr,
                        CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_NONE, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                        CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS)
    return OBJB_FAIL(OBJB_ERR_DRIVER, "grouped Q4_0 MoE pairs", "cuTensorMapEncodeTiled failed (" + std::to_string(r) + ")");
  return OBJB_OK;
}

}  // namespace

bool moe_pairs_tc_supported(const objb_moe_layer* l) {
  return l && l->fmt == OBJB_Q4_0 && !l->d_gate_scale && (l->flags & OBJB_MOE_UNALIGNED) == 0 &&
         l->hidden % 256 == 0 && l->intermediate % 256 == 0;
}

int moe_pairs_tc_scratch_bytes(const objb_moe_layer* l, size_t num_pairs, size_t num_tokens, size_t* out) {
  OBJB_TRY(validate_tc(l, num_pairs, num_tokens));
  int device = 0;
  OBJB_TRY(current_device(&device));
  DeviceProps props;
  OBJB_TRY(device_props(device, &props));
  *out = tc_layout(num_pairs, num_tokens, l->hidden, l->intermediate, l->num_experts, props.sm_count).total;
  return OBJB_OK;
}

// The multi-token pairs of moe_pairs for Q4_0 layers on the tensor cores:
// slices of the expert-sorted pair list, digit planes of the T token vectors
// and their slice images, gate and up of every pair in one grouped launch,
// SwiGLU straight into the digit planes of the P activations, their slice
// images, and down into v[pair_out[p]] (or v[p]).
int moe_pairs_tc(const objb_moe_layer* l, size_t num_pairs, const int32_t* pe, const int32_t* pt, const int32_t* po,
                 size_t num_tokens, const float* x, float* v, size_t v_rows, float limit, cudaStream_t stream,
                 void* scratch, size_t scratch_bytes, unsigned* err_word, const int32_t* d_count) {
  OBJB_TRY(validate_tc(l, num_pairs, num_tokens));
  if (!pe || !pt || !x || !v || !scratch)
    return OBJB_FAIL(OBJB_ERR_INVALID_INPUT, "grouped Q4_0 MoE pairs", "null device pointer");
  if (v_rows < (po ? 1 : num_pairs) || v_rows > (1u << 30))
    return OBJB_FAIL(OBJB_ERR_INVALID_INPUT, "grouped Q4_0 MoE pairs", "v_rows cannot hold the pair outputs");
  int device = 0;
  OBJB_TRY(current_device(&device));
  DeviceProps props;
  OBJB_TRY(device_props(device, &props));
  const TcLayout L = tc_layout(num_pairs, num_tokens, l->hidden, l->intermediate, l->num_experts, props.sm_count);
  if (scratch_bytes < L.total)
    return OBJB_FAIL(OBJB_ERR_INVALID_INPUT, "grouped Q4_0 MoE pairs",
                     "scratch of " + std::to_string(scratch_bytes) + " bytes < needed " + std::to_string(L.total));
  unsigned* err = err_word;
  if (!err) OBJB_TRY(device_error_word(device, &err));
  uint8_t* sc = static_cast<uint8_t*>(scratch);
  int8_t* planes_x = reinterpret_cast<int8_t*>(sc + L.planes_x);
  float* xsc_x = reinterpret_cast<float*>(sc + L.xsc_x);
  uint8_t* wflag_x = sc + L.wflag_x;
  uint8_t* wflag_a = sc + L.wflag_a;
  uint8_t* wany_x = sc + L.wany_x;
  uint8_t* wany_a = sc + L.wany_a;
  float* g = reinterpret_cast<float*>(sc + L.g);
  float* u = reinterpret_cast<float*>(sc + L.u);
  int8_t* planes_a = reinterpret_cast<int8_t*>(sc + L.planes_a);
  float* xsc_a = reinterpret_cast<float*>(sc + L.xsc_a);
  int32_t* run_start = reinterpret_cast<int32_t*>(sc + L.run_start);
  int32_t* slice_start = reinterpret_cast<int32_t*>(sc + L.slice_start);
  int32_t* slice_len = reinterpret_cast<int32_t*>(sc + L.slice_len);
  int32_t* slice_unit = reinterpret_cast<int32_t*>(sc + L.slice_unit);
  int32_t* slice_order = reinterpret_cast<int32_t*>(sc + L.slice_order);
  int32_t* nslices = reinterpret_cast<int32_t*>(sc + L.nslices);
  uint8_t* bimg = sc + L.bimg;
  float* ximg = reinterpret_cast<float*>(sc + L.ximg);
  CUtensorMap* maps = reinterpret_cast<CUtensorMap*>(sc + L.maps);
  const int P = static_cast<int>(num_pairs), T = static_cast<int>(num_tokens);
  const int H = static_cast<int>(l->hidden), I = static_cast<int>(l->intermediate), O = static_cast<int>(l->out_dim);
  auto warp_grid = [&](int nvec, int C) {
    const long long warps = static_cast<long long>(nvec) * (C / 32);
    return static_cast<int>(std::max(1LL, std::min((warps * 32 + 255) / 256, 16LL * props.sm_count)));
  };
  const size_t row_gu = static_cast<size_t>(H / 32) * 18, row_dn = static_cast<size_t>(I / 32) * 18;
  CUtensorMap tm_gu, tm_dn;
  OBJB_TRY(tc_encode_tiled(&tm_gu, scratch, row_gu, static_cast<size_t>(I), std::min(dev::kTcRows, I)));
  OBJB_TRY(tc_encode_tiled(&tm_dn, scratch, row_dn, static_cast<size_t>(O), std::min(dev::kTcRows, O)));
  const int max_slices = static_cast<int>(tc_max_units(num_pairs, l->num_experts));
  const size_t smem = sizeof(dev::TcSmem);
  OBJB_TRY(ensure_smem_attr(dev::tc_q4_grouped_kernel, device, smem));
  const int img_grid = 4 * props.sm_count;

  OBJB_TRY(launch_pdl(dev::tc_slices_kernel, 1, 1024, 0, stream, pe, P, d_count, dev::kTcNvp, dev::kTcUnit, run_start,
                      slice_start, slice_len, slice_unit, nslices,
                      static_cast<int>(tc_max_units(num_pairs, l->num_experts)), err, wany_x, T, wany_a, slice_order));
  OBJB_TRY(launch_pdl(dev::tc_maps_kernel, std::max(1, (3 * max_slices + 255) / 256), 256, 0, stream, tm_gu, tm_dn,
                      static_cast<const int32_t*>(slice_start), static_cast<const int32_t*>(nslices), max_slices, pe,
                      reinterpret_cast<const uint8_t* const*>(l->d_gate),
                      reinterpret_cast<const uint8_t* const*>(l->d_up),
                      reinterpret_cast<const uint8_t* const*>(l->d_down), static_cast<int>(l->num_experts), maps));
  OBJB_TRY(launch_pdl(dev::tc_planes_kernel, warp_grid(T, H), 256, 0, stream, x, static_cast<size_t>(H), T,
                      static_cast<const int32_t*>(nullptr), H, planes_x, xsc_x, wflag_x, wany_x));
  OBJB_TRY(launch_pdl(dev::tc_image_kernel, img_grid, 256, 0, stream, static_cast<const int32_t*>(slice_start),
                      static_cast<const int32_t*>(slice_len), static_cast<const int32_t*>(slice_unit),
                      static_cast<const int32_t*>(nslices), static_cast<const int8_t*>(planes_x),
                      static_cast<const float*>(xsc_x), pt, T, H, bimg, ximg));
  dev::TcArgs a{};
  a.W = reinterpret_cast<const uint8_t* const*>(l->d_gate);
  a.W2 = reinterpret_cast<const uint8_t* const*>(l->d_up);
  a.num_experts = static_cast<int>(l->num_experts);
  a.R = I;
  a.C = H;
  a.pe = pe;
  a.slot_vec = pt;
  a.slot_out = nullptr;
  a.slice_start = slice_start;
  a.slice_len = slice_len;
  a.slice_unit = slice_unit;
  a.nslices = nslices;
  a.slice_order = slice_order;
  a.bimg = bimg;
  a.ximg = ximg;
  a.maps = maps;
  a.map0 = 0;
  a.box_rows = std::min(dev::kTcRows, I);
  a.nvec = T;
  a.out = g;
  a.out2 = u;
  a.out_rows = P;
  a.err = err;
  OBJB_TRY(launch_pdl(dev::tc_q4_grouped_kernel, props.sm_count / 2 * 2, dev::kTcThreads, smem, stream, a));
  OBJB_TRY(launch_pdl(dev::tc_swiglu_planes_kernel, warp_grid(P, I), 256, 0, stream, g,
                      static_cast<const float*>(u), P, d_count, I, limit, planes_a, xsc_a, wflag_a, wany_a, pe, pt, T,
                      x, H, static_cast<const uint8_t*>(wflag_x), static_cast<const uint8_t*>(wany_x), a.W, a.W2,
                      a.num_experts));
  OBJB_TRY(launch_pdl(dev::tc_image_kernel, img_grid, 256, 0, stream, static_cast<const int32_t*>(slice_start),
                      static_cast<const int32_t*>(slice_len), static_cast<const int32_t*>(slice_unit),
                      static_cast<const int32_t*>(nslices), static_cast<const int8_t*>(planes_a),
                      static_cast<const float*>(xsc_a), static_cast<const int32_t*>(nullptr), P, I, bimg, ximg));
  a.W = reinterpret_cast<const uint8_t* const*>(l->d_down);
  a.W2 = nullptr;
  a.R = O;
  a.C = I;
  a.map0 = 2;
  a.box_rows = std::min(dev::kTcRows, O);
  a.slot_vec = nullptr;
  a.slot_out = po;
  a.nvec = P;
  a.out = v;
  a.out2 = nullptr;
  a.out_rows = static_cast<int>(v_rows);
  OBJB_TRY(launch_pdl(dev::tc_q4_grouped_kernel, props.sm_count / 2 * 2, dev::kTcThreads, smem, stream, a));
  OBJB_TRY(launch_pdl(dev::tc_wide_down_kernel, warp_grid(P, 32), 256, 0, stream,
                      static_cast<const float*>(g), P, d_count, I, O, static_cast<const uint8_t*>(wflag_a),
                      static_cast<const uint8_t*>(wany_a), pe, po,
                      static_cast<int>(v_rows), a.W, a.num_experts, static_cast<const int32_t*>(nslices), v));
  return OBJB_OK;
}


// ---------------------------------------------------------------- official FP8 x FP4 pairs (block-scaled)
namespace {

struct MxLayout {
  size_t codes_x, scales_x, g, u, codes_a, scales_a, run_start, slice_start, slice_len, slice_unit, slice_order, nslices,
      bimg, sfimg, maps, total;
};

// Image units (16 vectors) of a pair list grouped by expert: sum ceil(len / 16)
// <= P / 16 + slices, slices <= P / 128 + distinct experts.  The scale atoms
// are sized by units too (every slice has at least one unit).
size_t mx_max_units(size_t P, size_t E) { return P / 16 + P / 128 + std::min(P, E) + 2; }

MxLayout mx_layout(size_t P, size_t T, size_t H, size_t I, size_t E, int sm_count) {
  MxLayout L;
  size_t off = 0;
  auto take = [&](size_t bytes) {
    const size_t at = off;
    off += align256(bytes);
    return at;
  };
  const size_t units = mx_max_units(P, E), nchunks = std::max(H, I) / dev::kMxStepCols;
  L.codes_x = take(T * H);
  L.scales_x = take(T * (H / 128));
  L.g = take(P * I * 4);
  L.u = take(P * I * 4);
  L.codes_a = take(P * I);
  L.scales_a = take(P * (I / 128));
  L.run_start = take(P * 4);
  L.slice_start = take(P * 4);
  L.slice_len = take(P * 4);
  L.slice_unit = take(P * 4);
  L.slice_order = take(P * 4);
  L.nslices = take(8);
  L.bimg = take(units * nchunks * dev::kMxUnitBBytes);
  L.sfimg = take(units * nchunks * dev::kMxSfAtom);
  L.maps = take(3 * mx_max_units(P, E) * sizeof(CUtensorMap));  // slices <= units
  L.total = off;
  return L;
}

int validate_mx(const objb_moe_layer* l, size_t num_pairs, size_t num_tokens) {
  const char* act = "official FP8 x FP4 MoE pairs";
  if (!l) return OBJB_FAIL(OBJB_ERR_INVALID_INPUT, act, "null layer");
  if (l->fmt != OBJB_FP4_E2M1 || !l->d_gate_scale || !l->d_up_scale || !l->d_down_scale)
    return OBJB_FAIL(OBJB_ERR_UNSUPPORTED, act, "needs a split FP4 E2M1 layer (weights + E8M0 scale tables)");
  if ((l->flags & OBJB_MOE_UNALIGNED) != 0)
    return OBJB_FAIL(OBJB_ERR_UNSUPPORTED, act, "expert tensors must be 16-byte aligned");
  if (!l->d_gate || !l->d_up || !l->d_down || l->num_experts == 0 || l->num_experts > (1u << 20))
    return OBJB_FAIL(OBJB_ERR_INVALID_INPUT, act, "missing expert tables");
  if (l->hidden == 0 || l->intermediate == 0 || l->out_dim == 0 || l->hidden > (1u << 20) ||
      l->intermediate > (1u << 20) || l->out_dim > (1u << 20))
    return OBJB_FAIL(OBJB_ERR_INVALID_INPUT, act, "shape out of range");
  if (l->hidden % 128 || l->intermediate % 128)
    return OBJB_FAIL(OBJB_ERR_INVALID_INPUT, act, "hidden and intermediate must be multiples of 128 (act_quant blocks)");
  if (num_pairs == 0 || num_pairs > (1u << 20) || num_tokens == 0 || num_tokens > (1u << 20))
    return OBJB_FAIL(OBJB_ERR_INVALID_INPUT, act, "need 1 <= num_pairs, num_tokens <= 2^20");
  if (num_pairs * std::max(l->intermediate, l->out_dim) > (1u << 30) || num_tokens * l->hidden > (1ull << 34))
    return OBJB_FAIL(OBJB_ERR_INVALID_INPUT, act, "num_pairs * rows too large");
  return OBJB_OK;
}

}  // namespace

int moe_pairs_official_tc_scratch_bytes(const objb_moe_layer* l, size_t num_pairs, size_t num_tokens, size_t* out) {
  OBJB_TRY(validate_mx(l, num_pairs, num_tokens));
  int device = 0;
  OBJB_TRY(current_device(&device));
  DeviceProps props;
  OBJB_TRY(device_props(device, &props));
  *out = mx_layout(num_pairs, num_tokens, l->hidden, l->intermediate, l->num_experts, props.sm_count).total;
  return OBJB_OK;
}

// The routed experts of the official path over (expert, token) pairs:
// act_quant of the tokens, slices, slice images, gate and up on block-scaled
// MMAs, the official SwiGLU, act_quant of the activations, their images,
// and down into v[pair_out[p]] (unweighted).
int moe_pairs_official_tc(const objb_moe_layer* l, size_t num_pairs, const int32_t* pe, const int32_t* pt,
                          const int32_t* po, size_t num_tokens, const float* x, float* v, size_t v_rows, float limit,
                          cudaStream_t stream, void* scratch, size_t scratch_bytes, const int32_t* d_count) {
  const char* act = "official FP8 x FP4 MoE pairs";
  OBJB_TRY(validate_mx(l, num_pairs, num_tokens));
  if (!pe || !pt || !x || !v || !scratch) return OBJB_FAIL(OBJB_ERR_INVALID_INPUT, act, "null device pointer");
  if (v_rows < (po ? 1 : num_pairs) || v_rows > (1u << 30))
    return OBJB_FAIL(OBJB_ERR_INVALID_INPUT, act, "v_rows cannot hold the pair outputs");
  int device = 0;
  OBJB_TRY(current_device(&device));
  DeviceProps props;
  OBJB_TRY(device_props(device, &props));
  const MxLayout L = mx_layout(num_pairs, num_tokens, l->hidden, l->intermediate, l->num_experts, props.sm_count);
  if (scratch_bytes < L.total)
    return OBJB_FAIL(OBJB_ERR_INVALID_INPUT, act,
                     "scratch of " + std::to_string(scratch_bytes) + " bytes < needed " + std::to_string(L.total));
  unsigned* err = nullptr;
  OBJB_TRY(device_error_word(device, &err));
  uint8_t* sc = static_cast<uint8_t*>(scratch);
  uint8_t* codes_x = sc + L.codes_x;
  uint8_t* scales_x = sc + L.scales_x;
  float* g = reinterpret_cast<float*>(sc + L.g);
  float* u = reinterpret_cast<float*>(sc + L.u);
  uint8_t* codes_a = sc + L.codes_a;
  uint8_t* scales_a = sc + L.scales_a;
  int32_t* run_start = reinterpret_cast<int32_t*>(sc + L.run_start);
  int32_t* slice_start = reinterpret_cast<int32_t*>(sc + L.slice_start);
  int32_t* slice_len = reinterpret_cast<int32_t*>(sc + L.slice_len);
  int32_t* slice_unit = reinterpret_cast<int32_t*>(sc + L.slice_unit);
  int32_t* slice_order = reinterpret_cast<int32_t*>(sc + L.slice_order);
  int32_t* nslices = reinterpret_cast<int32_t*>(sc + L.nslices);
  uint8_t* bimg = sc + L.bimg;
  uint8_t* sfimg = sc + L.sfimg;
  CUtensorMap* maps = reinterpret_cast<CUtensorMap*>(sc + L.maps);
  const int P = static_cast<int>(num_pairs), T = static_cast<int>(num_tokens);
  const int H = static_cast<int>(l->hidden), I = static_cast<int>(l->intermediate), O = static_cast<int>(l->out_dim);
  CUtensorMap tm_gu, tm_dn;
  OBJB_TRY(tc_encode_tiled(&tm_gu, scratch, static_cast<size_t>(H / 2), static_cast<size_t>(I),
                           std::min(dev::kTcRows, I), dev::kMxRawRow));
  OBJB_TRY(tc_encode_tiled(&tm_dn, scratch, static_cast<size_t>(I / 2), static_cast<size_t>(O),
                           std::min(dev::kTcRows, O), dev::kMxRawRow));
  const size_t smem = sizeof(dev::MxSmem);
  OBJB_TRY(ensure_smem_attr(dev::mx_grouped_kernel, device, smem));
  const int img_grid = 2 * props.sm_count;

  OBJB_TRY(act_quant(x, num_tokens, l->hidden, codes_x, scales_x, stream, "act_quant hidden"));
  OBJB_TRY(launch_pdl(dev::tc_slices_kernel, 1, 1024, 0, stream, pe, P, d_count, dev::kMxNvp, dev::kTcUnit, run_start,
                      slice_start, slice_len, slice_unit, nslices,
                      static_cast<int>(mx_max_units(num_pairs, l->num_experts)), err, static_cast<uint8_t*>(nullptr), 0,
                      static_cast<uint8_t*>(nullptr), slice_order));
  {
    const int max_slices = static_cast<int>(mx_max_units(num_pairs, l->num_experts));
    OBJB_TRY(launch_pdl(dev::tc_maps_kernel, std::max(1, (3 * max_slices + 255) / 256), 256, 0, stream, tm_gu, tm_dn,
                        static_cast<const int32_t*>(slice_start), static_cast<const int32_t*>(nslices), max_slices,
                        pe, reinterpret_cast<const uint8_t* const*>(l->d_gate),
                        reinterpret_cast<const uint8_t* const*>(l->d_up),
                        reinterpret_cast<const uint8_t* const*>(l->d_down), static_cast<int>(l->num_experts), maps));
  }
  OBJB_TRY(launch_pdl(dev::mx_image_kernel, img_grid, 256, 0, stream, static_cast<const int32_t*>(slice_start),
                      static_cast<const int32_t*>(slice_len), static_cast<const int32_t*>(slice_unit),
                      static_cast<const int32_t*>(nslices), static_cast<const uint8_t*>(codes_x),
                      static_cast<const uint8_t*>(scales_x), pt, T, H, bimg, sfimg));
  dev::MxArgs a{};
  a.W = reinterpret_cast<const uint8_t* const*>(l->d_gate);
  a.WS = reinterpret_cast<const uint8_t* const*>(l->d_gate_scale);
  a.W2 = reinterpret_cast<const uint8_t* const*>(l->d_up);
  a.WS2 = reinterpret_cast<const uint8_t* const*>(l->d_up_scale);
  a.num_experts = static_cast<int>(l->num_experts);
  a.R = I;
  a.C = H;
  a.pe = pe;
  a.slot_vec = pt;
  a.slot_out = nullptr;
  a.slice_start = slice_start;
  a.slice_len = slice_len;
  a.slice_unit = slice_unit;
  a.nslices = nslices;
  a.slice_order = slice_order;
  a.bimg = bimg;
  a.sfimg = sfimg;
  a.maps = maps;
  a.map0 = 0;
  a.box_rows = std::min(dev::kTcRows, I);
  a.nvec = T;
  a.out = g;
  a.out2 = u;
  a.out_rows = P;
  a.err = err;
  OBJB_TRY(launch_pdl(dev::mx_grouped_kernel, props.sm_count, dev::kMxThreads, smem, stream, a));
  {
    const size_t n = static_cast<size_t>(P) * I;
    const int sg = static_cast<int>(std::max<size_t>(1, std::min<size_t>((n + 255) / 256, 8ull * props.sm_count)));
    OBJB_TRY(launch_pdl(dev::mx_swiglu_kernel, sg, 256, 0, stream, g, static_cast<const float*>(u), n, d_count, I,
                        limit));
  }
  OBJB_TRY(act_quant(g, num_pairs, l->intermediate, codes_a, scales_a, stream, "act_quant intermediate"));
  OBJB_TRY(launch_pdl(dev::mx_image_kernel, img_grid, 256, 0, stream, static_cast<const int32_t*>(slice_start),
                      static_cast<const int32_t*>(slice_len), static_cast<const int32_t*>(slice_unit),
                      static_cast<const int32_t*>(nslices), static_cast<const uint8_t*>(codes_a),
                      static_cast<const uint8_t*>(scales_a), static_cast<const int32_t*>(nullptr), P, I, bimg,
                      sfimg));
  a.W = reinterpret_cast<const uint8_t* const*>(l->d_down);
  a.WS = reinterpret_cast<const uint8_t* const*>(l->d_down_scale);
  a.W2 = nullptr;
  a.WS2 = nullptr;
  a.R = O;
  a.C = I;
  a.box_rows = std::min(dev::kTcRows, O);
  a.slot_vec = nullptr;
  a.slot_out = po;
  a.nvec = P;
  a.out = v;
  a.out2 = nullptr;
  a.out_rows = static_cast<int>(v_rows);
  a.map0 = 2;
  OBJB_TRY(launch_pdl(dev::mx_grouped_kernel, props.sm_count, dev::kMxThreads, smem, stream, a));
  return OBJB_OK;
}

}  // namespace objb

extern "C" {

int objb_moe_pairs_tc_scratch_bytes(const objb_moe_layer* layer, size_t num_pairs, size_t num_tokens,
                                    size_t* bytes) {
  objb::clear_error();
  if (!bytes) return OBJB_FAIL(OBJB_ERR_INVALID_INPUT, "objb_moe_pairs_tc_scratch_bytes", "null output pointer");
  return objb::moe_pairs_tc_scratch_bytes(layer, num_pairs, num_tokens, bytes);
}

int objb_moe_pairs_tc_device(const objb_moe_layer* layer, size_t num_pairs, const int32_t* d_num_pairs,
                             const int32_t* d_pair_expert, const int32_t* d_pair_token, const int32_t* d_pair_out,
                             size_t num_tokens, const float* d_x, float* d_v, size_t v_rows, float swiglu_limit,
                             objb_stream_t stream_) {
  objb::clear_error();
  cudaStream_t stream = static_cast<cudaStream_t>(stream_);
  size_t need = 0;
  OBJB_TRY(objb::moe_pairs_tc_scratch_bytes(layer, num_pairs, num_tokens, &need));
  int device = 0;
  OBJB_TRY(objb::current_device(&device));
  void* ws = nullptr;
  OBJB_TRY(objb::workspace_get(device, stream, need, &ws));
  return objb::moe_pairs_tc(layer, num_pairs, d_pair_expert, d_pair_token, d_pair_out, num_tokens, d_x, d_v, v_rows,
                            swiglu_limit, stream, ws, need, nullptr, d_num_pairs);
}

int objb_moe_pairs_official_tc_scratch_bytes(const objb_moe_layer* layer, size_t num_pairs, size_t num_tokens,
                                             size_t* bytes) {
  objb::clear_error();
  if (!bytes)
    return OBJB_FAIL(OBJB_ERR_INVALID_INPUT, "objb_moe_pairs_official_tc_scratch_bytes", "null output pointer");
  return objb::moe_pairs_official_tc_scratch_bytes(layer, num_pairs, num_tokens, bytes);
}

int objb_moe_pairs_official_tc_device(const objb_moe_layer* layer, size_t num_pairs, const int32_t* d_num_pairs,
                                      const int32_t* d_pair_expert, const int32_t* d_pair_token,
                                      const int32_t* d_pair_out, size_t num_tokens, const float* d_x, float* d_v,
                                      size_t v_rows, float swiglu_limit, objb_stream_t stream_) {
  objb::clear_error();
  cudaStream_t stream = static_cast<cudaStream_t>(stream_);
  size_t need = 0;
  OBJB_TRY(objb::moe_pairs_official_tc_scratch_bytes(layer, num_pairs, num_tokens, &need));
  int device = 0;
  OBJB_TRY(objb::current_device(&device));
  void* ws = nullptr;
  OBJB_TRY(objb::workspace_get(device, stream, need, &ws));
  return objb::moe_pairs_official_tc(layer, num_pairs, d_pair_expert, d_pair_token, d_pair_out, num_tokens, d_x, d_v,
                                     v_rows, swiglu_limit, stream, ws, need, d_num_pairs);
}

}  // extern "C"


