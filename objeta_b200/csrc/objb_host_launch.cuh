// objb_host_launch.cuh -- host-side launch helpers shared by the kernels'
// translation units: large-shared-memory opt-in, x-image builds and
// programmatic-dependent launches.
#pragma once

#include <cuda_runtime.h>

#include <algorithm>
#include <cstring>
#include <type_traits>

#include "objb_common.h"
#include "objb_gemv.cuh"
#include "objb_launch.h"

namespace objb {

template <class K>
int ensure_smem_attr(K kernel, int device, size_t bytes) {
  return ensure_smem_attr_ptr(reinterpret_cast<const void*>(kernel), device, bytes);
}

// Launches the x-image prep kernel for `nvec` vectors into `img`, then lets
// the caller launch the consumer kernel with programmatic serialization.
// Launches `kernel` with programmatic stream serialization: it may start while
// the previous kernel in the stream is still running, and must wait
// (griddepcontrol.wait) before touching anything that kernel produces.
template <class... KArgs, class... Args>
int launch_pdl(void (*kernel)(KArgs...), int grid, int threads, size_t smem, cudaStream_t stream,
               Args... args) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(grid);
  cfg.blockDim = dim3(threads);
  cfg.dynamicSmemBytes = smem;
  cfg.stream = stream;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  OBJB_CUDA(cudaLaunchKernelEx(&cfg, kernel, args...), "launch pipelined kernel");
  return OBJB_OK;
}

template <class RD>
int launch_ximage(const RowLayoutHost& L, const float* x, size_t x_stride, int nvec, uint4* img,
                  size_t img_stride_quads, cudaStream_t stream, const int32_t* count = nullptr) {
  dev::RowLayout dl;
  std::memcpy(&dl, &L, sizeof(dl));
  // Launched with programmatic serialization: the kernel waits
  // (griddepcontrol.wait) for the preceding grid before reading x, so its
  // launch overlaps that grid's tail.
  if constexpr (dev::IsSplitDigitRD<RD>::value) {
    const int warps = L.nseg * 32 * RD::P * nvec;
    const int grid = std::max(1, std::min((warps + 7) / 8, 2048));
    return launch_pdl(dev::ximage_split_digits_kernel<RD::P>, grid, 256, 0, stream, dl, x, x_stride, nvec, img,
                      img_stride_quads, count);
  } else if constexpr (dev::IsDigitRD<RD>::value) {
    const int warps = L.nseg * 32 * 2 * nvec;
    const int grid = std::max(1, std::min((warps + 7) / 8, 2048));
    return launch_pdl(dev::ximage_digits_kernel<dev::IsDigitRD<RD>::fmt>, grid, 256, 0, stream, dl, x, x_stride,
                      nvec, img, img_stride_quads, count);
  } else {
    const int n = L.nseg * 32 * RD::XRegs::kQuads * nvec;
    const int grid = std::max(1, std::min((n + 255) / 256, 2048));
    return launch_pdl(dev::ximage_f32_kernel<RD>, grid, 256, 0, stream, dl, x, x_stride, nvec, img,
                      img_stride_quads, count);
  }
}

template <class RD>
size_t ximage_quads(const RowLayoutHost& L) {
  return static_cast<size_t>(RD::XRegs::kQuads) * L.nseg * 32;
}

// Whether the pipelined kernel forms the x registers of ONE vector x itself
// (a program-level x): float quads straight from x (16-byte aligned) for the
// row formats where that beats the image launch, or a digit image built in
// every CTA, which only pays up to 128 blocks (4096 columns: it hides under
// the first stage's copy) and must fit one ring slot.
template <class RD>
bool inline_x_ok(const RowLayoutHost& L, const float* x) {
  constexpr int kInlineDigitBlocks = 128;
  if (!aligned16(x)) return false;
  if (dev::IsFloatRD<RD>::value) return dev::DirectQuadsOnce<RD>::value;
  return dev::IsDigitRD<RD>::value && L.nblocks <= kInlineDigitBlocks && L.nslots >= 2 &&
         ximage_quads<RD>(L) * 16 <= static_cast<size_t>(L.stage_bytes);
}

// Whether each job may read its own float vector base + i * stride directly:
// float-quad rows whose lanes read near-coalesced quads (for the others a
// per-job read costs more than the image launch it saves), every vector
// 16-byte aligned.
template <class RD>
bool direct_x_ok(const float* base, size_t stride_floats) {
  return dev::IsFloatRD<RD>::value && dev::NearCoalescedQuads<RD>::value && aligned16(base) &&
         stride_floats % 4 == 0;
}



}  // namespace objb
