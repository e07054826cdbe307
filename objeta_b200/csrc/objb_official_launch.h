// objb_official_launch.h -- host launchers of the official DeepSeek activation
// path (official.cu), shared with the MoE and executor translation units.
#pragma once

#include <cuda_runtime.h>

#include <cstddef>
#include <cstdint>

#include "objb_launch.h"
#include "../../include/objeta_b200.h"

namespace objb {

// act_quant of rows x cols f32 (cols % 128 == 0) into E4M3 codes and E8M0
// scales (one per 128 values), bit-identical to the reference CPU act_quant.
int act_quant(const float* x, size_t rows, size_t cols, uint8_t* values, uint8_t* scales, cudaStream_t stream,
              const char* action);

// Row plan of an FP8 x FP4 (split layout) matrix for the pipelined kernel.
bool plan_fp8_fp4(int rows, int cols, bool dual, RowLayoutHost* L);
size_t fp8_image_quads(const RowLayoutHost& L);
// x images of nvec act_quant outputs (codes [nvec][L.cols], scales [nvec][L.cols/128]).
int launch_ximage_fp8(const RowLayoutHost& L, const uint8_t* codes, const uint8_t* scales, int nvec, uint4* img,
                      size_t img_stride_quads, cudaStream_t stream);

// The FP8 shared expert of the official path, added onto out (weight 1).
size_t shared_expert_fp8_scratch(int H, int I, int O);
int shared_expert_fp8(const objb_fp8_shared_expert* sh, const float* x, int H, int I, int O, float limit, float* out,
                      cudaStream_t stream, void* scratch, size_t scratch_bytes);

int gemv_fp8_fp8(const uint8_t* act, const uint8_t* act_s, const uint8_t* w, const uint8_t* ws, float* y, int rows,
                 int cols, cudaStream_t stream);

}  // namespace objb
