// objb_moe_launch.h -- internal entry points of the device MoE layer, used by
// the C ABI (moe.cu) and the host-slice executor (executor.cpp).
#pragma once

#include <cuda_runtime.h>

#include <cstddef>
#include <cstdint>

#include "../../include/objeta_b200.h"

namespace objb {

// Scratch a selected-expert launch needs: the SwiGLU activations of the
// top_k experts plus the x images of the hidden vector and of the
// activations (or only the activations on the generic path).
int moe_scratch_bytes(const objb_moe_layer* l, size_t top_k, size_t* out);

// One token through the layer with caller-provided scratch.
int moe_selected(const objb_moe_layer* l, const int32_t* ids, const float* weights, size_t top_k,
                 const float* x, float* out, float limit, cudaStream_t stream, void* scratch,
                 size_t scratch_bytes, cudaEvent_t mid = nullptr, unsigned* err_word = nullptr);

int router_topk(const float* logits, size_t n, size_t top_k, int renorm, int32_t* ids, float* weights,
                cudaStream_t stream);

}  // namespace objb
