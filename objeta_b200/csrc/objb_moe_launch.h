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

// Multi-token MoE over (expert, token) pairs: v[pair_out[p]] = down(SwiGLU(
// gate x[pair_token[p]], up x[pair_token[p]])) of expert pair_expert[p].
int moe_pairs_scratch_bytes(const objb_moe_layer* l, size_t num_pairs, size_t num_tokens, size_t* out);
int moe_pairs(const objb_moe_layer* l, size_t num_pairs, const int32_t* pair_expert, const int32_t* pair_token,
              const int32_t* pair_out, size_t num_tokens, const float* x, float* v, size_t v_rows, float limit,
              cudaStream_t stream, void* scratch, size_t scratch_bytes, unsigned* err_word = nullptr,
              const int32_t* d_num_pairs = nullptr);
// The same pairs on the tensor cores (Q4_0 layers, hidden / intermediate
// multiples of 256, pairs grouped by expert), grouped.cu.
int moe_pairs_tc_scratch_bytes(const objb_moe_layer* l, size_t num_pairs, size_t num_tokens, size_t* out);
int moe_pairs_tc(const objb_moe_layer* l, size_t num_pairs, const int32_t* pe, const int32_t* pt, const int32_t* po,
                 size_t num_tokens, const float* x, float* v, size_t v_rows, float limit, cudaStream_t stream,
                 void* scratch, size_t scratch_bytes, unsigned* err_word, const int32_t* d_count);
// Pair count from which the multi-token paths take the tensor cores.
constexpr size_t kTcMinPairs = 256;
int moe_combine(const float* v, size_t v_rows, const int32_t* slot_row, const float* weights, size_t num_tokens,
                size_t top_k, size_t out_dim, float* out, cudaStream_t stream, unsigned* err_word = nullptr);
int router_topk_batched(const float* logits, size_t num_tokens, size_t n, size_t top_k, int renorm, int32_t* ids,
                        float* weights, cudaStream_t stream);

// Official DeepSeek routed experts (FP8 activations, split FP4 weights).
int moe_official_scratch_bytes(const objb_moe_layer* l, size_t top_k, size_t* out);
int moe_official_selected(const objb_moe_layer* l, const int32_t* ids, const float* weights, size_t top_k,
                          const float* x, float* out, float limit, cudaStream_t stream, void* scratch,
                          size_t scratch_bytes, cudaEvent_t mid = nullptr, unsigned* err_word = nullptr);

int router_topk(const float* logits, size_t n, size_t top_k, int renorm, int32_t* ids, float* weights,
                cudaStream_t stream);

}  // namespace objb
