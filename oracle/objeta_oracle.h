/*
 * objeta_oracle.h -- TEST INFRASTRUCTURE ONLY.
 *
 * A plain-C CPU restatement of the arithmetic of objeta's `objeta-cuda` hot
 * path (Rust crate `objeta-cuda`, plus two helpers from `objeta-parser`).  It
 * is the checker for the CUDA product in `objeta_b200/`: only `tests/`,
 * `__graft_entry__.smoke()` and the `cpu_baseline` / `--impl reference` legs
 * of `bench.py` may load it.  Nothing in the product links or calls it.
 *
 * Every function names the reference file:line it restates.  Paths are
 * relative to the objeta repository root.  The file is compiled with
 * `-O2 -fno-fast-math -ffp-contract=off` so every f32 add / mul / div rounds
 * once, exactly like the Rust code it follows (rustc never contracts a*b+c
 * into an FMA), and it calls glibc's expf / log2f / ceilf / roundf, which is
 * what Rust's f32::exp / log2 / ceil / round lower to on Linux.
 */
#ifndef OBJETA_ORACLE_H
#define OBJETA_ORACLE_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* QuantFormat ordinals, in the order of the Rust enum (quant.rs:25-31). */
enum { ORO_Q4_0 = 0, ORO_Q5_0 = 1, ORO_IQ3_0 = 2, ORO_FP4_E2M1 = 3 };

/* Return codes: 0 ok, 5 = CudaErrorKind::InvalidInput + 1 (lib.rs:39-48). */
enum { ORO_OK = 0, ORO_INVALID_INPUT = 5 };

size_t oro_block_bytes(int fmt);

uint16_t oro_f32_to_f16_bits(float value);
float oro_f16_to_f32_bits(uint16_t bits);
float oro_decode_f8_e8m0(uint8_t raw);
float oro_f8e8m0_to_f32(uint8_t raw);
float oro_f8e4m3_to_f32(uint8_t raw);

void oro_q4_quantize_block(const float *src, uint8_t *dst);
void oro_q5_quantize_block(const float *src, uint8_t *dst);
void oro_iq3_quantize_block(const float *src, uint8_t *dst);
void oro_fp4_quantize_block(const float *src, uint8_t *dst);

int oro_quantize_matrix(int fmt, const float *matrix, size_t rows, size_t cols,
                        uint8_t *out);

float oro_dot_row(int fmt, const uint8_t *row_q, const float *x, size_t cols);
int oro_gemv(int fmt, const uint8_t *qweights, const float *x, size_t rows,
             size_t cols, float *y);
/* Row-parallel variant of oro_gemv (same per-row arithmetic), for the CPU
 * baseline timing; threads <= 0 means all online cores. */
int oro_gemv_threads(int fmt, const uint8_t *qweights, const float *x,
                     size_t rows, size_t cols, float *y, int threads);
int oro_dequantize_matrix(int fmt, const uint8_t *qw, size_t rows, size_t cols,
                          float *out);
void oro_dense_gemv(const float *matrix, const float *x, size_t rows,
                    size_t cols, float *y);

void oro_fp4_decode_split(const uint8_t *weight, const uint8_t *scale,
                          size_t rows, size_t cols, size_t block_size,
                          float *out);

int oro_selected_moe_q4(const uint8_t *const *w_gate,
                        const uint8_t *const *w_up,
                        const uint8_t *const *w_down, size_t num_experts,
                        const int64_t *sel_ids, const float *sel_weights,
                        size_t num_selected, const float *x, size_t hidden,
                        size_t intermediate, size_t out_dim, float *out,
                        int threads);

int oro_selected_moe_native_fp4(
    const uint8_t *const *gate_w, const uint8_t *const *gate_s,
    const uint8_t *const *up_w, const uint8_t *const *up_s,
    const uint8_t *const *down_w, const uint8_t *const *down_s,
    size_t num_experts, const int64_t *sel_ids, const float *sel_weights,
    size_t num_selected, const float *x, size_t hidden, size_t intermediate,
    size_t out_dim, float *out, int threads);

int oro_router_from_logits(const float *logits, size_t num_experts,
                           size_t top_k, int renormalize, int64_t *ids,
                           float *weights);
int oro_router(const float *router_weights, const float *hidden,
               size_t num_experts, size_t hidden_size, size_t top_k,
               int64_t *ids, float *weights);

void oro_seeded_f32s(size_t len, uint64_t seed, float *out);

/* DeepSeek gate (dsl_moe.rs:768-881); score_func 0 softmax, 1 sigmoid,
 * 2 sqrt-softplus; tid2eid may be NULL (non-hash layer). */
int oro_deepseek_gate(const float *gate_weight, const float *gate_bias, const int64_t *tid2eid,
                      size_t tid2eid_len, const float *hidden, int64_t input_id, size_t num_experts,
                      size_t hidden_size, size_t top_k, int score_func, float route_scale, int64_t *ids,
                      float *weights);

/* Official DeepSeek arithmetic (deepseek.rs:1444-1715). */
uint8_t oro_f32_to_f8e4m3_exact(float v);
int oro_act_quant(const float *x, size_t n, size_t block, uint8_t *y, uint8_t *s);
void oro_fp8_act_fp4_weight_gemv_f32(const uint8_t *act, const uint8_t *act_s, const uint8_t *w,
                                     const uint8_t *ws, size_t rows, size_t cols, float *y);
void oro_fp8_act_fp8_weight_gemv(const uint8_t *act, const uint8_t *act_s, const uint8_t *w,
                                 const uint8_t *ws, size_t rows, size_t cols, float *y);
int oro_routed_expert_fp4_official_f32(const uint8_t *gw, const uint8_t *gs, const uint8_t *uw,
                                       const uint8_t *us, const uint8_t *dw, const uint8_t *ds,
                                       const float *x, size_t dim, size_t inter, size_t out_dim,
                                       float swiglu_limit, float *out);
int oro_shared_expert_fp8_official(const uint8_t *w1, const uint8_t *s1, const uint8_t *w3,
                                   const uint8_t *s3, const uint8_t *w2, const uint8_t *s2,
                                   const float *x, size_t dim, size_t inter, float swiglu_limit,
                                   float *out);

#ifdef __cplusplus
}
#endif
#endif
