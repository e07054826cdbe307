/*
 * objeta_b200.h -- C ABI of libobjeta_b200.so, the B200 (sm_100a) build of
 * objeta-cuda's quantized GEMV / selected-expert MoE path.
 *
 * This is the boundary a Rust (or any FFI) facade binds.  Every entry point
 * cites the reference Rust item it replaces, as
 * `crates/objeta-cuda/src/<file>:<line>` of the objeta repository.
 *
 * Conventions
 *  - Every function returns an int status: 0 (OBJB_OK) or the reference's
 *    CudaErrorKind ordinal + 1 (crates/objeta-cuda/src/lib.rs:39-48).  The
 *    message of the last failure on the calling thread is available from
 *    objb_last_error().
 *  - `objb_stream_t` is a cudaStream_t.  NULL is the legacy default stream,
 *    which is what the reference's stream 0 is (stream.rs:16).
 *  - `*_device` entry points take device pointers and are asynchronous on the
 *    given stream; `*_host` / executor entry points take host slices and
 *    return host results, like the reference's Rust API.
 *  - Kernels are prebuilt for sm_100a.  There is no NVRTC, no other
 *    architecture and no CPU fallback: on a machine without an sm_100 device
 *    every compute entry point fails with OBJB_ERR_RUNTIME.
 */
#ifndef OBJETA_B200_H
#define OBJETA_B200_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* Status codes = CudaErrorKind ordinal + 1 (lib.rs:39-48). */
enum {
  OBJB_OK = 0,
  OBJB_ERR_DRIVER = 1,
  OBJB_ERR_RUNTIME = 2,
  OBJB_ERR_NVRTC = 3, /* never returned: nothing is compiled at run time */
  OBJB_ERR_IO = 4,
  OBJB_ERR_INVALID_INPUT = 5,
  OBJB_ERR_UNSUPPORTED = 6,
  OBJB_ERR_INTERNAL = 7
};

/* QuantFormat (quant.rs:25-31), same ordinals. */
enum { OBJB_Q4_0 = 0, OBJB_Q5_0 = 1, OBJB_IQ3_0 = 2, OBJB_FP4_E2M1 = 3 };

/* ExpertTensorKind (moe.rs:37-54), same ordinals. */
enum {
  OBJB_KIND_GATE = 0,
  OBJB_KIND_UP = 1,
  OBJB_KIND_DOWN = 2,
  OBJB_KIND_GATE_WEIGHT = 3,
  OBJB_KIND_GATE_SCALE = 4,
  OBJB_KIND_UP_WEIGHT = 5,
  OBJB_KIND_UP_SCALE = 6,
  OBJB_KIND_DOWN_WEIGHT = 7,
  OBJB_KIND_DOWN_SCALE = 8,
  OBJB_KIND_SHARED_GATE_WEIGHT = 9,
  OBJB_KIND_SHARED_GATE_SCALE = 10,
  OBJB_KIND_SHARED_UP_WEIGHT = 11,
  OBJB_KIND_SHARED_UP_SCALE = 12,
  OBJB_KIND_SHARED_DOWN_WEIGHT = 13,
  OBJB_KIND_SHARED_DOWN_SCALE = 14
};

typedef void *objb_stream_t;

/* ------------------------------------------------------------------ misc */

/* Copies the calling thread's last error message (NUL-terminated, truncated
 * to len) and returns its status.  Replaces the Display of CudaError
 * (lib.rs:50-60): "<Kind> error during <action> at <module>:<line> (<file>):
 * <message>". */
int objb_last_error(char *buf, size_t len);

/* ABI version of this header (major * 100 + minor). */
int objb_abi_version(void);

/* QuantFormat metadata (quant.rs:33-96). Strings are static. */
typedef struct {
  uint32_t block_size;
  uint32_t block_bytes;
  uint32_t packed_values_per_byte;
  const char *kernel_name;
  const char *format_label;
  const char *scale_dtype;
  const char *nibble_order;
} objb_format_info;
int objb_format_info_get(int fmt, objb_format_info *out);

/* QGemvShape (quant.rs:98-143): blocks_per_row, quantized row / matrix bytes.
 * Fails with OBJB_ERR_INVALID_INPUT "cols .. must be a multiple of block_size"
 * exactly where validate_quant_inputs (quant.rs:751-812) does. */
typedef struct {
  size_t rows, cols, block_size, block_bytes;
  size_t blocks_per_row, quantized_row_bytes, quantized_matrix_bytes;
} objb_qgemv_shape;
int objb_qgemv_shape_new(int fmt, size_t rows, size_t cols, objb_qgemv_shape *out);

/* BackendDeviceInfo (ffi.rs:14-24) plus SM count and L2 size. */
typedef struct {
  int ordinal;
  size_t total_global_mem_bytes;
  int compute_capability_major;
  int compute_capability_minor;
  int multiprocessor_count;
  size_t l2_cache_bytes;
} objb_device_info;
int objb_device_info_get(int device, objb_device_info *out);

/* QGemvNumerics (quant.rs:156-161) and compare_outputs (quant.rs:676-723):
 * cosine similarity and relative L2 error from f64 sums in element order,
 * max |actual - reference| in f32; InvalidInput "reference len .. != actual
 * len .." on a length mismatch.  Host arrays. */
typedef struct {
  float cosine_similarity;
  float relative_l2_error;
  float max_abs_error;
} objb_qgemv_numerics;
int objb_compare_outputs(const float *reference, size_t reference_len, const float *actual,
                         size_t actual_len, objb_qgemv_numerics *out);

/* Reads and clears the device's error word.  Kernels with bounded waits
 * (bulk-copy pipelines, peer flags) record a nonzero code there instead of
 * hanging when a wait expires; 0 means no wait has expired.  Replaces no
 * reference item (the reference has no bounded waits). */
int objb_device_error_take(int device, unsigned *word);

/* Pins / unpins a host range for asynchronous uploads (replaces
 * PinnedHostBuffer, memory.rs:30-80). */
int objb_host_register(void *ptr, size_t bytes);
int objb_host_unregister(void *ptr);

/* --------------------------------------------------------- QuantBackend */

/* QGemvTelemetry (quant.rs:145-154), same fields. */
typedef struct {
  float h2d_ms, kernel_ms, d2h_ms, unaccounted_ms, total_ms;
  size_t bytes_read;
  float effective_gbps;
} objb_qgemv_telemetry;

typedef struct objb_quant_backend objb_quant_backend;

/* QuantBackend::new (quant.rs:203-213), bound to a CUDA device ordinal. */
int objb_quant_backend_new(int device, objb_quant_backend **out);
void objb_quant_backend_free(objb_quant_backend *qb);
/* QuantBackend::compile_format (quant.rs:221-238): validates the format and
 * makes sure its prebuilt sm_100a kernels are loaded on the device. */
int objb_quant_backend_compile_format(objb_quant_backend *qb, int fmt);

/* QuantBackend::gemv (quant.rs:256-302): host qweights / x in, host y out,
 * H2D + kernel + D2H on `stream`, telemetry filled like the reference
 * (bytes_read = packed bytes + 4*cols; effective_gbps from kernel time). */
int objb_gemv_host(objb_quant_backend *qb, int fmt, objb_stream_t stream,
                   const uint8_t *qweights, size_t qweights_len, const float *x,
                   size_t x_len, size_t rows, size_t cols, float *y,
                   objb_qgemv_telemetry *telemetry);

/* QuantBackend::launch_kernel (quant.rs:324-366): y[rows] = dequant(W) x,
 * device pointers, asynchronous on `stream`.  W is the reference's
 * interleaved block layout (18 / 22 / 14 / 17 bytes per 32 weights). */
int objb_gemv_device(int fmt, const void *d_qweights, const float *d_x, float *d_y,
                     size_t rows, size_t cols, objb_stream_t stream);

/* QuantBackend::launch_kernel_split_fp4 (quant.rs:368-408): DeepSeek split
 * layout, weight [rows, cols/2] (low nibble first) + E8M0 scale
 * [rows, cols/32]. */
int objb_gemv_fp4_split_device(const void *d_weight, const void *d_scale,
                               const float *d_x, float *d_y, size_t rows,
                               size_t cols, objb_stream_t stream);

/* Diagnostics (no reference counterpart; host arithmetic only, no GPU needed):
 * how the pipelined kernel streams a rows x cols matrix of `fmt` (split_fp4:
 * the DeepSeek split layout) with `blocks_per_lane` 32-column blocks per lane
 * (2; 1 for split FP4 rows), one matrix or a gate/up pair (dual), as a plain
 * GEMV (moe_program 0) or inside the MoE / FFN programs (1).  out[0..8] =
 * column segments (warps per row), row groups, rows per stage, ring slots,
 * bytes per slot, dynamic shared memory, rows per stage that keep every row
 * group busy, 1 if a 16-byte aligned x (one vector per launch) is formed
 * inside the kernel instead of by an x-image launch, the ring budget in bytes.
 * OBJB_ERR_UNSUPPORTED: the shape takes the fallback kernel. */
int objb_pipe_plan_info(int fmt, int split_fp4, size_t rows, size_t cols, int blocks_per_lane, int dual,
                        int moe_program, int32_t *out, int nout);

/* Dense bf16 GEMV (no QuantFormat in the reference; the shared expert of a
 * DeepSeek-style layer): y[rows] = W x with W bf16 [rows, cols] row-major,
 * widened to f32 as the reference's bf16 conversion does (objeta-parser
 * lib.rs:334-337), f32 accumulation.  cols must be a multiple of 32. */
int objb_gemv_bf16_device(const void *d_w, const float *d_x, float *d_y, size_t rows,
                          size_t cols, objb_stream_t stream);

/* One dense SwiGLU FFN in bf16 (the shared expert): act = SwiGLU(gate x,
 * up x) as silu_mul computes it (moe.cu:2-22), v = down act; d_out = v, or
 * d_out += v when accumulate is nonzero (routed output + shared output).
 * gate / up are [intermediate, hidden], down [out_dim, intermediate]. */
int objb_ffn_bf16_device(const void *d_gate, const void *d_up, const void *d_down,
                         size_t hidden, size_t intermediate, size_t out_dim,
                         const float *d_x, float *d_out, int accumulate, float swiglu_limit,
                         objb_stream_t stream);

/* quantize_matrix_cpu (quant.rs:506-581) on the device: packs a dense f32
 * [rows, cols] matrix into the format's blocks, byte-identical to the
 * reference CPU packers (q4/q5/iq3/fp4_quantize_block, quant.rs:814-926). */
int objb_quantize_matrix_device(int fmt, const float *d_matrix, size_t rows,
                                size_t cols, void *d_out, objb_stream_t stream);

/* decode_deepseek_fp4_to_f32 (objeta-parser/src/deepseek.rs:862-918): split
 * FP4 weight + E8M0 scale (block 32) to dense f32; code 8 decodes to +0.0
 * as in the parser's FP4_E2M1FN_TABLE (deepseek.rs:789-792). */
int objb_fp4_decode_split_device(const void *d_weight, const void *d_scale,
                                 size_t rows, size_t cols, float *d_out,
                                 objb_stream_t stream);

/* ------------------------------------------------ selected-expert MoE */

/* objb_moe_layer.flags */
enum {
  /* Some expert tensor pointer is not 16-byte aligned (or a row is not a
   * multiple of 16 bytes): run the generic path instead of the bulk-copy
   * pipeline. */
  OBJB_MOE_UNALIGNED = 1
};

/* One MoE layer resident on the device.  The expert tensors keep the
 * reference's layouts: ExpertWeights (moe.rs:13-18) -- Q4_0 (or Q5_0 / IQ3_0 /
 * interleaved FP4) gate / up [intermediate x hidden] and down
 * [out_dim x intermediate] -- or DeepSeekFp4ExpertWeights (moe.rs:27-35),
 * fmt = OBJB_FP4_E2M1 with the three scale tables set: split weight
 * [rows, cols/2] + E8M0 scale [rows, cols/32].  d_gate / d_up / d_down (and
 * the scale tables) are DEVICE arrays of num_experts device pointers. */
typedef struct {
  int fmt;
  uint32_t flags;
  size_t hidden, intermediate, out_dim, num_experts;
  const void *const *d_gate;
  const void *const *d_up;
  const void *const *d_down;
  const void *const *d_gate_scale;
  const void *const *d_up_scale;
  const void *const *d_down_scale;
} objb_moe_layer;

/* cpu_router (crates/objeta-cuda/src/bin/deepseek_single_layer_moe.rs:
 * 720-740) on the device: softmax of the logits, the top_k of a stable
 * descending sort (ties keep the lower expert index), weights = the kept
 * probabilities, divided by their sum when renormalize != 0. */
int objb_router_topk_device(const float *d_logits, size_t num_experts, size_t top_k,
                            int renormalize, int32_t *d_ids, float *d_weights,
                            objb_stream_t stream);

/* Bytes of device scratch objb_moe_selected_device uses for top_k experts
 * (it takes them from a per-(device, stream) workspace allocated on first
 * use, so make the first call on a stream outside graph capture). */
int objb_moe_scratch_bytes(const objb_moe_layer *layer, size_t top_k, size_t *bytes);

/* The selected-expert MoE FFN of MoeExecutor::execute_selected_moe_cuda /
 * execute_selected_moe_native_fp4_cuda (moe.rs:352-751, 816-1280) for one
 * token, with the selection (d_ids, d_weights: top_k entries) and x already
 * on the device: out = sum_k w_k * down_k(silu(gate_k x) * up_k x), summed in
 * selection order.  swiglu_limit > 0 clamps as silu_mul does (moe.cu:2-22).
 * Two pipelined launches (gate+up with SwiGLU fused; down with the weighted
 * combine fused) plus two small x-image builds; asynchronous on `stream`. */
int objb_moe_selected_device(const objb_moe_layer *layer, const int32_t *d_ids,
                             const float *d_weights, size_t top_k, const float *d_x,
                             float *d_out, float swiglu_limit, objb_stream_t stream);

/* No counterpart in the reference.  The same launch as
 * objb_moe_selected_device for callers that cannot let a library allocate
 * device memory (a host framework that reserves all HBM up front and forbids
 * allocation on its hot path, or whose allocator must see every byte): the
 * scratch comes from a fixed 4 MiB array in the library's device image (held
 * on every GPU that loads the library until the process exits) instead of a
 * cudaMalloc'd workspace; nothing is allocated.  Layers whose scratch
 * (objb_moe_scratch_bytes) exceeds 4 MiB - 256 bytes are rejected with
 * OBJB_ERR_INVALID_INPUT.  The first call on a device looks up the array's
 * device address (once per device, with that device current); make that
 * first call before any stream capture.  All calls on a device share the one
 * array: calls that overlap on the GPU (different streams, or host threads
 * racing) race on it.  Each call clears the error word at the array's start
 * and overwrites the scratch it reads; nothing needs clearing between calls.
 * A device-side error (an out-of-range expert id, a pipeline wait that ran
 * out) is not reported through objb_device_error_take: it turns every element
 * of d_out into NaN. */
int objb_moe_selected_device_noalloc(const objb_moe_layer *layer, const int32_t *d_ids,
                                     const float *d_weights, size_t top_k, const float *d_x,
                                     float *d_out, float swiglu_limit, objb_stream_t stream);

/* ---- multi-token MoE (no counterpart in the reference, which runs one token
 * per execute_selected_moe_cuda call; the per-pair arithmetic is the same).
 *
 * objb_moe_pairs_device runs the layer over num_pairs (expert, token) pairs:
 * for pair p, e = d_pair_expert[p] and t = d_pair_token[p] (0 <= t <
 * num_tokens, x row t of d_x [num_tokens][hidden]); the unweighted down
 * output down_e(SwiGLU(gate_e x_t, up_e x_t)) is written to row
 * d_pair_out[p] of d_v [v_rows][out_dim] (row p when d_pair_out is NULL).
 * Pairs are computed in the given order: group them by expert so each
 * expert's weights are streamed once while they sit in L2.  Every output row
 * is bit-identical to the value the single-token launch computes for the same
 * expert and x.  Out-of-range ids or rows are clamped to 0 and flagged in the
 * device error word (bit 8).  Scratch comes from the per-stream workspace,
 * sized for num_pairs.  d_num_pairs (may be NULL): a device int32 holding the
 * number of pairs to run (at most num_pairs), written by an earlier kernel on
 * the stream -- the work is then split over the SMs inside the kernels, so a
 * pair list built on the device needs no host round trip (aligned layers
 * only). */
int objb_moe_pairs_scratch_bytes(const objb_moe_layer *layer, size_t num_pairs,
                                 size_t num_tokens, size_t *bytes);
int objb_moe_pairs_device(const objb_moe_layer *layer, size_t num_pairs,
                          const int32_t *d_num_pairs, const int32_t *d_pair_expert,
                          const int32_t *d_pair_token, const int32_t *d_pair_out,
                          size_t num_tokens, const float *d_x, float *d_v, size_t v_rows,
                          float swiglu_limit, objb_stream_t stream);

/* objb_moe_pairs_device for Q4_0 layers on the tensor cores (tcgen05 kind::i8
 * MMAs into tensor memory): the same arguments and outputs, with each run of
 * equal experts in the pair list taken 32 pairs at a time against one
 * 128-row tile of the expert's matrix, so a weight tile is decoded once per
 * 32 pairs instead of once per pair.  Block sums are the same exact integers
 * as the CUDA-core path; the f32 block terms are added in another order, so
 * rows agree with objb_moe_pairs_device within the f32 tolerance, not
 * bit for bit (each row is still a function of (expert, x) alone, whatever
 * else is in the pair list).  Pairs must be grouped by expert; an expert
 * that appears in several separate runs is streamed once per run.  Q4_0
 * layers with 16-byte aligned experts and hidden, intermediate multiples of
 * 256 only (OBJB_ERR_UNSUPPORTED otherwise). */
int objb_moe_pairs_tc_scratch_bytes(const objb_moe_layer *layer, size_t num_pairs,
                                    size_t num_tokens, size_t *bytes);
int objb_moe_pairs_tc_device(const objb_moe_layer *layer, size_t num_pairs,
                             const int32_t *d_num_pairs, const int32_t *d_pair_expert,
                             const int32_t *d_pair_token, const int32_t *d_pair_out,
                             size_t num_tokens, const float *d_x, float *d_v, size_t v_rows,
                             float swiglu_limit, objb_stream_t stream);

/* The routed experts of execute_selected_moe_official_routed_fp4_cuda
 * (moe.rs:1393-1548) over (expert, token) pairs on block-scaled tensor cores
 * (no reference counterpart for many tokens; the reference runs one token
 * per call).  Same pair arguments as objb_moe_pairs_device; the layer is a
 * split FP4 E2M1 layer with its E8M0 scale tables, d_x [num_tokens][hidden]
 * f32.  Per pair: act_quant(x) -> FP8 x FP4 gate and up ->
 * SwiGLU with only the up value clamped to +-swiglu_limit (deepseek.rs:
 * 1707-1711) -> act_quant -> FP8 x FP4 down into row d_pair_out[p] of d_v
 * (unweighted; combine with objb_moe_combine_device).  The FP8 x FP4 dots
 * run as tcgen05.mma.kind::mxf8f6f4.block_scale: E2M1 weights and E4M3
 * activations with their UE8M0 block scales multiplied exactly and summed in
 * f32 by the tensor core, so rows match the CUDA-core official path within
 * the f32 tolerance (and the re-quantized activation may move by one FP8
 * step, as between any two orders of summation).  Pairs must be grouped by
 * expert; up to 128 pairs of an expert share one pass over a weight tile.
 * hidden and intermediate: multiples of 128. */
int objb_moe_pairs_official_tc_scratch_bytes(const objb_moe_layer *layer, size_t num_pairs,
                                             size_t num_tokens, size_t *bytes);
int objb_moe_pairs_official_tc_device(const objb_moe_layer *layer, size_t num_pairs,
                                      const int32_t *d_num_pairs, const int32_t *d_pair_expert,
                                      const int32_t *d_pair_token, const int32_t *d_pair_out,
                                      size_t num_tokens, const float *d_x, float *d_v,
                                      size_t v_rows, float swiglu_limit, objb_stream_t stream);

/* The weighted top-k combine (moe.rs:1319-1321) for num_tokens tokens:
 * d_out[t][i] = sum over j = 0..top_k-1, in slot order, of
 * d_weights[t][j] * d_v[d_slot_row[t][j]][i], starting from 0 -- the exact
 * arithmetic of the single-token fused combine. */
int objb_moe_combine_device(const float *d_v, size_t v_rows, const int32_t *d_slot_row,
                            const float *d_weights, size_t num_tokens, size_t top_k,
                            size_t out_dim, float *d_out, objb_stream_t stream);

/* objb_router_topk_device for num_tokens rows of logits [num_tokens][num_experts]
 * (one CTA per token); ids / weights are [num_tokens][top_k]. */
int objb_router_topk_batched_device(const float *d_logits, size_t num_tokens,
                                    size_t num_experts, size_t top_k, int renormalize,
                                    int32_t *d_ids, float *d_weights, objb_stream_t stream);

/* Router + selected-expert MoE in one call: logits -> (d_ids, d_weights) ->
 * out.  d_ids / d_weights receive the selection. */
int objb_moe_forward_device(const objb_moe_layer *layer, const float *d_logits,
                            size_t top_k, int renormalize, int32_t *d_ids, float *d_weights,
                            const float *d_x, float *d_out, float swiglu_limit,
                            objb_stream_t stream);

/* ------------------------------------------------------- expert cache */

/* ExpertCacheKey (moe.rs:56-62): tensor_kind = OBJB_KIND_*, quant_format =
 * OBJB_Q4_0 ... */
typedef struct {
  size_t layer_id;
  size_t expert_id;
  int32_t tensor_kind;
  int32_t quant_format;
} objb_expert_cache_key;

/* The public counters of CudaExpertCache (moe.rs:70-89), same names, plus the
 * number of tensors that did not fit the cache's slab and were allocated on
 * their own. */
typedef struct {
  size_t capacity_bytes, resident_bytes, pinned_bytes;
  size_t hit_count, miss_count, eviction_count;
  int32_t bypass_oversized_experts;
  size_t cache_insert_attempt_count, cache_insert_accept_count, cache_insert_bypass_count;
  size_t oversized_tensor_bypass_count, oversized_expert_bypass_count, self_eviction_risk_count;
  size_t overflow_allocations;
} objb_expert_cache_stats;

typedef struct objb_expert_cache objb_expert_cache;

/* CudaExpertCache::new (moe.rs:92-111): a byte-capacity LRU cache of expert
 * tensors resident on `device`. */
int objb_expert_cache_new(int device, size_t capacity_bytes, objb_expert_cache **out);
void objb_expert_cache_free(objb_expert_cache *cache);

/* get (moe.rs:113-122): on a hit counts it, moves the key to most-recent
 * and returns the device pointer; on a miss counts it and returns NULL. */
int objb_expert_cache_get(objb_expert_cache *cache, const objb_expert_cache_key *key,
                          const void **d_ptr);

/* insert (moe.rs:124-154): uploads `bytes` from host_src and makes it
 * resident (evicting least-recent non-pinned tensors until it fits), or, when
 * bytes > capacity, counts an oversized bypass and returns a buffer that is
 * not cached (*resident = 0), valid until the next release point.  The upload
 * runs on the cache's side stream; `stream` is made to wait for it. */
int objb_expert_cache_insert(objb_expert_cache *cache, const objb_expert_cache_key *key,
                             const void *host_src, size_t bytes, objb_stream_t stream,
                             const void **d_ptr, int *resident);

/* The README's get_or_insert (README.md:121-124): get, and on a miss insert;
 * counters move exactly as the executor's inline get/insert (moe.rs:508-518).
 * *hit = 1 on a hit (host_src is then not read). */
int objb_expert_cache_get_or_insert(objb_expert_cache *cache, const objb_expert_cache_key *key,
                                    const void *host_src, size_t bytes, objb_stream_t stream,
                                    const void **d_ptr, int *hit);

/* The same with the README's lazy `load_fn` (README.md:121-124): `load` runs
 * only on a miss and hands back the host bytes to upload (it must keep them
 * valid until the call returns); a nonzero return from it is passed through
 * as this call's status with nothing inserted.  `load` runs without the
 * cache's lock held, but the cache is externally synchronised (one owning
 * thread): `load` must not use this cache. */
typedef int (*objb_expert_load_fn)(void *user, const void **host_src, size_t *bytes);
int objb_expert_cache_get_or_load(objb_expert_cache *cache, const objb_expert_cache_key *key,
                                  objb_expert_load_fn load, void *user, objb_stream_t stream,
                                  const void **d_ptr, int *hit);

/* touch / evict_lru / pin / insert_pinned / clear / reset_counters
 * (moe.rs:156-226). evict_lru reports the evicted key in *evicted. */
int objb_expert_cache_touch(objb_expert_cache *cache, const objb_expert_cache_key *key);
int objb_expert_cache_evict_lru(objb_expert_cache *cache, objb_expert_cache_key *evicted, int *found);
int objb_expert_cache_pin(objb_expert_cache *cache, const objb_expert_cache_key *key);
int objb_expert_cache_insert_pinned(objb_expert_cache *cache, const objb_expert_cache_key *key,
                                    const void *host_src, size_t bytes, objb_stream_t stream,
                                    const void **d_ptr);
int objb_expert_cache_clear(objb_expert_cache *cache);
int objb_expert_cache_reset_counters(objb_expert_cache *cache);

/* The public fields of the reference struct. */
int objb_expert_cache_stats_get(objb_expert_cache *cache, objb_expert_cache_stats *out);
int objb_expert_cache_set_bypass_oversized_experts(objb_expert_cache *cache, int bypass);
/* Executor-side admission counters (moe.rs:483-494, the executor bumps the
 * cache's public fields directly in the reference). which: 0 =
 * oversized_expert_bypass, 1 = self_eviction_risk, 2 = insert attempt +
 * bypass (one bypassed tensor of a bypassed expert). */
int objb_expert_cache_count(objb_expert_cache *cache, int which);

/* Membership and LRU order (least recent first), for inspection. */
int objb_expert_cache_contains(objb_expert_cache *cache, const objb_expert_cache_key *key, int *found);
int objb_expert_cache_lru_keys(objb_expert_cache *cache, objb_expert_cache_key *out, size_t cap,
                               size_t *n);

/* Release point: every pointer handed out so far has had all of its reads
 * enqueued on `stream`.  Slots evicted before this call become reusable once
 * `stream` reaches this point, and bypass buffers are freed in stream order.
 * (No reference counterpart: the reference keeps evicted buffers alive with
 * Arc reference counts.) */
int objb_expert_cache_release(objb_expert_cache *cache, objb_stream_t stream);

/* --------------------------------------------------------- MoeExecutor */

/* ExpertWeights (moe.rs:13-18): host slices of one expert. */
typedef struct {
  const uint8_t *w_gate;
  size_t w_gate_len;
  const uint8_t *w_up;
  size_t w_up_len;
  const uint8_t *w_down;
  size_t w_down_len;
} objb_expert_weights;

/* DeepSeekFp4ExpertWeights (moe.rs:27-35). */
typedef struct {
  const uint8_t *gate_weight;
  size_t gate_weight_len;
  const uint8_t *gate_scale;
  size_t gate_scale_len;
  const uint8_t *up_weight;
  size_t up_weight_len;
  const uint8_t *up_scale;
  size_t up_scale_len;
  const uint8_t *down_weight;
  size_t down_weight_len;
  const uint8_t *down_scale;
  size_t down_scale_len;
} objb_fp4_expert_weights;

/* MoeTelemetry (moe.rs:236-276), same fields (bytes_by_tensor_kind flattened
 * into bytes_gate / bytes_up / bytes_down). */
typedef struct {
  size_t selected_expert_count;
  size_t logical_expert_bytes_requested;
  size_t actual_expert_bytes_loaded;
  size_t resident_cache_bytes_reused;
  size_t weight_bytes_loaded, weight_bytes_reused, scale_bytes_loaded, scale_bytes_reused;
  size_t resident_cache_resident_bytes, resident_cache_capacity_bytes;
  size_t resident_cache_hit_count, resident_cache_miss_count, resident_cache_eviction_count;
  size_t resident_cache_insert_attempt_count, resident_cache_insert_accept_count;
  size_t resident_cache_insert_bypass_count, resident_cache_oversized_tensor_bypass_count;
  size_t resident_cache_oversized_expert_bypass_count, resident_cache_self_eviction_risk_count;
  size_t dequantized_scratch_bytes;
  float h2d_ms, gate_up_qgemv_ms, activation_ms, down_qgemv_ms, accum_ms, unaccounted_ms, total_ms,
      shared_expert_ms;
  size_t bytes_gate, bytes_up, bytes_down;
  size_t bytes_per_expert, selected_working_set_bytes;
  size_t routed_fp4_bytes_loaded, routed_fp4_bytes_reused, shared_fp8_bytes_loaded, shared_fp8_bytes_reused;
  size_t total_logical_bytes, total_loaded_bytes, total_reused_bytes;
} objb_moe_telemetry;

typedef struct objb_moe_executor objb_moe_executor;

/* MoeExecutor::new / compile (moe.rs:292-307). */
int objb_moe_executor_new(int device, objb_moe_executor **out);
void objb_moe_executor_free(objb_moe_executor *ex);
int objb_moe_executor_compile(objb_moe_executor *ex);

/* MoeExecutor::execute_selected_moe_cuda (moe.rs:352-751): host experts,
 * host selection (expert index, weight) in order, host x; writes out[out_dim]
 * and the telemetry.  fmt is OBJB_Q4_0 for the reference path (Q5_0 / IQ3_0
 * run the same way).  With a cache, tensors are looked up / uploaded / evicted
 * with the reference's counters and byte accounting; without one every tensor
 * is uploaded for this call.  Fails with InvalidInput on the reference's
 * validation errors and Internal if the byte invariant logical == loaded +
 * reused does not hold. */
int objb_moe_execute_selected(objb_moe_executor *ex, objb_stream_t stream, int fmt,
                              const objb_expert_weights *experts, size_t num_experts,
                              const int64_t *selected_ids, const float *selected_weights,
                              size_t num_selected, const float *x, size_t x_len, size_t hidden,
                              size_t intermediate, size_t out_dim, size_t layer_id,
                              objb_expert_cache *cache, float *out, objb_moe_telemetry *telemetry);

/* MoeExecutor::execute_selected_moe_native_fp4_cuda (moe.rs:816-1280). */
int objb_moe_execute_selected_native_fp4(objb_moe_executor *ex, objb_stream_t stream,
                                         const objb_fp4_expert_weights *experts, size_t num_experts,
                                         const int64_t *selected_ids, const float *selected_weights,
                                         size_t num_selected, const float *x, size_t x_len,
                                         size_t hidden, size_t intermediate, size_t out_dim,
                                         size_t layer_id, objb_expert_cache *cache, float *out,
                                         objb_moe_telemetry *telemetry);

/* Multi-token form of objb_moe_execute_selected (no reference counterpart:
 * the reference runs one token per call) on device activations: num_pairs
 * (expert, token) pairs given as host int32 arrays (pair_out may be NULL:
 * row p), d_x [num_tokens][hidden] and d_v [v_rows][out_dim] on the device.
 * Each distinct expert among the pairs is resolved once, in order of first
 * appearance, with the reference executor's admission rules (moe.rs:483-583:
 * oversized-expert bypass or self-eviction risk, then get / insert per
 * tensor); then all pairs run as one objb_moe_pairs_device launch sequence.
 * Telemetry counts each distinct expert once.  Synchronises `stream`. */
int objb_moe_execute_pairs(objb_moe_executor *ex, objb_stream_t stream, int fmt,
                           const objb_expert_weights *experts, size_t num_experts,
                           const int32_t *pair_expert, const int32_t *pair_token,
                           const int32_t *pair_out, size_t num_pairs, const float *d_x,
                           size_t num_tokens, size_t hidden, size_t intermediate,
                           size_t out_dim, size_t layer_id, objb_expert_cache *cache,
                           float *d_v, size_t v_rows, objb_moe_telemetry *tel);

/* ---- expert parallelism, device side (no counterpart in the reference).
 * A rank holds experts [rank*E/G, (rank+1)*E/G).  After the host framework
 * all-gathers the routing table d_ids_all [G][T][top_k] (and the routing
 * weights and token rows [G*T][hidden]):
 *  - objb_ep_build_pairs_device writes this rank's pairs (local expert id,
 *    token row s*T + t, output row (s*T + t)*top_k + j) grouped by expert into
 *    arrays of G*T*top_k entries and their number into *d_num_pairs, for
 *    objb_moe_pairs_device with d_num_pairs (v has G*T*top_k rows);
 *  - objb_ep_partial_combine_device folds, per routing row (s, t), w * v over
 *    the slots whose expert is local, in slot order: d_partial [G][T][out_dim];
 *  - after an all-to-all of the partials, objb_ep_sum_partials_device adds
 *    d_parts [G][T][out_dim] over ranks in rank order into d_out [T][out_dim].
 * Expert ids out of range are dropped and flagged (device error word bit 8). */
int objb_ep_build_pairs_device(const int32_t *d_ids_all, size_t world, size_t tokens,
                               size_t top_k, size_t num_experts, size_t rank,
                               int32_t *d_pair_expert, int32_t *d_pair_token,
                               int32_t *d_pair_out, int32_t *d_num_pairs, objb_stream_t stream);
int objb_ep_partial_combine_device(const int32_t *d_ids_all, const float *d_w_all,
                                   const float *d_v, size_t world, size_t tokens, size_t top_k,
                                   size_t num_experts, size_t rank, size_t out_dim,
                                   float *d_partial, objb_stream_t stream);
int objb_ep_sum_partials_device(const float *d_parts, size_t world, size_t tokens,
                                size_t out_dim, float *d_out, objb_stream_t stream);

/* The same step with ONE all-gather instead of three (no reference
 * counterpart).  A rank packs its step into a buffer of
 * objb_ep_packed_rows(T, top_k, H) rows of H floats: its T token rows, then
 * its routing ids (int32 bits) and weights, zero-padded
 * (objb_ep_pack_device).  After an all-gather of those buffers into d_recv
 * [G][rows][H], the pair builder and the partial combine read ids, weights
 * and token rows straight from it: pair_token is then a row of d_recv seen
 * as [G*rows][H] (pass it to objb_moe_pairs_device with num_tokens =
 * G*rows); pair_out and the partials are as above. */
size_t objb_ep_packed_rows(size_t tokens, size_t top_k, size_t hidden);
int objb_ep_pack_device(const float *d_x, const int32_t *d_ids, const float *d_w, size_t tokens,
                        size_t top_k, size_t hidden, float *d_send, objb_stream_t stream);
int objb_ep_build_pairs_packed_device(const float *d_recv, size_t world, size_t tokens,
                                      size_t top_k, size_t hidden, size_t num_experts, size_t rank,
                                      int32_t *d_pair_expert, int32_t *d_pair_token,
                                      int32_t *d_pair_out, int32_t *d_num_pairs,
                                      objb_stream_t stream);
int objb_ep_partial_combine_packed_device(const float *d_recv, const float *d_v, size_t world,
                                          size_t tokens, size_t top_k, size_t hidden,
                                          size_t num_experts, size_t rank, size_t out_dim,
                                          float *d_partial, objb_stream_t stream);

/* cpu_gate_ref (dsl_moe.rs:768-881), the DeepSeek V4 gate, for num_tokens
 * tokens (one CTA each): logits = W h with W f32 [num_experts][hidden_size]
 * (sequential f32 sums, bit-identical to the reference); scores by
 * score_func (0 softmax, 1 sigmoid, 2 sqrt-softplus); ids = top_k of
 * scores + bias (d_gate_bias may be NULL; stable: ties keep the lower index)
 * or, for a hash layer (d_tid2eid != NULL, d_input_ids required),
 * tid2eid[input_id * top_k + k]; weights = scores[ids], normalised by their
 * sum unless softmax, times route_scale.  An input id out of range gives ids
 * -1, NaN weights and device error word bit 8. */
int objb_deepseek_gate_device(const float *d_gate_weight, const float *d_gate_bias,
                              const int64_t *d_tid2eid, size_t tid2eid_len, const float *d_hidden,
                              const int64_t *d_input_ids, size_t num_tokens, size_t num_experts,
                              size_t hidden_size, size_t top_k, int score_func, float route_scale,
                              int32_t *d_ids, float *d_weights, objb_stream_t stream);

/* ---- official DeepSeek arithmetic: activations quantized to F8_E4M3 with one
 * E8M0 scale per 128 values (deepseek.rs:1444-1525 for the codecs). */

/* cuda_act_quant_device (quant.rs:1229-1282): rows x cols f32 -> E4M3 codes
 * [rows][cols] + E8M0 scales [rows][cols/128], bit-identical to the reference
 * CPU act_quant (cpu_act_quant, deepseek.rs:1484).  InvalidInput "cols ..
 * not divisible by 128". */
int objb_act_quant_device(const float *d_x, size_t rows, size_t cols, uint8_t *d_values,
                          uint8_t *d_scales, objb_stream_t stream);

/* cuda_fp8_act_fp4_weight_gemv_device (quant.rs:1284-1326): y[rows] = W a with
 * a = act_quant output (E4M3 [cols] + E8M0 [cols/128]) and W the split FP4
 * layout (weight [rows, cols/2], E8M0 [rows, cols/32]).  Block sums are exact
 * integers (act * 2^9 in three 7-bit digits, 2 * FP4 in int8, dp4a). */
int objb_gemv_fp8_fp4_device(const uint8_t *d_act, const uint8_t *d_act_scales,
                             const void *d_weight, const void *d_weight_scales, float *d_y,
                             size_t rows, size_t cols, objb_stream_t stream);

/* cuda_fp8_act_fp8_weight_gemv_device (quant.rs:1328-1363): weight E4M3
 * [rows, cols] with E8M0 scales on a 128 x 128 tile grid. */
int objb_gemv_fp8_fp8_device(const uint8_t *d_act, const uint8_t *d_act_scales,
                             const void *d_weight, const void *d_weight_scales, float *d_y,
                             size_t rows, size_t cols, objb_stream_t stream);

/* The routed experts of execute_selected_moe_official_routed_fp4_cuda
 * (moe.rs:1393-1548) on a device-resident split-FP4 layer: act_quant(x) ->
 * FP8 x FP4 gate/up with SwiGLU -> act_quant(act) -> FP8 x FP4 down with the
 * weighted combine in selection order.  The SwiGLU is the official CPU
 * path's (deepseek.rs:1707-1711): only the up value is clamped to
 * +-swiglu_limit (the reference executor passes 10).  hidden and
 * intermediate must be multiples of 512. */
int objb_moe_official_scratch_bytes(const objb_moe_layer *layer, size_t top_k, size_t *bytes);
int objb_moe_official_selected_device(const objb_moe_layer *layer, const int32_t *d_ids,
                                      const float *d_weights, size_t top_k, const float *d_x,
                                      float *d_out, float swiglu_limit, objb_stream_t stream);

/* DeepSeekFp8SharedExpertWeightsDevice (moe.rs:1372-1379): device pointers. */
typedef struct {
  const void *gate_weight, *gate_scale;
  const void *up_weight, *up_scale;
  const void *down_weight, *down_scale;
} objb_fp8_shared_expert;

/* MoeExecutor::execute_selected_moe_official_routed_fp4_cuda (moe.rs:1393):
 * host split-FP4 experts through the cache (as the native FP4 call), the
 * official routed arithmetic, and, when `shared` is not NULL, the FP8 shared
 * expert (act_quant -> FP8 x FP8 gate/up -> SwiGLU (up clamped to +-10) -> act_quant ->
 * down) added with weight 1.  Telemetry as the reference (routed FP4 bytes,
 * shared FP8 bytes, shared_expert_ms). */
int objb_moe_execute_selected_official_fp4(
    objb_moe_executor *ex, objb_stream_t stream, const objb_fp4_expert_weights *experts,
    size_t num_experts, const int64_t *selected_ids, const float *selected_weights,
    size_t num_selected, const float *x, size_t x_len, size_t hidden, size_t intermediate,
    size_t out_dim, size_t layer_id, objb_expert_cache *cache,
    const objb_fp8_shared_expert *shared, float *out, objb_moe_telemetry *telemetry);

/* ---- safetensors weights (ModelWeights, objeta-parser lib.rs:97-330): an
 * mmap of one file or of every *.safetensors file of a directory (file-name
 * order), indexed by tensor name; "__metadata__" is skipped. */
enum {
  OBJB_DTYPE_F32 = 0,
  OBJB_DTYPE_F16 = 1,
  OBJB_DTYPE_BF16 = 2,
  OBJB_DTYPE_I64 = 3,
  OBJB_DTYPE_I32 = 4,
  OBJB_DTYPE_I8 = 5,
  OBJB_DTYPE_U8 = 6,
  OBJB_DTYPE_F8_E8M0 = 7,
  OBJB_DTYPE_F8_E4M3 = 8,
  OBJB_DTYPE_BOOL = 9
};

/* TensorInfo (lib.rs:21-28); offset is absolute in its file. */
typedef struct {
  int dtype;
  int ndim;
  size_t shape[8];
  size_t offset, nbytes, nelem;
} objb_tensor_info;

typedef struct objb_weights objb_weights;

/* ModelWeights::open: Io for unreadable paths, InvalidInput for malformed
 * headers ("header length exceeds file size", "invalid tensor entry ..",
 * "Unknown dtype: .."). */
int objb_weights_open(const char *path, objb_weights **out);
void objb_weights_close(objb_weights *w);
int objb_weights_count(objb_weights *w, size_t *n);                       /* len() */
int objb_weights_name_at(objb_weights *w, size_t i, const char **name);   /* keys(), sorted */
int objb_weights_info(objb_weights *w, const char *name, objb_tensor_info *info);
/* get_raw: a pointer into the mapping, valid until objb_weights_close. */
int objb_weights_raw(objb_weights *w, const char *name, const void **data, size_t *nbytes);
/* get_f32: F32 as is, F16 / BF16 widened as the reference (lib.rs:285-337). */
int objb_weights_get_f32(objb_weights *w, const char *name, float *out, size_t out_len);
/* Pins the weights for asynchronous DMA into the expert cache or the device:
 * the mapping itself (read-only host registration) where the platform
 * allows it, else a pinned host slab holding a copy of each file.  Pointers
 * from objb_weights_raw taken after this call point into pinned memory. */
int objb_weights_pin(objb_weights *w);
int objb_weights_to_device(objb_weights *w, const char *name, void *d_dst, size_t dst_bytes,
                           objb_stream_t stream);

#ifdef __cplusplus
}
#endif
#endif /* OBJETA_B200_H */
