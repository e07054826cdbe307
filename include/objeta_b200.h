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

#ifdef __cplusplus
}
#endif
#endif /* OBJETA_B200_H */
