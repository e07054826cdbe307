// objb_common.h -- status codes, error recording and format metadata shared by
// every translation unit of libobjeta_b200.so (host side).
#pragma once

#include <cuda_runtime.h>

#include <cstddef>
#include <cstdint>
#include <string>

#include "../../include/objeta_b200.h"

namespace objb {

// Records `kind` plus a formatted message as this thread's last error and
// returns `kind`.  The message layout follows the reference's CudaError
// Display impl (crates/objeta-cuda/src/lib.rs:51-52):
//   "<Kind> error during <action> at <module>:<line> (<file>): <message>".
int set_error(int kind, const char* action, const std::string& message, const char* file,
              int line);
void clear_error();

// Converts a CUDA runtime error into a Runtime status with the CUDA message.
int cuda_status(cudaError_t e, const char* action, const char* file, int line);

#define OBJB_FAIL(kind, action, msg) ::objb::set_error((kind), (action), (msg), __FILE__, __LINE__)
#define OBJB_CUDA(call, action)                                                  \
  do {                                                                           \
    cudaError_t objb_e_ = (call);                                                \
    if (objb_e_ != cudaSuccess) return ::objb::cuda_status(objb_e_, (action), __FILE__, __LINE__); \
  } while (0)
#define OBJB_TRY(expr)              \
  do {                              \
    int objb_rc_ = (expr);          \
    if (objb_rc_ != OBJB_OK) return objb_rc_; \
  } while (0)

// QuantFormat::block_bytes (crates/objeta-cuda/src/quant.rs:43-50).
inline int block_bytes(int fmt) {
  switch (fmt) {
    case OBJB_Q4_0: return 18;
    case OBJB_Q5_0: return 22;
    case OBJB_IQ3_0: return 14;
    case OBJB_FP4_E2M1: return 17;
    default: return 0;
  }
}
inline bool valid_format(int fmt) { return block_bytes(fmt) != 0; }
const char* format_label(int fmt);

// validate_shape_metadata + validate_quant_inputs (quant.rs:751-812): cols must
// be a multiple of block_size (32); the message text is the reference's.
int validate_gemv_shape(int fmt, size_t rows, size_t cols);

// Lazily created per-device error word used by kernels with bounded waits.
int device_error_word(int device, unsigned int** out);

// Per-(device, stream) device workspace, grow-only, at least
// kWorkspaceMinBytes.  Work on one stream is ordered, so one buffer per stream
// is race-free; it cannot be allocated while the stream is being captured.
constexpr size_t kWorkspaceMinBytes = 1u << 20;
int workspace_get(int device, cudaStream_t stream, size_t bytes, void** out);

}  // namespace objb
