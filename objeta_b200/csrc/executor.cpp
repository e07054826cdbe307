// executor.cpp -- MoeExecutor (moe.rs:286-1280): the host-slice selected-expert
// MoE API.  Per call it validates like the reference, uploads x, resolves every
// tensor of every selected expert through the cache (or uploads it for this
// call), then runs the whole selection as one fused device MoE (objb_moe) and
// copies the output back, filling MoeTelemetry with the reference's byte
// accounting.
#include <cuda_runtime.h>

#include <algorithm>
#include <cstring>
#include <mutex>
#include <set>
#include <string>
#include <vector>

#include "objb_cache.h"
#include "objb_common.h"
#include "objb_launch.h"
#include "objb_moe_launch.h"
#include "objb_official_launch.h"

namespace objb {
int cache_get(objb_expert_cache* c, const objb_expert_cache_key* k, const void** out);
int cache_insert(objb_expert_cache* c, const objb_expert_cache_key* k, const void* host, size_t bytes,
                 cudaStream_t stream, const void** out, int* resident);
int cache_release(objb_expert_cache* c, cudaStream_t stream);
void cache_begin_batch(objb_expert_cache* c);
int cache_end_batch(objb_expert_cache* c, cudaStream_t stream);
}  // namespace objb

struct objb_moe_executor {
  int device = 0;
  std::mutex mu;
  cudaEvent_t ev[8] = {};
  // grow-only device buffers
  void* d_x = nullptr;
  size_t d_x_cap = 0;
  void* d_out = nullptr;
  size_t d_out_cap = 0;
  void* d_meta = nullptr;  // pointer tables, ids, weights
  size_t d_meta_cap = 0;
  void* d_scratch = nullptr;
  size_t d_scratch_cap = 0;
  void* h_meta = nullptr;  // pinned staging of the meta block
  size_t h_meta_cap = 0;
};

namespace objb {
namespace {

struct DeviceGuard {
  int prev = -1;
  bool switched = false;
  int enter(int device) {
    OBJB_CUDA(cudaGetDevice(&prev), "query current device");
    if (prev != device) {
      OBJB_CUDA(cudaSetDevice(device), "select device");
      switched = true;
    }
    return OBJB_OK;
  }
  ~DeviceGuard() {
    if (switched) cudaSetDevice(prev);
  }
};

int grow_dev(void** p, size_t* cap, size_t need, const char* what) {
  if (need <= *cap && *p) return OBJB_OK;
  if (*p) {
    OBJB_CUDA(cudaDeviceSynchronize(), "drain before growing a buffer");
    cudaFree(*p);
  }
  *p = nullptr;
  *cap = 0;
  OBJB_CUDA(cudaMalloc(p, std::max<size_t>(need, 256)), what);
  *cap = std::max<size_t>(need, 256);
  return OBJB_OK;
}

int grow_host(void** p, size_t* cap, size_t need) {
  if (need <= *cap && *p) return OBJB_OK;
  if (*p) cudaFreeHost(*p);
  *p = nullptr;
  *cap = 0;
  OBJB_CUDA(cudaMallocHost(p, std::max<size_t>(need, 256)), "allocate pinned staging");
  *cap = std::max<size_t>(need, 256);
  return OBJB_OK;
}

// One tensor of a selected expert, in the reference's load order.
struct TensorRef {
  const uint8_t* host;
  size_t len;
  int32_t kind;
  bool is_scale;
};

int fail_len(const char* what, size_t got, size_t want) {
  return OBJB_FAIL(OBJB_ERR_INVALID_INPUT, (std::string("validate expert ") + what + " size").c_str(),
                   std::string(what) + " len " + std::to_string(got) + " != expected " + std::to_string(want));
}

// Byte accounting and per-call uploads of one executor call.
struct Resolved {
  size_t weight_loaded = 0, weight_reused = 0, scale_loaded = 0, scale_reused = 0;
  size_t bytes_gate = 0, bytes_up = 0, bytes_down = 0;
  std::vector<void*> transients;  // bypassed tensors, freed after the call
};

// Resolves the 3 (or 6) tensors of expert `expert_id` to device pointers the
// way the reference executor does (moe.rs:483-583): an expert larger than the
// whole cache is either bypassed (uploaded for this call only) or counted as
// a self-eviction risk; each tensor is then looked up (hit: reused bytes) or
// inserted (miss: loaded bytes).  Without a cache every tensor is uploaded.
int resolve_expert(objb_expert_cache* cache, cudaStream_t stream, int fmt, bool split, size_t layer_id,
                   size_t expert_id, const TensorRef* t, const void** ptrs, Resolved* r) {
  const int ntens = split ? 6 : 3;
  size_t expert_bytes = 0;
  for (int i = 0; i < ntens; ++i) expert_bytes += t[i].len;
  // bytes_by_tensor_kind: gate / up / down (weight + scale for FP4)
  if (split) {
    r->bytes_gate += t[0].len + t[1].len;
    r->bytes_up += t[2].len + t[3].len;
    r->bytes_down += t[4].len + t[5].len;
  } else {
    r->bytes_gate += t[0].len;
    r->bytes_up += t[1].len;
    r->bytes_down += t[2].len;
  }
  bool bypass = false;
  if (cache) {
    std::lock_guard<std::mutex> lk(cache->mu);
    if (expert_bytes > cache->st.capacity_bytes) {  // moe.rs:483-494
      if (cache->st.bypass_oversized_experts) {
        bypass = true;
        cache->st.oversized_expert_bypass_count += 1;
      } else {
        cache->st.self_eviction_risk_count += 1;
      }
    }
  }
  int rc = OBJB_OK;
  for (int i = 0; i < ntens && rc == OBJB_OK; ++i) {
    size_t& loaded = t[i].is_scale ? r->scale_loaded : r->weight_loaded;
    size_t& reused = t[i].is_scale ? r->scale_reused : r->weight_reused;
    const void* dp = nullptr;
    if (cache && !bypass) {
      std::lock_guard<std::mutex> lk(cache->mu);
      objb_expert_cache_key key{layer_id, expert_id, t[i].kind, fmt};
      rc = cache_get(cache, &key, &dp);
      if (rc == OBJB_OK && dp) {
        reused += t[i].len;
      } else if (rc == OBJB_OK) {
        loaded += t[i].len;
        rc = cache_insert(cache, &key, t[i].host, t[i].len, stream, &dp, nullptr);
      }
    } else {
      if (cache) {  // bypassed expert: counted as a bypassed insert per tensor
        std::lock_guard<std::mutex> lk(cache->mu);
        cache->st.cache_insert_attempt_count += 1;
        cache->st.cache_insert_bypass_count += 1;
      }
      void* p = nullptr;
      cudaError_t e = cudaMallocAsync(&p, std::max<size_t>(t[i].len, 16), stream);
      if (e == cudaSuccess && t[i].len) e = cudaMemcpyAsync(p, t[i].host, t[i].len, cudaMemcpyHostToDevice, stream);
      if (e != cudaSuccess) rc = cuda_status(e, "upload expert tensor", __FILE__, __LINE__);
      if (p) r->transients.push_back(p);
      loaded += t[i].len;
      dp = p;
    }
    ptrs[i] = dp;
  }
  return rc;
}

// The shared body of execute_selected_moe_cuda / _native_fp4_cuda.
// tensors_of(k) fills the 3 (or 6) TensorRefs of selected expert k; the
// device tables get one entry per selected slot.
// The official DeepSeek variant of a call (execute_selected_moe_official_routed_fp4_cuda).
struct Official {
  float swiglu_limit = 10.0f;  // the reference executor's silu_mul limit (moe.rs:1525)
  const objb_fp8_shared_expert* shared = nullptr;
};

template <class TensorsOf>
int execute(objb_moe_executor* ex, cudaStream_t stream, int fmt, bool split, size_t num_selected,
            const int64_t* sel_ids, const float* sel_weights, const float* x, size_t hidden,
            size_t intermediate, size_t out_dim, size_t layer_id, objb_expert_cache* cache, float* out,
            objb_moe_telemetry* tel, size_t single_expert_bytes, TensorsOf tensors_of,
            const Official* official = nullptr) {
  DeviceGuard g;
  OBJB_TRY(g.enter(ex->device));
  const size_t K = num_selected;
  const int ntens = split ? 6 : 3;
  cudaEvent_t* ev = ex->ev;
  OBJB_CUDA(cudaEventRecord(ev[0], stream), "record total start");
  OBJB_CUDA(cudaEventRecord(ev[1], stream), "record h2d start");
  OBJB_TRY(grow_dev(&ex->d_x, &ex->d_x_cap, hidden * 4, "allocate device x"));
  OBJB_TRY(grow_dev(&ex->d_out, &ex->d_out_cap, out_dim * 4, "allocate device out"));
  OBJB_CUDA(cudaMemcpyAsync(ex->d_x, x, hidden * 4, cudaMemcpyHostToDevice, stream), "copy x to device");

  Resolved res;
  std::vector<const void*> ptrs(K * ntens, nullptr);
  std::set<int64_t> unique;
  int rc = OBJB_OK;
  for (size_t k = 0; k < K && rc == OBJB_OK; ++k) {
    TensorRef t[6];
    tensors_of(k, t);
    unique.insert(sel_ids[k]);
    rc = resolve_expert(cache, stream, fmt, split, layer_id, static_cast<size_t>(sel_ids[k]), t, &ptrs[k * ntens],
                        &res);
  }
  size_t& weight_loaded = res.weight_loaded;
  size_t& weight_reused = res.weight_reused;
  size_t& scale_loaded = res.scale_loaded;
  size_t& scale_reused = res.scale_reused;
  size_t& bytes_gate = res.bytes_gate;
  size_t& bytes_up = res.bytes_up;
  size_t& bytes_down = res.bytes_down;
  std::vector<void*>& transients = res.transients;
  if (rc == OBJB_OK) rc = cudaEventRecord(ev[2], stream) == cudaSuccess ? OBJB_OK : OBJB_FAIL(OBJB_ERR_RUNTIME, "record h2d stop", "cudaEventRecord failed");

  // Device tables: one entry per selected slot; ids are the slots themselves.
  uint32_t flags = 0;
  for (const void* p : ptrs)
    if (reinterpret_cast<uintptr_t>(p) & 15u) flags |= OBJB_MOE_UNALIGNED;
  const size_t meta = K * ntens * sizeof(void*) + K * sizeof(int32_t) + K * sizeof(float) + 64;
  if (rc == OBJB_OK) rc = grow_host(&ex->h_meta, &ex->h_meta_cap, meta);
  if (rc == OBJB_OK) rc = grow_dev(&ex->d_meta, &ex->d_meta_cap, meta, "allocate MoE tables");
  objb_moe_layer layer = {};
  const int32_t* d_ids = nullptr;
  const float* d_w = nullptr;
  if (rc == OBJB_OK) {
    // the previous call ended with a stream synchronize, so the staging
    // block is free (calls on one executor are serialised by its mutex)
    uint8_t* h = static_cast<uint8_t*>(ex->h_meta);
    const void** tab = reinterpret_cast<const void**>(h);
    for (int i = 0; i < ntens; ++i)
      for (size_t k = 0; k < K; ++k) tab[i * K + k] = ptrs[k * ntens + i];
    int32_t* ids = reinterpret_cast<int32_t*>(h + K * ntens * sizeof(void*));
    float* w = reinterpret_cast<float*>(ids + K);
    for (size_t k = 0; k < K; ++k) {
      ids[k] = static_cast<int32_t>(k);
      w[k] = sel_weights[k];
    }
    OBJB_CUDA(cudaMemcpyAsync(ex->d_meta, ex->h_meta, meta, cudaMemcpyHostToDevice, stream), "copy MoE tables");
    const void* const* dtab = static_cast<const void* const*>(ex->d_meta);
    d_ids = reinterpret_cast<const int32_t*>(static_cast<uint8_t*>(ex->d_meta) + K * ntens * sizeof(void*));
    d_w = reinterpret_cast<const float*>(d_ids + K);
    layer.fmt = fmt;
    layer.flags = flags;
    layer.hidden = hidden;
    layer.intermediate = intermediate;
    layer.out_dim = out_dim;
    layer.num_experts = K;
    if (split) {
      layer.d_gate = dtab;
      layer.d_gate_scale = dtab + K;
      layer.d_up = dtab + 2 * K;
      layer.d_up_scale = dtab + 3 * K;
      layer.d_down = dtab + 4 * K;
      layer.d_down_scale = dtab + 5 * K;
    } else {
      layer.d_gate = dtab;
      layer.d_up = dtab + K;
      layer.d_down = dtab + 2 * K;
    }
  }
  if (rc == OBJB_OK && K > 0) {
    size_t need = 0;
    rc = official ? moe_official_scratch_bytes(&layer, K, &need) : moe_scratch_bytes(&layer, K, &need);
    if (official && official->shared)
      need = std::max(need, shared_expert_fp8_scratch(static_cast<int>(hidden), static_cast<int>(intermediate),
                                                      static_cast<int>(out_dim)));
    if (rc == OBJB_OK) rc = grow_dev(&ex->d_scratch, &ex->d_scratch_cap, need, "allocate MoE scratch");
    if (rc == OBJB_OK) rc = cudaEventRecord(ev[3], stream) == cudaSuccess ? OBJB_OK : OBJB_ERR_RUNTIME;
    if (rc == OBJB_OK)
      rc = official ? moe_official_selected(&layer, d_ids, d_w, K, static_cast<const float*>(ex->d_x),
                                            static_cast<float*>(ex->d_out), official->swiglu_limit, stream,
                                            ex->d_scratch, ex->d_scratch_cap, ev[4])
                    : moe_selected(&layer, d_ids, d_w, K, static_cast<const float*>(ex->d_x),
                                   static_cast<float*>(ex->d_out), 0.0f, stream, ex->d_scratch, ex->d_scratch_cap,
                                   ev[4]);
  } else if (rc == OBJB_OK) {
    cudaEventRecord(ev[3], stream);
    OBJB_CUDA(cudaMemsetAsync(ex->d_out, 0, out_dim * 4, stream), "zero output");
    cudaEventRecord(ev[4], stream);
  }
  if (rc == OBJB_OK) rc = cudaEventRecord(ev[5], stream) == cudaSuccess ? OBJB_OK : OBJB_ERR_RUNTIME;
  const bool shared = official && official->shared;
  if (rc == OBJB_OK && shared) {
    // the shared expert reads the device x and adds onto the routed output
    rc = shared_expert_fp8(official->shared, static_cast<const float*>(ex->d_x), static_cast<int>(hidden),
                           static_cast<int>(intermediate), static_cast<int>(out_dim), official->swiglu_limit,
                           static_cast<float*>(ex->d_out), stream, ex->d_scratch, ex->d_scratch_cap);
    if (rc == OBJB_OK) rc = cudaEventRecord(ev[7], stream) == cudaSuccess ? OBJB_OK : OBJB_ERR_RUNTIME;
  }
  if (rc == OBJB_OK) {
    cudaError_t e = cudaMemcpyAsync(out, ex->d_out, out_dim * 4, cudaMemcpyDeviceToHost, stream);
    if (e != cudaSuccess) rc = cuda_status(e, "copy output to host", __FILE__, __LINE__);
  }
  if (rc == OBJB_OK) cudaEventRecord(ev[6], stream);
  // release point: everything this call handed to the kernels is enqueued
  if (cache) {
    std::lock_guard<std::mutex> lk(cache->mu);
    int r2 = cache_release(cache, stream);
    if (rc == OBJB_OK) rc = r2;
  }
  for (void* p : transients) cudaFreeAsync(p, stream);
  cudaError_t se = cudaStreamSynchronize(stream);
  if (rc != OBJB_OK) return rc;
  if (se != cudaSuccess) return cuda_status(se, "synchronize MoE stream", __FILE__, __LINE__);
  {
    unsigned* w = nullptr;
    OBJB_TRY(device_error_word(ex->device, &w));
    unsigned v = 0;
    OBJB_CUDA(cudaMemcpy(&v, w, sizeof(v), cudaMemcpyDeviceToHost), "read device error word");
    if (v) {
      cudaMemset(w, 0, sizeof(unsigned));
      return OBJB_FAIL(OBJB_ERR_INTERNAL, "run selected-expert MoE", "device error word " + std::to_string(v));
    }
  }
  const size_t logical = bytes_gate + bytes_up + bytes_down;
  const size_t loaded = weight_loaded + scale_loaded, reused = weight_reused + scale_reused;
  if (logical != loaded + reused)  // moe.rs:743-748
    return OBJB_FAIL(OBJB_ERR_INTERNAL, "account MoE bytes", "MoE Byte invariant violated!");
  if (tel) {
    std::memset(tel, 0, sizeof(*tel));
    float h2d = 0, gu = 0, dn = 0, d2h = 0, tot = 0;
    cudaEventElapsedTime(&h2d, ev[1], ev[2]);
    cudaEventElapsedTime(&gu, ev[3], ev[4]);
    cudaEventElapsedTime(&dn, ev[4], ev[5]);
    float sh_ms = 0;
    if (shared) {
      cudaEventElapsedTime(&sh_ms, ev[5], ev[7]);
      cudaEventElapsedTime(&d2h, ev[7], ev[6]);
    } else {
      cudaEventElapsedTime(&d2h, ev[5], ev[6]);
    }
    cudaEventElapsedTime(&tot, ev[0], ev[6]);
    tel->selected_expert_count = K;
    tel->logical_expert_bytes_requested = logical;
    tel->actual_expert_bytes_loaded = loaded;
    tel->resident_cache_bytes_reused = reused;
    tel->weight_bytes_loaded = weight_loaded;
    tel->weight_bytes_reused = weight_reused;
    tel->scale_bytes_loaded = scale_loaded;
    tel->scale_bytes_reused = scale_reused;
    if (cache) {
      std::lock_guard<std::mutex> lk(cache->mu);
      const objb_expert_cache_stats& s = cache->st;
      tel->resident_cache_resident_bytes = s.resident_bytes;
      tel->resident_cache_capacity_bytes = s.capacity_bytes;
      tel->resident_cache_hit_count = s.hit_count;
      tel->resident_cache_miss_count = s.miss_count;
      tel->resident_cache_eviction_count = s.eviction_count;
      tel->resident_cache_insert_attempt_count = s.cache_insert_attempt_count;
      tel->resident_cache_insert_accept_count = s.cache_insert_accept_count;
      tel->resident_cache_insert_bypass_count = s.cache_insert_bypass_count;
      tel->resident_cache_oversized_tensor_bypass_count = s.oversized_tensor_bypass_count;
      tel->resident_cache_oversized_expert_bypass_count = s.oversized_expert_bypass_count;
      tel->resident_cache_self_eviction_risk_count = s.self_eviction_risk_count;
    }
    tel->dequantized_scratch_bytes = 0;  // blocks decode in registers; nothing is expanded
    tel->h2d_ms = h2d;
    tel->gate_up_qgemv_ms = gu;  // SwiGLU is fused into the gate/up launch
    tel->activation_ms = 0.0f;
    tel->down_qgemv_ms = dn;     // the weighted accumulate is fused into the down launch
    tel->accum_ms = 0.0f;
    tel->total_ms = tot;
    tel->unaccounted_ms = std::max(0.0f, tot - h2d - gu - dn - d2h - sh_ms);
    if (official) {  // moe.rs:1612-1650
      const size_t shared_bytes =
          shared ? 2 * (intermediate * hidden) + out_dim * intermediate +
                       2 * (intermediate * hidden / 128) + out_dim * intermediate / 128
                 : 0;
      tel->shared_expert_ms = sh_ms;
      tel->routed_fp4_bytes_loaded = loaded;
      tel->routed_fp4_bytes_reused = reused;
      tel->shared_fp8_bytes_loaded = shared_bytes;
      tel->shared_fp8_bytes_reused = 0;
      tel->total_logical_bytes = unique.size() * single_expert_bytes + shared_bytes;
      tel->total_loaded_bytes = loaded + shared_bytes;
      tel->total_reused_bytes = reused;
    }
    tel->bytes_gate = bytes_gate;
    tel->bytes_up = bytes_up;
    tel->bytes_down = bytes_down;
    tel->bytes_per_expert = single_expert_bytes;
    tel->selected_working_set_bytes = unique.size() * single_expert_bytes;
  }
  return OBJB_OK;
}

// Multi-token form: the distinct experts of a pair list are resolved once
// each, in first-appearance order (the cache sees the lookups in that order),
// and every pair runs on its expert's tensors; x and v stay on the device.
// With a cache the experts go in chunks of at most half its capacity: a
// chunk's lookups and uploads (one wait of the stream per chunk), then its
// pair launches, then a release point -- so the next chunk's uploads, on the
// cache's side stream, reuse the slots of the chunk before and overlap this
// chunk's kernels.  A chunk of kTcMinPairs pairs or more on a Q4_0 layer runs
// on the tensor cores.  Ends with a stream synchronize like the single-token
// call (the pinned staging block is reused by the next call).
int execute_pairs(objb_moe_executor* ex, cudaStream_t stream, int fmt, const objb_expert_weights* experts,
                  size_t num_experts, const int32_t* pair_expert, const int32_t* pair_token, const int32_t* pair_out,
                  size_t P, const float* d_x, size_t T, size_t hidden, size_t intermediate, size_t out_dim,
                  size_t layer_id, objb_expert_cache* cache, float* d_v, size_t v_rows, objb_moe_telemetry* tel) {
  DeviceGuard g;
  OBJB_TRY(g.enter(ex->device));
  cudaEvent_t* ev = ex->ev;
  OBJB_CUDA(cudaEventRecord(ev[0], stream), "record total start");
  // distinct experts, first appearance order -> table slot
  std::vector<int32_t> slot_of(num_experts, -1);
  std::vector<int32_t> uniq;
  for (size_t p = 0; p < P; ++p) {
    const int32_t e = pair_expert[p];
    if (slot_of[e] < 0) {
      slot_of[e] = static_cast<int32_t>(uniq.size());
      uniq.push_back(e);
    }
  }
  const size_t U = uniq.size();
  // chunks of experts
  size_t C = U;
  if (cache && U) {
    const objb_expert_weights& e0 = experts[uniq[0]];
    const size_t eb = e0.w_gate_len + e0.w_up_len + e0.w_down_len;
    const size_t cap = cache->st.capacity_bytes;
    C = std::max<size_t>(1, std::min(U, eb ? cap / (2 * eb) : U));
  }
  const size_t nchunks = U ? (U + C - 1) / C : 0;
  // pairs ordered by slot (chunks contiguous, grouped by expert; stable)
  std::vector<size_t> start(U + 1, 0);
  for (size_t p = 0; p < P; ++p) start[slot_of[pair_expert[p]] + 1] += 1;
  for (size_t u = 0; u < U; ++u) start[u + 1] += start[u];
  std::vector<int32_t> order(P);
  {
    std::vector<size_t> cur(start.begin(), start.end() - 1);
    for (size_t p = 0; p < P; ++p) order[cur[slot_of[pair_expert[p]]]++] = static_cast<int32_t>(p);
  }
  // one table block per chunk: 3 * U_c pointers, then pe / pt / po of its pairs
  std::vector<size_t> meta_off(nchunks + 1, 0);
  for (size_t c = 0; c < nchunks; ++c) {
    const size_t u0 = c * C, u1 = std::min(U, u0 + C);
    const size_t pc = start[u1] - start[u0];
    meta_off[c + 1] = meta_off[c] + ((u1 - u0) * 3 * sizeof(void*) + 3 * pc * sizeof(int32_t) + 255) / 256 * 256;
  }
  const bool tc_shape = fmt == OBJB_Q4_0 && hidden % 256 == 0 && intermediate % 256 == 0;
  int rc = OBJB_OK;
  size_t need = 0;
  for (size_t c = 0; c < nchunks && rc == OBJB_OK; ++c) {  // scratch for the largest chunk, grown before any launch
    const size_t u0 = c * C, u1 = std::min(U, u0 + C);
    const size_t pc = start[u1] - start[u0];
    objb_moe_layer probe = {};  // the shape only: the sizes do not read the tables
    static const void* const kNoTable[1] = {nullptr};
    probe.fmt = fmt;
    probe.hidden = hidden;
    probe.intermediate = intermediate;
    probe.out_dim = out_dim;
    probe.num_experts = u1 - u0;
    probe.d_gate = probe.d_up = probe.d_down = kNoTable;
    size_t n = 0;
    rc = (tc_shape && pc >= kTcMinPairs) ? moe_pairs_tc_scratch_bytes(&probe, pc, T, &n)
                                         : moe_pairs_scratch_bytes(&probe, pc, T, &n);
    need = std::max(need, n);
  }
  if (rc == OBJB_OK) rc = grow_host(&ex->h_meta, &ex->h_meta_cap, std::max<size_t>(meta_off[nchunks], 64));
  if (rc == OBJB_OK) rc = grow_dev(&ex->d_meta, &ex->d_meta_cap, std::max<size_t>(meta_off[nchunks], 64), "allocate MoE tables");
  if (rc == OBJB_OK) rc = grow_dev(&ex->d_scratch, &ex->d_scratch_cap, std::max<size_t>(need, 256), "allocate MoE scratch");
  Resolved res;
  std::vector<const void*> ptrs(U * 3, nullptr);
  bool first = true;
  for (size_t c = 0; c < nchunks && rc == OBJB_OK; ++c) {
    const size_t u0 = c * C, u1 = std::min(U, u0 + C), uc = u1 - u0;
    if (cache) {
      std::lock_guard<std::mutex> lk(cache->mu);
      cache_begin_batch(cache);
    }
    for (size_t u = u0; u < u1 && rc == OBJB_OK; ++u) {
      const objb_expert_weights& e = experts[uniq[u]];
      TensorRef t[3] = {TensorRef{e.w_gate, e.w_gate_len, OBJB_KIND_GATE, false},
                        TensorRef{e.w_up, e.w_up_len, OBJB_KIND_UP, false},
                        TensorRef{e.w_down, e.w_down_len, OBJB_KIND_DOWN, false}};
      rc = resolve_expert(cache, stream, fmt, false, layer_id, static_cast<size_t>(uniq[u]), t, &ptrs[u * 3], &res);
    }
    if (cache) {
      std::lock_guard<std::mutex> lk(cache->mu);
      const int r2 = cache_end_batch(cache, stream);  // the stream waits for this chunk's uploads
      if (rc == OBJB_OK) rc = r2;
    }
    if (rc != OBJB_OK) break;
    uint32_t flags = 0;
    for (size_t u = u0; u < u1; ++u)
      for (int i = 0; i < 3; ++i)
        if (reinterpret_cast<uintptr_t>(ptrs[u * 3 + i]) & 15u) flags |= OBJB_MOE_UNALIGNED;
    const size_t p0 = start[u0], pc = start[u1] - p0;
    uint8_t* h = static_cast<uint8_t*>(ex->h_meta) + meta_off[c];
    uint8_t* d = static_cast<uint8_t*>(ex->d_meta) + meta_off[c];
    const void** tab = reinterpret_cast<const void**>(h);
    for (int i = 0; i < 3; ++i)
      for (size_t u = 0; u < uc; ++u) tab[i * uc + u] = ptrs[(u0 + u) * 3 + i];
    int32_t* pe = reinterpret_cast<int32_t*>(h + uc * 3 * sizeof(void*));
    int32_t* pt = pe + pc;
    int32_t* po = pt + pc;
    for (size_t q = 0; q < pc; ++q) {
      const int32_t p = order[p0 + q];
      pe[q] = slot_of[pair_expert[p]] - static_cast<int32_t>(u0);
      pt[q] = pair_token[p];
      po[q] = pair_out ? pair_out[p] : p;
    }
    const size_t bytes = uc * 3 * sizeof(void*) + 3 * pc * sizeof(int32_t);
    OBJB_CUDA(cudaMemcpyAsync(d, h, bytes, cudaMemcpyHostToDevice, stream), "copy MoE tables");
    const void* const* dtab = reinterpret_cast<const void* const*>(d);
    const int32_t* d_pe = reinterpret_cast<const int32_t*>(d + uc * 3 * sizeof(void*));
    objb_moe_layer layer = {};
    layer.fmt = fmt;
    layer.flags = flags;
    layer.hidden = hidden;
    layer.intermediate = intermediate;
    layer.out_dim = out_dim;
    layer.num_experts = uc;
    layer.d_gate = dtab;
    layer.d_up = dtab + uc;
    layer.d_down = dtab + 2 * uc;
    if (first) {
      cudaEventRecord(ev[2], stream);
      cudaEventRecord(ev[3], stream);
      first = false;
    }
    if (tc_shape && pc >= kTcMinPairs && !(flags & OBJB_MOE_UNALIGNED))
      rc = moe_pairs_tc(&layer, pc, d_pe, d_pe + pc, d_pe + 2 * pc, T, d_x, d_v, v_rows, 0.0f, stream, ex->d_scratch,
                        ex->d_scratch_cap, nullptr, nullptr);
    else
      rc = moe_pairs(&layer, pc, d_pe, d_pe + pc, d_pe + 2 * pc, T, d_x, d_v, v_rows, 0.0f, stream, ex->d_scratch,
                     ex->d_scratch_cap);
    if (cache) {  // release point: this chunk's tensors are read by work already enqueued
      std::lock_guard<std::mutex> lk(cache->mu);
      const int r2 = cache_release(cache, stream);
      if (rc == OBJB_OK) rc = r2;
    }
  }
  if (first) {
    cudaEventRecord(ev[2], stream);
    cudaEventRecord(ev[3], stream);
  }
  cudaEventRecord(ev[5], stream);
  for (void* p : res.transients) cudaFreeAsync(p, stream);
  cudaError_t se = cudaStreamSynchronize(stream);
  if (rc != OBJB_OK) return rc;
  if (se != cudaSuccess) return cuda_status(se, "synchronize MoE stream", __FILE__, __LINE__);
  {
    unsigned* w = nullptr;
    OBJB_TRY(device_error_word(ex->device, &w));
    unsigned v = 0;
    OBJB_CUDA(cudaMemcpy(&v, w, sizeof(v), cudaMemcpyDeviceToHost), "read device error word");
    if (v) {
      cudaMemset(w, 0, sizeof(unsigned));
      return OBJB_FAIL(OBJB_ERR_INTERNAL, "run multi-token MoE", "device error word " + std::to_string(v));
    }
  }
  const size_t logical = res.bytes_gate + res.bytes_up + res.bytes_down;
  const size_t loaded = res.weight_loaded + res.scale_loaded, reused = res.weight_reused + res.scale_reused;
  if (logical != loaded + reused)
    return OBJB_FAIL(OBJB_ERR_INTERNAL, "account MoE bytes", "MoE Byte invariant violated!");
  if (tel) {
    std::memset(tel, 0, sizeof(*tel));
    float h2d = 0, comp = 0, tot = 0;
    cudaEventElapsedTime(&h2d, ev[0], ev[2]);
    cudaEventElapsedTime(&comp, ev[3], ev[5]);
    cudaEventElapsedTime(&tot, ev[0], ev[5]);
    tel->selected_expert_count = U;
    tel->logical_expert_bytes_requested = logical;
    tel->actual_expert_bytes_loaded = loaded;
    tel->resident_cache_bytes_reused = reused;
    tel->weight_bytes_loaded = res.weight_loaded;
    tel->weight_bytes_reused = res.weight_reused;
    if (cache) {
      std::lock_guard<std::mutex> lk(cache->mu);
      const objb_expert_cache_stats& s = cache->st;
      tel->resident_cache_resident_bytes = s.resident_bytes;
      tel->resident_cache_capacity_bytes = s.capacity_bytes;
      tel->resident_cache_hit_count = s.hit_count;
      tel->resident_cache_miss_count = s.miss_count;
      tel->resident_cache_eviction_count = s.eviction_count;
      tel->resident_cache_insert_attempt_count = s.cache_insert_attempt_count;
      tel->resident_cache_insert_accept_count = s.cache_insert_accept_count;
      tel->resident_cache_insert_bypass_count = s.cache_insert_bypass_count;
      tel->resident_cache_oversized_tensor_bypass_count = s.oversized_tensor_bypass_count;
      tel->resident_cache_oversized_expert_bypass_count = s.oversized_expert_bypass_count;
      tel->resident_cache_self_eviction_risk_count = s.self_eviction_risk_count;
    }
    tel->h2d_ms = h2d;               // until the first chunk's uploads landed
    tel->gate_up_qgemv_ms = comp;  // from there: the pairs of every chunk, overlapped with the later uploads
    tel->total_ms = tot;
    tel->unaccounted_ms = std::max(0.0f, tot - h2d - comp);
    tel->bytes_gate = res.bytes_gate;
    tel->bytes_up = res.bytes_up;
    tel->bytes_down = res.bytes_down;
    tel->bytes_per_expert = U ? logical / U : 0;
    tel->selected_working_set_bytes = logical;
  }
  return OBJB_OK;
}

int validate_common(size_t x_len, size_t hidden, size_t intermediate, const char* which) {
  if (x_len != hidden)
    return OBJB_FAIL(OBJB_ERR_INVALID_INPUT, (std::string("validate ") + which + " input x size").c_str(),
                     "x len " + std::to_string(x_len) + " != hidden " + std::to_string(hidden));
  if (hidden % 32 || intermediate % 32)
    return OBJB_FAIL(OBJB_ERR_INVALID_INPUT, (std::string("validate ") + which + " shape").c_str(),
                     "hidden and intermediate must be multiples of block_size 32");
  return OBJB_OK;
}

int check_index(int64_t e, size_t n) {
  if (e < 0 || static_cast<size_t>(e) >= n)
    return OBJB_FAIL(OBJB_ERR_INVALID_INPUT, "validate expert index",
                     "expert index " + std::to_string(e) + " out of bounds (len=" + std::to_string(n) + ")");
  return OBJB_OK;
}

}  // namespace
}  // namespace objb

using namespace objb;

extern "C" {

int objb_moe_executor_new(int device, objb_moe_executor** out) {
  clear_error();
  if (!out) return OBJB_FAIL(OBJB_ERR_INVALID_INPUT, "objb_moe_executor_new", "null output pointer");
  DeviceProps props;
  OBJB_TRY(device_props(device, &props));
  auto* ex = new objb_moe_executor();
  ex->device = device;
  DeviceGuard g;
  int rc = g.enter(device);
  for (auto& e : ex->ev)
    if (rc == OBJB_OK && cudaEventCreate(&e) != cudaSuccess)
      rc = OBJB_FAIL(OBJB_ERR_RUNTIME, "create executor events", "cudaEventCreate failed");
  if (rc != OBJB_OK) {
    delete ex;
    return rc;
  }
  *out = ex;
  return OBJB_OK;
}

void objb_moe_executor_free(objb_moe_executor* ex) {
  if (!ex) return;
  DeviceGuard g;
  g.enter(ex->device);
  cudaDeviceSynchronize();
  for (auto& e : ex->ev)
    if (e) cudaEventDestroy(e);
  if (ex->d_x) cudaFree(ex->d_x);
  if (ex->d_out) cudaFree(ex->d_out);
  if (ex->d_meta) cudaFree(ex->d_meta);
  if (ex->d_scratch) cudaFree(ex->d_scratch);
  if (ex->h_meta) cudaFreeHost(ex->h_meta);
  delete ex;
}

int objb_moe_executor_compile(objb_moe_executor* ex) {
  clear_error();
  if (!ex) return OBJB_FAIL(OBJB_ERR_INVALID_INPUT, "objb_moe_executor_compile", "null executor");
  return OBJB_OK;  // kernels are prebuilt for sm_100a and loaded with the library
}

int objb_moe_execute_selected(objb_moe_executor* ex, objb_stream_t stream, int fmt, const objb_expert_weights* experts,
                              size_t num_experts, const int64_t* sel_ids, const float* sel_weights,
                              size_t num_selected, const float* x, size_t x_len, size_t hidden, size_t intermediate,
                              size_t out_dim, size_t layer_id, objb_expert_cache* cache, float* out,
                              objb_moe_telemetry* tel) {
  clear_error();
  if (!ex || !out || !x) return OBJB_FAIL(OBJB_ERR_INVALID_INPUT, "objb_moe_execute_selected", "null argument");
  if (fmt != OBJB_Q4_0 && fmt != OBJB_Q5_0 && fmt != OBJB_IQ3_0)
    return OBJB_FAIL(OBJB_ERR_UNSUPPORTED, "objb_moe_execute_selected",
                     "interleaved-block MoE supports Q4_0, Q5_0 and IQ3_0 (use the native FP4 entry point)");
  std::lock_guard<std::mutex> lk(ex->mu);
  OBJB_TRY(validate_common(x_len, hidden, intermediate, "execute_selected_moe_cuda"));
  const size_t bb = static_cast<size_t>(block_bytes(fmt));
  const size_t gu = intermediate * (hidden / 32) * bb;
  const size_t dn = out_dim * (intermediate / 32) * bb;
  for (size_t k = 0; k < num_selected; ++k) {
    OBJB_TRY(check_index(sel_ids[k], num_experts));
    const objb_expert_weights& e = experts[sel_ids[k]];
    if (e.w_gate_len != gu) return fail_len("w_gate", e.w_gate_len, gu);
    if (e.w_up_len != gu) return fail_len("w_up", e.w_up_len, gu);
    if (e.w_down_len != dn) return fail_len("w_down", e.w_down_len, dn);
  }
  auto tensors_of = [&](size_t k, TensorRef* t) {
    const objb_expert_weights& e = experts[sel_ids[k]];
    t[0] = TensorRef{e.w_gate, e.w_gate_len, OBJB_KIND_GATE, false};
    t[1] = TensorRef{e.w_up, e.w_up_len, OBJB_KIND_UP, false};
    t[2] = TensorRef{e.w_down, e.w_down_len, OBJB_KIND_DOWN, false};
  };
  return execute(ex, static_cast<cudaStream_t>(stream), fmt, false, num_selected, sel_ids, sel_weights, x, hidden,
                 intermediate, out_dim, layer_id, cache, out, tel, 2 * gu + dn, tensors_of);
}

int objb_moe_execute_selected_native_fp4(objb_moe_executor* ex, objb_stream_t stream,
                                         const objb_fp4_expert_weights* experts, size_t num_experts,
                                         const int64_t* sel_ids, const float* sel_weights, size_t num_selected,
                                         const float* x, size_t x_len, size_t hidden, size_t intermediate,
                                         size_t out_dim, size_t layer_id, objb_expert_cache* cache, float* out,
                                         objb_moe_telemetry* tel) {
  clear_error();
  if (!ex || !out || !x) return OBJB_FAIL(OBJB_ERR_INVALID_INPUT, "objb_moe_execute_selected_native_fp4", "null argument");
  std::lock_guard<std::mutex> lk(ex->mu);
  OBJB_TRY(validate_common(x_len, hidden, intermediate, "execute_selected_moe_native_fp4_cuda"));
  const size_t guw = intermediate * (hidden / 2), gus = intermediate * (hidden / 32);
  const size_t dnw = out_dim * (intermediate / 2), dns = out_dim * (intermediate / 32);
  for (size_t k = 0; k < num_selected; ++k) {
    OBJB_TRY(check_index(sel_ids[k], num_experts));
    const objb_fp4_expert_weights& e = experts[sel_ids[k]];
    if (e.gate_weight_len != guw) return fail_len("gate_weight", e.gate_weight_len, guw);
    if (e.gate_scale_len != gus) return fail_len("gate_scale", e.gate_scale_len, gus);
    if (e.up_weight_len != guw) return fail_len("up_weight", e.up_weight_len, guw);
    if (e.up_scale_len != gus) return fail_len("up_scale", e.up_scale_len, gus);
    if (e.down_weight_len != dnw) return fail_len("down_weight", e.down_weight_len, dnw);
    if (e.down_scale_len != dns) return fail_len("down_scale", e.down_scale_len, dns);
  }
  auto tensors_of = [&](size_t k, TensorRef* t) {
    const objb_fp4_expert_weights& e = experts[sel_ids[k]];
    t[0] = TensorRef{e.gate_weight, e.gate_weight_len, OBJB_KIND_GATE_WEIGHT, false};
    t[1] = TensorRef{e.gate_scale, e.gate_scale_len, OBJB_KIND_GATE_SCALE, true};
    t[2] = TensorRef{e.up_weight, e.up_weight_len, OBJB_KIND_UP_WEIGHT, false};
    t[3] = TensorRef{e.up_scale, e.up_scale_len, OBJB_KIND_UP_SCALE, true};
    t[4] = TensorRef{e.down_weight, e.down_weight_len, OBJB_KIND_DOWN_WEIGHT, false};
    t[5] = TensorRef{e.down_scale, e.down_scale_len, OBJB_KIND_DOWN_SCALE, true};
  };
  return execute(ex, static_cast<cudaStream_t>(stream), OBJB_FP4_E2M1, true, num_selected, sel_ids, sel_weights, x,
                 hidden, intermediate, out_dim, layer_id, cache, out, tel, 2 * (guw + gus) + dnw + dns, tensors_of);
}

int objb_moe_execute_pairs(objb_moe_executor* ex, objb_stream_t stream, int fmt, const objb_expert_weights* experts,
                           size_t num_experts, const int32_t* pair_expert, const int32_t* pair_token,
                           const int32_t* pair_out, size_t num_pairs, const float* d_x, size_t num_tokens,
                           size_t hidden, size_t intermediate, size_t out_dim, size_t layer_id,
                           objb_expert_cache* cache, float* d_v, size_t v_rows, objb_moe_telemetry* tel) {
  clear_error();
  if (!ex || !experts || !pair_expert || !pair_token || !d_x || !d_v)
    return OBJB_FAIL(OBJB_ERR_INVALID_INPUT, "objb_moe_execute_pairs", "null argument");
  if (fmt != OBJB_Q4_0 && fmt != OBJB_Q5_0 && fmt != OBJB_IQ3_0)
    return OBJB_FAIL(OBJB_ERR_UNSUPPORTED, "objb_moe_execute_pairs",
                     "the multi-token executor supports Q4_0, Q5_0 and IQ3_0 experts");
  if (num_pairs == 0 || num_tokens == 0 || num_experts == 0 || num_experts > (1u << 20))
    return OBJB_FAIL(OBJB_ERR_INVALID_INPUT, "objb_moe_execute_pairs", "empty pair list, tokens or experts");
  std::lock_guard<std::mutex> lk(ex->mu);
  OBJB_TRY(validate_common(hidden, hidden, intermediate, "execute_pairs"));
  const size_t bb = static_cast<size_t>(block_bytes(fmt));
  const size_t gu = intermediate * (hidden / 32) * bb;
  const size_t dn = out_dim * (intermediate / 32) * bb;
  for (size_t p = 0; p < num_pairs; ++p) {
    OBJB_TRY(check_index(pair_expert[p], num_experts));
    if (pair_token[p] < 0 || static_cast<size_t>(pair_token[p]) >= num_tokens)
      return OBJB_FAIL(OBJB_ERR_INVALID_INPUT, "validate pair token",
                       "token index " + std::to_string(pair_token[p]) + " out of bounds (len=" +
                           std::to_string(num_tokens) + ")");
    const size_t row = pair_out ? static_cast<size_t>(pair_out[p]) : p;
    if ((pair_out && pair_out[p] < 0) || row >= v_rows)
      return OBJB_FAIL(OBJB_ERR_INVALID_INPUT, "validate pair output row",
                       "output row " + std::to_string(row) + " out of bounds (v_rows=" + std::to_string(v_rows) + ")");
    const objb_expert_weights& e = experts[pair_expert[p]];
    if (e.w_gate_len != gu) return fail_len("w_gate", e.w_gate_len, gu);
    if (e.w_up_len != gu) return fail_len("w_up", e.w_up_len, gu);
    if (e.w_down_len != dn) return fail_len("w_down", e.w_down_len, dn);
  }
  return execute_pairs(ex, static_cast<cudaStream_t>(stream), fmt, experts, num_experts, pair_expert, pair_token,
                       pair_out, num_pairs, d_x, num_tokens, hidden, intermediate, out_dim, layer_id, cache, d_v,
                       v_rows, tel);
}

int objb_moe_execute_selected_official_fp4(objb_moe_executor* ex, objb_stream_t stream,
                                           const objb_fp4_expert_weights* experts, size_t num_experts,
                                           const int64_t* sel_ids, const float* sel_weights, size_t num_selected,
                                           const float* x, size_t x_len, size_t hidden, size_t intermediate,
                                           size_t out_dim, size_t layer_id, objb_expert_cache* cache,
                                           const objb_fp8_shared_expert* shared, float* out,
                                           objb_moe_telemetry* tel) {
  clear_error();
  if (!ex || !out || !x)
    return OBJB_FAIL(OBJB_ERR_INVALID_INPUT, "objb_moe_execute_selected_official_fp4", "null argument");
  std::lock_guard<std::mutex> lk(ex->mu);
  OBJB_TRY(validate_common(x_len, hidden, intermediate, "execute_selected_moe_official_routed_fp4_cuda"));
  if (hidden % 128 || intermediate % 128)
    return OBJB_FAIL(OBJB_ERR_INVALID_INPUT, "validate official MoE shape",
                     "hidden and intermediate must be multiples of 128 (act_quant blocks)");
  const size_t guw = intermediate * (hidden / 2), gus = intermediate * (hidden / 32);
  const size_t dnw = out_dim * (intermediate / 2), dns = out_dim * (intermediate / 32);
  for (size_t k = 0; k < num_selected; ++k) {
    OBJB_TRY(check_index(sel_ids[k], num_experts));
    const objb_fp4_expert_weights& e = experts[sel_ids[k]];
    if (e.gate_weight_len != guw) return fail_len("gate_weight", e.gate_weight_len, guw);
    if (e.gate_scale_len != gus) return fail_len("gate_scale", e.gate_scale_len, gus);
    if (e.up_weight_len != guw) return fail_len("up_weight", e.up_weight_len, guw);
    if (e.up_scale_len != gus) return fail_len("up_scale", e.up_scale_len, gus);
    if (e.down_weight_len != dnw) return fail_len("down_weight", e.down_weight_len, dnw);
    if (e.down_scale_len != dns) return fail_len("down_scale", e.down_scale_len, dns);
  }
  auto tensors_of = [&](size_t k, TensorRef* t) {
    const objb_fp4_expert_weights& e = experts[sel_ids[k]];
    t[0] = TensorRef{e.gate_weight, e.gate_weight_len, OBJB_KIND_GATE_WEIGHT, false};
    t[1] = TensorRef{e.gate_scale, e.gate_scale_len, OBJB_KIND_GATE_SCALE, true};
    t[2] = TensorRef{e.up_weight, e.up_weight_len, OBJB_KIND_UP_WEIGHT, false};
    t[3] = TensorRef{e.up_scale, e.up_scale_len, OBJB_KIND_UP_SCALE, true};
    t[4] = TensorRef{e.down_weight, e.down_weight_len, OBJB_KIND_DOWN_WEIGHT, false};
    t[5] = TensorRef{e.down_scale, e.down_scale_len, OBJB_KIND_DOWN_SCALE, true};
  };
  Official off;
  off.shared = shared;
  return execute(ex, static_cast<cudaStream_t>(stream), OBJB_FP4_E2M1, true, num_selected, sel_ids, sel_weights, x,
                 hidden, intermediate, out_dim, layer_id, cache, out, tel, 2 * (guw + gus) + dnw + dns, tensors_of,
                 &off);
}

}  // extern "C"
