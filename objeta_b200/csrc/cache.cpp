// cache.cpp -- CudaExpertCache (moe.rs:70-227) on the device: reference LRU /
// admission bookkeeping over a slab arena with stream-ordered slot reuse.
#include <cuda_runtime.h>

#include <algorithm>
#include <string>

#include "objb_cache.h"
#include "objb_common.h"

using Cache = objb_expert_cache;

namespace objb {
namespace {

constexpr size_t kClassAlign = 256;

size_t size_class(size_t bytes) { return std::max<size_t>(kClassAlign, (bytes + kClassAlign - 1) / kClassAlign * kClassAlign); }

Cache::Key to_key(const objb_expert_cache_key* k) {
  return Cache::Key{k->layer_id, k->expert_id, k->tensor_kind, k->quant_format};
}

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

int ensure_side(Cache* c) {
  if (c->side) return OBJB_OK;
  OBJB_CUDA(cudaStreamCreateWithFlags(&c->side, cudaStreamNonBlocking), "create cache upload stream");
  OBJB_CUDA(cudaEventCreateWithFlags(&c->upload_ev, cudaEventDisableTiming), "create upload event");
  return OBJB_OK;
}

// The upload stream waits for `ev` (skipped when it just did: the event is
// kept alive, so its handle cannot have been reused meanwhile).
int side_wait(Cache* c, const std::shared_ptr<Cache::Event>& ev) {
  if (!ev || !ev->ev || ev == c->side_waited) return OBJB_OK;
  OBJB_CUDA(cudaStreamWaitEvent(c->side, ev->ev, 0), "order slot reuse after its last reads");
  c->side_waited = ev;
  return OBJB_OK;
}

// The release event that closed `epoch`, or a later one (still a valid fence)
// when that one has been dropped from the window.
std::shared_ptr<Cache::Event> fence_of(Cache* c, uint64_t epoch) {
  for (auto& e : c->closed)
    if (e.first >= epoch) return e.second;
  return nullptr;
}

// Storage for `bytes`: a free slot of the same class (its reuse fence is
// waited on by the upload stream), else fresh arena space, else an overflow
// allocation of its own.
int alloc_slot(Cache* c, size_t bytes, Cache::Slot* out) {
  const size_t cls = size_class(bytes);
  auto it = c->free_slots.find(cls);
  if (it != c->free_slots.end() && !it->second.empty()) {
    *out = it->second.back();
    it->second.pop_back();
    if (out->ready) OBJB_TRY(side_wait(c, out->ready));
    out->ready.reset();
    return OBJB_OK;
  }
  if (!c->arena && c->st.capacity_bytes > 0) {
    const size_t want = size_class(c->st.capacity_bytes) + kClassAlign;
    if (cudaMalloc(&c->arena, want) == cudaSuccess) {
      c->arena_bytes = want;
    } else {
      cudaGetLastError();
      c->arena = nullptr;
    }
  }
  if (c->arena && c->bump + cls <= c->arena_bytes) {
    out->ptr = reinterpret_cast<void*>(reinterpret_cast<uint8_t*>(c->arena) + c->bump);
    out->cls = cls;
    out->ready.reset();
    c->bump += cls;
    return OBJB_OK;
  }
  void* p = nullptr;
  OBJB_CUDA(cudaMallocAsync(&p, cls, c->side), "allocate overflow cache slot");
  ++c->overflow_allocations;
  out->ptr = p;
  out->cls = 0;
  out->ready.reset();
  return OBJB_OK;
}

// A slot whose entry was last handed out in `last_epoch`: free at once behind
// that epoch's release event when the epoch is closed, else pending until the
// next release point.
void retire_slot(Cache* c, const Cache::Slot& s, uint64_t last_epoch) {
  if (!s.ptr) return;
  if (last_epoch < c->epoch && s.cls != 0) {
    auto f = fence_of(c, last_epoch);
    if (f) {
      Cache::Slot r = s;
      r.ready = f;
      c->free_slots[r.cls].push_back(r);
      return;
    }
  }
  c->pending.push_back(s);
}

// evict_lru (moe.rs:164-176): removes the first non-pinned key from the LRU
// order and, when it is still mapped, evicts it.  kNone: only pinned keys
// (or nothing) left; kStale: a key that was no longer mapped was dropped from
// the order (the reference returns None there too, but has made progress).
enum EvictResult { kEvicted, kStale, kNone };
EvictResult evict_lru_ex(Cache* c, Cache::Key* evicted) {
  for (auto it = c->order.begin(); it != c->order.end(); ++it) {
    if (c->pinned.count(*it)) continue;
    const Cache::Key k = *it;
    c->order.erase(it);
    auto m = c->map.find(k);
    if (m != c->map.end()) {
      c->st.resident_bytes -= m->second.size;
      c->st.eviction_count += 1;
      retire_slot(c, m->second.slot, m->second.last_epoch);
      c->map.erase(m);
      if (evicted) *evicted = k;
      return kEvicted;
    }
    return kStale;
  }
  return kNone;
}
bool evict_lru(Cache* c, Cache::Key* evicted) { return evict_lru_ex(c, evicted) == kEvicted; }

void touch(Cache* c, const Cache::Key& k) {
  for (auto it = c->order.begin(); it != c->order.end(); ++it) {
    if (*it == k) {
      c->order.erase(it);
      c->order.push_back(k);
      return;
    }
  }
}

// The caller's stream waits for the uploads issued so far.
int flush_uploads(Cache* c, cudaStream_t stream) {
  if (!c->uploads_pending) return OBJB_OK;
  OBJB_CUDA(cudaEventRecord(c->upload_ev, c->side), "record uploads");
  OBJB_CUDA(cudaStreamWaitEvent(stream, c->upload_ev, 0), "order uploads before use");
  c->uploads_pending = false;
  return OBJB_OK;
}

int upload(Cache* c, void* dst, const void* host, size_t bytes, cudaStream_t stream) {
  OBJB_TRY(ensure_side(c));
  if (bytes) OBJB_CUDA(cudaMemcpyAsync(dst, host, bytes, cudaMemcpyHostToDevice, c->side), "upload expert tensor");
  c->uploads_pending = true;
  return c->defer_wait ? OBJB_OK : flush_uploads(c, stream);
}

// insert (moe.rs:124-154).
int insert(Cache* c, const Cache::Key& k, const void* host, size_t bytes, cudaStream_t stream, const void** out,
           int* resident) {
  c->st.cache_insert_attempt_count += 1;
  if (bytes > c->st.capacity_bytes) {
    c->st.oversized_tensor_bypass_count += 1;
    c->st.cache_insert_bypass_count += 1;
    void* p = nullptr;
    OBJB_CUDA(cudaMallocAsync(&p, std::max<size_t>(bytes, 16), stream), "allocate bypass buffer");
    c->transients.push_back(p);
    if (bytes) OBJB_CUDA(cudaMemcpyAsync(p, host, bytes, cudaMemcpyHostToDevice, stream), "upload bypassed tensor");
    *out = p;
    if (resident) *resident = 0;
    return OBJB_OK;
  }
  c->st.cache_insert_accept_count += 1;
  auto old = c->map.find(k);
  if (old != c->map.end()) {
    c->st.resident_bytes -= old->second.size;
    retire_slot(c, old->second.slot, old->second.last_epoch);
    c->map.erase(old);
    for (auto it = c->order.begin(); it != c->order.end(); ++it)
      if (*it == k) {
        c->order.erase(it);
        break;
      }
  }
  // The reference loops while anything is left in `order`; when only pinned
  // keys remain it would spin forever, so stop there instead.
  while (c->st.resident_bytes + bytes > c->st.capacity_bytes && !c->order.empty()) {
    if (evict_lru_ex(c, nullptr) == kNone) break;
  }
  Cache::Entry e;
  e.size = bytes;
  e.last_epoch = c->epoch;
  OBJB_TRY(ensure_side(c));
  OBJB_TRY(alloc_slot(c, bytes, &e.slot));
  OBJB_TRY(upload(c, e.slot.ptr, host, bytes, stream));
  c->map[k] = e;
  c->st.resident_bytes += bytes;
  c->order.push_back(k);
  *out = e.slot.ptr;
  if (resident) *resident = 1;
  return OBJB_OK;
}

int get(Cache* c, const Cache::Key& k, const void** out) {
  auto it = c->map.find(k);
  if (it != c->map.end()) {
    c->st.hit_count += 1;
    touch(c, k);
    it->second.last_epoch = c->epoch;
    *out = it->second.slot.ptr;
  } else {
    c->st.miss_count += 1;
    *out = nullptr;
  }
  return OBJB_OK;
}

// A release point: everything handed out so far is read by work already
// enqueued on `stream`; closes the epoch.
int release(Cache* c, cudaStream_t stream) {
  {
    auto ev = std::make_shared<Cache::Event>();
    OBJB_CUDA(cudaEventCreateWithFlags(&ev->ev, cudaEventDisableTiming), "create release event");
    OBJB_CUDA(cudaEventRecord(ev->ev, stream), "record release point");
    c->closed.emplace_back(c->epoch, ev);
    while (c->closed.size() > 64) c->closed.pop_front();
    c->epoch += 1;
    for (auto& s : c->pending) {
      if (s.cls == 0) {
        // overflow slots come from cudaMallocAsync: freed in stream order
        OBJB_CUDA(cudaFreeAsync(s.ptr, stream), "free overflow slot");
      } else {
        s.ready = ev;
        c->free_slots[s.cls].push_back(s);
      }
    }
    c->pending.clear();
  }
  for (void* p : c->transients) OBJB_CUDA(cudaFreeAsync(p, stream), "free bypass buffer");
  c->transients.clear();
  return OBJB_OK;
}

}  // namespace

// Executor hooks (executor.cpp).
int cache_get(Cache* c, const objb_expert_cache_key* k, const void** out) { return get(c, to_key(k), out); }
int cache_insert(Cache* c, const objb_expert_cache_key* k, const void* host, size_t bytes, cudaStream_t stream,
                 const void** out, int* resident) {
  return insert(c, to_key(k), host, bytes, stream, out, resident);
}
int cache_release(Cache* c, cudaStream_t stream) { return release(c, stream); }
// A batch of lookups whose uploads the caller's stream waits for once, at
// cache_end_batch (the executor's chunks).
void cache_begin_batch(Cache* c) { c->defer_wait = true; }
int cache_end_batch(Cache* c, cudaStream_t stream) {
  c->defer_wait = false;
  if (!c->side) return OBJB_OK;
  return flush_uploads(c, stream);
}

}  // namespace objb

using namespace objb;

#define CACHE_CHECK(c)                                                                       \
  do {                                                                                       \
    clear_error();                                                                           \
    if (!(c)) return OBJB_FAIL(OBJB_ERR_INVALID_INPUT, "expert cache call", "null cache"); \
  } while (0)

extern "C" {

int objb_expert_cache_new(int device, size_t capacity_bytes, objb_expert_cache** out) {
  clear_error();
  if (!out) return OBJB_FAIL(OBJB_ERR_INVALID_INPUT, "objb_expert_cache_new", "null output pointer");
  int count = 0;
  OBJB_CUDA(cudaGetDeviceCount(&count), "count devices");
  if (device < 0 || device >= count)
    return OBJB_FAIL(OBJB_ERR_INVALID_INPUT, "objb_expert_cache_new", "no CUDA device " + std::to_string(device));
  auto* c = new objb_expert_cache();
  c->device = device;
  c->st.capacity_bytes = capacity_bytes;
  *out = c;
  return OBJB_OK;
}

void objb_expert_cache_free(objb_expert_cache* c) {
  if (!c) return;
  DeviceGuard g;
  g.enter(c->device);
  if (c->side) cudaStreamSynchronize(c->side);
  cudaDeviceSynchronize();
  for (auto& kv : c->map)
    if (kv.second.slot.cls == 0 && kv.second.slot.ptr) cudaFree(kv.second.slot.ptr);
  for (auto& s : c->pending)
    if (s.cls == 0 && s.ptr) cudaFree(s.ptr);
  for (void* p : c->transients) cudaFree(p);
  if (c->arena) cudaFree(c->arena);
  if (c->upload_ev) cudaEventDestroy(c->upload_ev);
  if (c->side) cudaStreamDestroy(c->side);
  delete c;
}

int objb_expert_cache_get(objb_expert_cache* c, const objb_expert_cache_key* key, const void** d_ptr) {
  CACHE_CHECK(c);
  if (!key || !d_ptr) return OBJB_FAIL(OBJB_ERR_INVALID_INPUT, "objb_expert_cache_get", "null argument");
  std::lock_guard<std::mutex> lk(c->mu);
  return get(c, to_key(key), d_ptr);
}

int objb_expert_cache_insert(objb_expert_cache* c, const objb_expert_cache_key* key, const void* host_src,
                             size_t bytes, objb_stream_t stream, const void** d_ptr, int* resident) {
  CACHE_CHECK(c);
  if (!key || !d_ptr || (!host_src && bytes))
    return OBJB_FAIL(OBJB_ERR_INVALID_INPUT, "objb_expert_cache_insert", "null argument");
  std::lock_guard<std::mutex> lk(c->mu);
  DeviceGuard g;
  OBJB_TRY(g.enter(c->device));
  return insert(c, to_key(key), host_src, bytes, static_cast<cudaStream_t>(stream), d_ptr, resident);
}

int objb_expert_cache_get_or_insert(objb_expert_cache* c, const objb_expert_cache_key* key, const void* host_src,
                                    size_t bytes, objb_stream_t stream, const void** d_ptr, int* hit) {
  CACHE_CHECK(c);
  if (!key || !d_ptr) return OBJB_FAIL(OBJB_ERR_INVALID_INPUT, "objb_expert_cache_get_or_insert", "null argument");
  std::lock_guard<std::mutex> lk(c->mu);
  const Cache::Key k = to_key(key);
  OBJB_TRY(get(c, k, d_ptr));
  if (*d_ptr) {
    if (hit) *hit = 1;
    return OBJB_OK;
  }
  if (hit) *hit = 0;
  if (!host_src && bytes) return OBJB_FAIL(OBJB_ERR_INVALID_INPUT, "objb_expert_cache_get_or_insert", "null host source");
  DeviceGuard g;
  OBJB_TRY(g.enter(c->device));
  return insert(c, k, host_src, bytes, static_cast<cudaStream_t>(stream), d_ptr, nullptr);
}

int objb_expert_cache_get_or_load(objb_expert_cache* c, const objb_expert_cache_key* key, objb_expert_load_fn load,
                                  void* user, objb_stream_t stream, const void** d_ptr, int* hit) {
  CACHE_CHECK(c);
  if (!key || !d_ptr || !load)
    return OBJB_FAIL(OBJB_ERR_INVALID_INPUT, "objb_expert_cache_get_or_load", "null argument");
  const Cache::Key k = to_key(key);
  {
    std::lock_guard<std::mutex> lk(c->mu);
    OBJB_TRY(get(c, k, d_ptr));
  }
  if (*d_ptr) {
    if (hit) *hit = 1;
    return OBJB_OK;
  }
  if (hit) *hit = 0;
  const void* src = nullptr;
  size_t bytes = 0;
  const int rc = load(user, &src, &bytes);
  if (rc != 0) return rc;
  if (!src && bytes) return OBJB_FAIL(OBJB_ERR_INVALID_INPUT, "objb_expert_cache_get_or_load", "load gave no bytes");
  std::lock_guard<std::mutex> lk(c->mu);
  DeviceGuard g;
  OBJB_TRY(g.enter(c->device));
  return insert(c, k, src, bytes, static_cast<cudaStream_t>(stream), d_ptr, nullptr);
}

int objb_expert_cache_touch(objb_expert_cache* c, const objb_expert_cache_key* key) {
  CACHE_CHECK(c);
  if (!key) return OBJB_FAIL(OBJB_ERR_INVALID_INPUT, "objb_expert_cache_touch", "null key");
  std::lock_guard<std::mutex> lk(c->mu);
  touch(c, to_key(key));
  return OBJB_OK;
}

int objb_expert_cache_evict_lru(objb_expert_cache* c, objb_expert_cache_key* evicted, int* found) {
  CACHE_CHECK(c);
  std::lock_guard<std::mutex> lk(c->mu);
  Cache::Key k{};
  const bool f = evict_lru(c, &k);
  if (found) *found = f ? 1 : 0;
  if (f && evicted) *evicted = objb_expert_cache_key{k.layer, k.expert, k.kind, k.fmt};
  return OBJB_OK;
}

int objb_expert_cache_pin(objb_expert_cache* c, const objb_expert_cache_key* key) {
  CACHE_CHECK(c);
  if (!key) return OBJB_FAIL(OBJB_ERR_INVALID_INPUT, "objb_expert_cache_pin", "null key");
  std::lock_guard<std::mutex> lk(c->mu);
  const Cache::Key k = to_key(key);
  auto it = c->map.find(k);
  if (it != c->map.end() && !c->pinned.count(k)) {
    c->pinned[k] = true;
    c->st.pinned_bytes += it->second.size;
  }
  return OBJB_OK;
}

// insert_pinned (moe.rs:190-205): evicts non-pinned tensors while over
// capacity (stopping when only pinned ones remain), replaces any previous
// buffer of the key and appends the key to the LRU order.
int objb_expert_cache_insert_pinned(objb_expert_cache* c, const objb_expert_cache_key* key, const void* host_src,
                                    size_t bytes, objb_stream_t stream, const void** d_ptr) {
  CACHE_CHECK(c);
  if (!key || !d_ptr || (!host_src && bytes))
    return OBJB_FAIL(OBJB_ERR_INVALID_INPUT, "objb_expert_cache_insert_pinned", "null argument");
  std::lock_guard<std::mutex> lk(c->mu);
  DeviceGuard g;
  OBJB_TRY(g.enter(c->device));
  while (c->st.resident_bytes + bytes > c->st.capacity_bytes && !c->order.empty()) {
    if (!evict_lru(c, nullptr)) break;
  }
  const Cache::Key k = to_key(key);
  Cache::Entry e;
  e.size = bytes;
  e.last_epoch = c->epoch;
  OBJB_TRY(ensure_side(c));
  OBJB_TRY(alloc_slot(c, bytes, &e.slot));
  OBJB_TRY(upload(c, e.slot.ptr, host_src, bytes, static_cast<cudaStream_t>(stream)));
  auto old = c->map.find(k);
  if (old != c->map.end()) {
    c->st.resident_bytes -= old->second.size;
    retire_slot(c, old->second.slot, old->second.last_epoch);
  }
  c->map[k] = e;
  c->st.resident_bytes += bytes;
  c->st.pinned_bytes += bytes;
  c->pinned[k] = true;
  c->order.push_back(k);
  *d_ptr = e.slot.ptr;
  return OBJB_OK;
}

int objb_expert_cache_clear(objb_expert_cache* c) {
  CACHE_CHECK(c);
  std::lock_guard<std::mutex> lk(c->mu);
  for (auto& kv : c->map) retire_slot(c, kv.second.slot, kv.second.last_epoch);
  c->map.clear();
  c->order.clear();
  c->pinned.clear();
  c->st.resident_bytes = 0;
  c->st.pinned_bytes = 0;
  return OBJB_OK;
}

int objb_expert_cache_reset_counters(objb_expert_cache* c) {
  CACHE_CHECK(c);
  std::lock_guard<std::mutex> lk(c->mu);
  c->st.hit_count = c->st.miss_count = c->st.eviction_count = 0;
  c->st.cache_insert_attempt_count = c->st.cache_insert_accept_count = c->st.cache_insert_bypass_count = 0;
  c->st.oversized_tensor_bypass_count = c->st.oversized_expert_bypass_count = c->st.self_eviction_risk_count = 0;
  return OBJB_OK;
}

int objb_expert_cache_stats_get(objb_expert_cache* c, objb_expert_cache_stats* out) {
  CACHE_CHECK(c);
  if (!out) return OBJB_FAIL(OBJB_ERR_INVALID_INPUT, "objb_expert_cache_stats_get", "null output");
  std::lock_guard<std::mutex> lk(c->mu);
  *out = c->st;
  out->overflow_allocations = c->overflow_allocations;
  return OBJB_OK;
}

int objb_expert_cache_set_bypass_oversized_experts(objb_expert_cache* c, int bypass) {
  CACHE_CHECK(c);
  std::lock_guard<std::mutex> lk(c->mu);
  c->st.bypass_oversized_experts = bypass ? 1 : 0;
  return OBJB_OK;
}

int objb_expert_cache_count(objb_expert_cache* c, int which) {
  CACHE_CHECK(c);
  std::lock_guard<std::mutex> lk(c->mu);
  switch (which) {
    case 0: c->st.oversized_expert_bypass_count += 1; break;
    case 1: c->st.self_eviction_risk_count += 1; break;
    case 2:
      c->st.cache_insert_attempt_count += 1;
      c->st.cache_insert_bypass_count += 1;
      break;
    default: return OBJB_FAIL(OBJB_ERR_INVALID_INPUT, "objb_expert_cache_count", "unknown counter");
  }
  return OBJB_OK;
}

int objb_expert_cache_contains(objb_expert_cache* c, const objb_expert_cache_key* key, int* found) {
  CACHE_CHECK(c);
  if (!key || !found) return OBJB_FAIL(OBJB_ERR_INVALID_INPUT, "objb_expert_cache_contains", "null argument");
  std::lock_guard<std::mutex> lk(c->mu);
  *found = c->map.count(to_key(key)) ? 1 : 0;
  return OBJB_OK;
}

int objb_expert_cache_lru_keys(objb_expert_cache* c, objb_expert_cache_key* out, size_t cap, size_t* n) {
  CACHE_CHECK(c);
  if (!n) return OBJB_FAIL(OBJB_ERR_INVALID_INPUT, "objb_expert_cache_lru_keys", "null count");
  std::lock_guard<std::mutex> lk(c->mu);
  size_t i = 0;
  for (const auto& k : c->order) {
    if (out && i < cap) out[i] = objb_expert_cache_key{k.layer, k.expert, k.kind, k.fmt};
    ++i;
  }
  *n = i;
  return OBJB_OK;
}

int objb_expert_cache_release(objb_expert_cache* c, objb_stream_t stream) {
  CACHE_CHECK(c);
  std::lock_guard<std::mutex> lk(c->mu);
  DeviceGuard g;
  OBJB_TRY(g.enter(c->device));
  return release(c, static_cast<cudaStream_t>(stream));
}

}  // extern "C"
