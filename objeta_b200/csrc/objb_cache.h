// objb_cache.h -- the device expert cache (CudaExpertCache, moe.rs:70-227).
//
// Bookkeeping (keys, LRU order, pins, every counter) follows the reference
// state machine step for step, so hit / miss / evict sequences are identical.
// Storage is B200-side: one device arena of the cache's capacity carved into
// size-class slots (all tensors of one kind in a layer have one size, so the
// arena does not fragment in practice); a slot that does not fit is allocated
// on its own ("overflow").  Uploads run on a cache-owned side stream and the
// caller's stream waits on an event, so misses stream in asynchronously from
// pinned host memory.  An evicted slot is not reused until the stream that
// read it passes a release point (release()), which is what keeps a buffer
// alive for the rest of a call in the reference (Arc<DeviceBuffer>).  Release
// points close "epochs": an entry remembers the epoch it was last handed out
// in, and when it is evicted after that epoch was closed its slot is free at
// once, the upload stream waiting (on the device) for that epoch's release
// event -- so a multi-token call that resolves its experts in chunks, with a
// release point after each chunk's launches, reuses the slots of chunk i - 1
// for chunk i + 1 while chunk i computes.
#pragma once

#include <cuda_runtime.h>

#include <cstddef>
#include <cstdint>
#include <deque>
#include <list>
#include <map>
#include <memory>
#include <mutex>
#include <set>
#include <unordered_map>
#include <vector>

#include "../../include/objeta_b200.h"

struct objb_expert_cache {
  struct Key {
    size_t layer, expert;
    int32_t kind, fmt;
    bool operator==(const Key& o) const {
      return layer == o.layer && expert == o.expert && kind == o.kind && fmt == o.fmt;
    }
  };
  struct KeyHash {
    size_t operator()(const Key& k) const {
      size_t h = k.layer * 0x9E3779B97F4A7C15ull;
      h ^= k.expert + 0x7F4A7C159E3779B9ull + (h << 6) + (h >> 2);
      h ^= static_cast<size_t>(k.kind) * 0x100000001B3ull + (h << 6) + (h >> 2);
      h ^= static_cast<size_t>(k.fmt) + (h << 6) + (h >> 2);
      return h;
    }
  };
  struct Event {
    cudaEvent_t ev = nullptr;
    ~Event() {
      if (ev) cudaEventDestroy(ev);
    }
  };
  // Device storage of one resident tensor.
  struct Slot {
    void* ptr = nullptr;
    size_t cls = 0;          // size class (bytes, 256-rounded); 0 = overflow allocation
    std::shared_ptr<Event> ready;  // reads of the previous owner finished (reuse fence)
  };
  struct Entry {
    Slot slot;
    size_t size = 0;
    uint64_t last_epoch = 0;  // epoch in which it was last handed out (get hit or insert)
  };

  int device = 0;
  std::mutex mu;
  objb_expert_cache_stats st = {};
  std::unordered_map<Key, Entry, KeyHash> map;
  std::list<Key> order;  // LRU order, front = least recent (may hold duplicates, as the reference's Vec)
  std::unordered_map<Key, bool, KeyHash> pinned;

  // storage
  uint8_t* arena = nullptr;
  size_t arena_bytes = 0, bump = 0;
  std::map<size_t, std::vector<Slot>> free_slots;  // size class -> reusable slots
  std::vector<Slot> pending;                       // evicted, waiting for a release point
  std::vector<void*> transients;                   // bypass buffers of the current epoch
  cudaStream_t side = nullptr;
  size_t overflow_allocations = 0;

  // epochs (release points)
  uint64_t epoch = 0;
  std::deque<std::pair<uint64_t, std::shared_ptr<Event>>> closed;  // (epoch, its release event), oldest first
  std::shared_ptr<Event> side_waited;  // the last fence the upload stream waited on (skip repeats)

  // uploads of a batch: the caller's stream waits once, after the batch
  bool defer_wait = false;
  bool uploads_pending = false;
  cudaEvent_t upload_ev = nullptr;
};
