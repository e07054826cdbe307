"""TEST INFRASTRUCTURE ONLY: pure-Python restatement of objeta's expert cache.

Restates ``CudaExpertCache`` (crates/objeta-cuda/src/moe.rs:70-227) and the
per-expert admission / lookup logic of the MoE executors
(moe.rs:483-583 for the Q4 path, moe.rs:753-814 and 993-1087 for the native
FP4 path).  Buffers are replaced by byte sizes: the model tracks keys, LRU
order, pins and every counter, which is what the product cache must reproduce
bit-exactly.  Used only by tests.
"""
from __future__ import annotations

from dataclasses import dataclass, field


@dataclass
class CacheModel:
    capacity_bytes: int
    resident_bytes: int = 0
    pinned_bytes: int = 0
    hit_count: int = 0
    miss_count: int = 0
    eviction_count: int = 0
    bypass_oversized_experts: bool = False
    cache_insert_attempt_count: int = 0
    cache_insert_accept_count: int = 0
    cache_insert_bypass_count: int = 0
    oversized_tensor_bypass_count: int = 0
    oversized_expert_bypass_count: int = 0
    self_eviction_risk_count: int = 0
    pinned: set = field(default_factory=set)
    sizes: dict = field(default_factory=dict)
    order: list = field(default_factory=list)
    events: list = field(default_factory=list)  # ("evict", key) in order

    # moe.rs:113-122
    def get(self, key) -> bool:
        if key in self.sizes:
            self.hit_count += 1
            self.touch(key)
            return True
        self.miss_count += 1
        return False

    # moe.rs:124-154
    def insert(self, key, size: int) -> bool:
        """Returns True when the tensor became resident, False on bypass."""
        self.cache_insert_attempt_count += 1
        if size > self.capacity_bytes:
            self.oversized_tensor_bypass_count += 1
            self.cache_insert_bypass_count += 1
            return False
        self.cache_insert_accept_count += 1
        if key in self.sizes:
            self.resident_bytes -= self.sizes.pop(key)
            if key in self.order:
                self.order.remove(key)
        # The reference loops while the order is non-empty; when only pinned
        # keys remain it would spin forever -- the model (like the product)
        # stops there.  A stale key dropped from the order still counts as
        # progress.
        while self.resident_bytes + size > self.capacity_bytes and self.order:
            if self.evict_lru() is None and not any(k not in self.pinned for k in self.order):
                break
        self.sizes[key] = size
        self.resident_bytes += size
        self.order.append(key)
        return True

    # moe.rs:156-161
    def touch(self, key):
        if key in self.order:
            self.order.remove(key)
            self.order.append(key)

    # moe.rs:164-176: first non-pinned key in LRU order.
    def evict_lru(self):
        for idx, k in enumerate(self.order):
            if k not in self.pinned:
                self.order.pop(idx)
                if k in self.sizes:
                    self.resident_bytes -= self.sizes.pop(k)
                    self.eviction_count += 1
                    self.events.append(("evict", k))
                    return k
                return None
        return None

    # moe.rs:179-186
    def pin(self, key):
        if key in self.sizes and key not in self.pinned:
            self.pinned.add(key)
            self.pinned_bytes += self.sizes[key]

    # moe.rs:190-205
    def insert_pinned(self, key, size: int):
        while self.resident_bytes + size > self.capacity_bytes and self.order:
            if self.evict_lru() is None:
                break
        old = self.sizes.get(key)
        self.sizes[key] = size
        if old is not None:
            self.resident_bytes -= old
        self.resident_bytes += size
        self.pinned_bytes += size
        self.pinned.add(key)
        self.order.append(key)

    # moe.rs:207-213
    def clear(self):
        self.sizes.clear()
        self.order.clear()
        self.pinned.clear()
        self.resident_bytes = 0
        self.pinned_bytes = 0

    # moe.rs:216-226
    def reset_counters(self):
        self.hit_count = 0
        self.miss_count = 0
        self.eviction_count = 0
        self.cache_insert_attempt_count = 0
        self.cache_insert_accept_count = 0
        self.cache_insert_bypass_count = 0
        self.oversized_tensor_bypass_count = 0
        self.oversized_expert_bypass_count = 0
        self.self_eviction_risk_count = 0

    def get_or_insert(self, key, size: int):
        """README-level API: get(key) else insert(key, load()) (same counters
        as the executor's inline path, moe.rs:508-518)."""
        if self.get(key):
            return True, True
        return False, self.insert(key, size)

    def counters(self) -> dict:
        return {k: getattr(self, k) for k in (
            "capacity_bytes", "resident_bytes", "pinned_bytes", "hit_count", "miss_count",
            "eviction_count", "cache_insert_attempt_count", "cache_insert_accept_count",
            "cache_insert_bypass_count", "oversized_tensor_bypass_count",
            "oversized_expert_bypass_count", "self_eviction_risk_count")}


def executor_lookup(cache: CacheModel | None, layer_id: int, selected, tensors):
    """Byte accounting of one executor call (moe.rs:458-583 / 993-1087).

    ``tensors(e)`` returns the ordered list of (kind, fmt, nbytes, is_scale)
    for expert e (3 tensors for Q4, 6 for native FP4).  Returns a dict with
    loaded / reused byte totals split into weights and scales.
    """
    acc = {"weight_loaded": 0, "weight_reused": 0, "scale_loaded": 0, "scale_reused": 0,
           "logical": 0}
    for e, _w in selected:
        ts = tensors(e)
        expert_bytes = sum(t[2] for t in ts)
        acc["logical"] += expert_bytes
        bypass = False
        if cache is not None and expert_bytes > cache.capacity_bytes:
            if cache.bypass_oversized_experts:
                bypass = True
                cache.oversized_expert_bypass_count += 1
            else:
                cache.self_eviction_risk_count += 1
        for kind, fmt, nbytes, is_scale in ts:
            pre = "scale" if is_scale else "weight"
            if bypass:
                cache.cache_insert_attempt_count += 1
                cache.cache_insert_bypass_count += 1
                acc[pre + "_loaded"] += nbytes
            elif cache is not None:
                key = (layer_id, e, kind, fmt)
                if cache.get(key):
                    acc[pre + "_reused"] += nbytes
                else:
                    acc[pre + "_loaded"] += nbytes
                    cache.insert(key, nbytes)
            else:
                acc[pre + "_loaded"] += nbytes
    return acc
