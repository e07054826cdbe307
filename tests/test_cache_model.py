"""CPU checks of the expert-cache restatement against the counter sequences
the reference's own tests assert (crates/objeta-cuda/src/moe.rs:1891-2559).
The product cache is compared with this model on the GPU (test_moe_gpu)."""
from oracle.cache_model import CacheModel, executor_lookup

Q4 = 0
FP4 = 3


def q4_tensors(gate_len, up_len, down_len):
    return lambda e: [(0, Q4, gate_len, False), (1, Q4, up_len, False), (2, Q4, down_len, False)]


def fp4_tensors(h, i, o):
    return lambda e: [(3, FP4, i * h // 2, False), (4, FP4, i * h // 32, True), (5, FP4, i * h // 2, False),
                      (6, FP4, i * h // 32, True), (7, FP4, o * i // 2, False), (8, FP4, o * i // 32, True)]


# Q4 expert 256/512/256: gate/up 512 rows x 8 blocks x 18 B, down 256 x 16 x 18
GATE = 512 * 8 * 18
DOWN = 256 * 16 * 18
EXPERT = 2 * GATE + DOWN
T = q4_tensors(GATE, GATE, DOWN)


def test_repeat_hits():
    # moe.rs:1950-2000: 6 misses, then 6 hits, no evictions
    c = CacheModel(1000 * 1024)
    a = executor_lookup(c, 0, [(0, .5), (1, .5)], T)
    assert a["weight_reused"] == 0 and c.miss_count == 6 and c.hit_count == 0
    a = executor_lookup(c, 0, [(0, .5), (1, .5)], T)
    assert a["weight_loaded"] == 0 and a["weight_reused"] == a["logical"]
    assert c.hit_count == 6 and c.miss_count == 6 and c.eviction_count == 0


def test_capacity_fits_all():
    # moe.rs:2002-2025
    c = CacheModel(4 * EXPERT)
    executor_lookup(c, 0, [(0, .5), (1, .5), (2, .5), (3, .5)], T)
    assert c.eviction_count == 0 and c.resident_bytes == 4 * EXPERT


def test_single_expert_capacity_evicts():
    # moe.rs:2027-2082
    c = CacheModel(EXPERT)
    executor_lookup(c, 0, [(0, 1.0)], T)
    assert c.eviction_count == 0 and c.resident_bytes == EXPERT
    executor_lookup(c, 0, [(1, 1.0)], T)
    assert c.eviction_count > 0 and c.resident_bytes == EXPERT
    a = executor_lookup(c, 0, [(0, 1.0)], T)
    assert a["weight_loaded"] == EXPERT and a["weight_reused"] == 0


def test_lru_touch_order():
    # moe.rs:2084-2166
    c = CacheModel(2 * EXPERT)
    for e in (0, 1, 0, 2):
        executor_lookup(c, 0, [(e, 1.0)], T)
    assert executor_lookup(c, 0, [(0, 1.0)], T)["weight_reused"] == EXPERT
    a = executor_lookup(c, 0, [(1, 1.0)], T)
    assert a["weight_reused"] == 0 and a["weight_loaded"] == EXPERT


def test_oversized_tensor_bypass():
    # moe.rs:2170-2226
    c = CacheModel(GATE - 1)
    executor_lookup(c, 0, [(0, 1.0)], T)
    assert (c.cache_insert_attempt_count, c.cache_insert_accept_count, c.cache_insert_bypass_count,
            c.oversized_tensor_bypass_count, c.oversized_expert_bypass_count, c.resident_bytes) == (3, 0, 3, 3, 0, 0)


def test_oversized_expert_bypass():
    # moe.rs:2228-2316
    c = CacheModel(EXPERT - 100, bypass_oversized_experts=True)
    executor_lookup(c, 0, [(0, 1.0)], T)
    assert (c.cache_insert_attempt_count, c.cache_insert_accept_count, c.cache_insert_bypass_count,
            c.oversized_tensor_bypass_count, c.oversized_expert_bypass_count,
            c.self_eviction_risk_count, c.resident_bytes) == (3, 0, 3, 0, 1, 0, 0)
    c = CacheModel(EXPERT - 100)
    a = executor_lookup(c, 0, [(0, 1.0)], T)
    assert c.self_eviction_risk_count == 1 and c.oversized_expert_bypass_count == 0
    assert c.cache_insert_accept_count > 0
    assert a["logical"] == a["weight_loaded"] + a["weight_reused"]


def test_native_fp4_cache_sequence():
    # moe.rs:2421-2559: expert_bytes == 208896, capacity two experts
    tf = fp4_tensors(256, 512, 256)
    eb = sum(t[2] for t in tf(0))
    assert eb == 208896
    c = CacheModel(2 * eb)
    seq = [(0, eb, 0), (0, 0, eb), (1, eb, 0), (2, eb, 0), (0, eb, 0)]
    for e, want_loaded, want_reused in seq:
        a = executor_lookup(c, 0, [(e, 1.0)], tf)
        assert a["weight_loaded"] + a["scale_loaded"] == want_loaded
        assert a["weight_reused"] + a["scale_reused"] == want_reused
    assert c.resident_bytes == 2 * eb


def test_pinned_survive_and_stop_eviction():
    # moe.rs:179-205: pinned keys are never evicted; insert_pinned stops when
    # only pinned keys remain
    c = CacheModel(100)
    c.insert_pinned(("s", 0), 60)
    c.insert(("r", 1), 30)
    c.insert(("r", 2), 30)  # evicts ("r", 1), not the pinned key
    assert ("s", 0) in c.sizes and ("r", 1) not in c.sizes and c.eviction_count == 1
    c.insert_pinned(("s", 1), 60)  # evicts ("r", 2), then stops: over capacity
    assert c.resident_bytes == 120 and c.pinned_bytes == 120
    assert c.evict_lru() is None


def test_reset_counters_keeps_residency():
    c = CacheModel(1000)
    c.insert(("a",), 10)
    c.get(("a",))
    c.reset_counters()
    assert c.hit_count == 0 and c.cache_insert_attempt_count == 0 and c.resident_bytes == 10
    c.clear()
    assert c.resident_bytes == 0 and not c.order
