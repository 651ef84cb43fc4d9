"""KVCacheManager host logic (no GPU): storage, accounting, dense-shadow release, the per-layer
policy eviction and the early exits of enforce_global_budget (kv_cache_manager.py)."""

import torch

from shadow_infer_b200.shadowkv import (
    ImportanceAgeEvictionPolicy,
    KVCacheEntry,
    KVCacheManager,
    LeastImportantEvictionPolicy,
    TokenHeadScore,
)


class StubPacked:
    """Stands in for a packed cache: fixed resident bytes, records evictions."""

    def __init__(self, resident=1000, seq_len=4, num_heads=2):
        self.resident = resident
        self.seq_len, self.num_heads = seq_len, num_heads
        self.evicted = []
        self.packed_data = {"fp16": {}}

    def resident_bytes(self):
        return self.resident

    def memory_bytes(self):
        return self.resident

    def evict(self, entries):
        self.evicted.append(set(entries))
        self.resident -= 10 * len(entries)
        return len(entries)


def test_store_retrieve_and_stats():
    m = KVCacheManager(num_layers=2)
    p = StubPacked()
    e0 = KVCacheEntry(k_tensor=None, v_tensor=None, precision="fp16", packed_kv=p, is_reused=True)
    e1 = KVCacheEntry(k_tensor=torch.zeros(4), v_tensor=torch.zeros(4), precision="fp32")
    m.store(0, e0)
    m.store(1, e1)
    assert m.retrieve(0) is e0 and m.retrieve_packed(0) is p and m.retrieve(5) is None
    assert m.get_memory_usage() == 1000 + 32
    stats = m.get_reuse_stats()
    assert stats["global_reuse_rate"] == 0.5 and stats["layer_0_reuse_rate"] == 1.0
    m.store_packed(3, {"packed_kv": p})
    assert m.retrieve_packed(3) is p
    m.store_prefetched(0, "next", e0)
    assert m.retrieve_prefetched(0, "next") is e0
    m.clear_prefetch_buffer("next")
    assert m.retrieve_prefetched(0, "next") is None
    assert "cached_layers=2" in repr(m)
    m.clear()
    assert m.get_memory_usage() == 0 and m.retrieve_packed(0) is None


def test_dense_shadow_release_and_accounting():
    m = KVCacheManager(num_layers=1)
    p = StubPacked(resident=500)
    e = KVCacheEntry(k_tensor=torch.zeros(8), v_tensor=torch.zeros(8), precision="mixed", packed_kv=p)
    m.store(0, e)
    assert m.get_memory_usage() == 500 + 64
    assert m._release_dense_shadows() is True
    assert e.k_tensor is None and m.get_memory_usage() == 500
    assert m._release_dense_shadows() is False


def test_per_layer_policy_eviction():
    p = StubPacked(resident=1000, seq_len=4, num_heads=2)
    m = KVCacheManager(num_layers=1, memory_budget_bytes=None)
    m.store(0, KVCacheEntry(k_tensor=None, v_tensor=None, precision="fp16", packed_kv=p))
    meta = {(t, h): TokenHeadScore(0, t, h, importance=float(t * 2 + h)) for t in range(4) for h in range(2)}
    m.set_token_head_meta(0, meta)
    m.memory_budget_bytes = 700
    m._enforce_budget(0)
    # estimated entry bytes = 1000 // 8 = 125; (1000 - 700) // 125 = 2 lowest-importance entries
    assert p.evicted == [{(0, 0), (0, 1)}]
    assert meta[(0, 0)].importance == -1.0 and meta[(0, 1)].importance == -1.0
    assert m.get_token_head_meta(0)[(1, 0)].importance == 2.0


def test_policies_select_lowest():
    entries = [TokenHeadScore(0, t, 0, importance=1.0 - 0.1 * t, age=t) for t in range(5)]
    sel = LeastImportantEvictionPolicy().select_for_eviction(entries, 100, 130, 10)
    assert sel == {(0, 4, 0), (0, 3, 0), (0, 2, 0)}
    assert LeastImportantEvictionPolicy().select_for_eviction(entries, 200, 130, 10) == set()
    aged = ImportanceAgeEvictionPolicy(age_decay=0.5).select_for_eviction(entries, 100, 110, 10)
    assert aged == {(0, 4, 0)}


def test_importance_matrix_and_global_budget_early_exits():
    m = KVCacheManager(num_layers=1)
    assert m.get_importance_matrix(0) is None
    imp = torch.rand(4, 2)
    m.set_importance_matrix(0, imp)
    got = m.get_importance_matrix(0)
    assert got.device.type == "cpu" and torch.equal(got, imp)
    assert m.enforce_global_budget(None) == 0 and m.enforce_global_budget(-5) == 0
    assert m.enforce_global_budget(100) == 0                  # no packed caches
    p = StubPacked(resident=100)
    m.store(0, KVCacheEntry(k_tensor=None, v_tensor=None, precision="fp16", packed_kv=p))
    assert m.enforce_global_budget(1000) == 0                 # under 0.9 * budget: nothing to do
