"""KVCacheManager.enforce_global_budget on the GPU vs the reference fixtures and the oracle.

The processed count, the usage before and after, every layer's resident bytes and the set of
surviving entries must equal the reference's exactly (integer/byte work).
"""

import numpy as np
import pytest
import torch

from golden_lib import case_arrays, load_pins
from oracle import shadowkv_oracle as O

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def skv():
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    import shadow_infer_b200.shadowkv as m
    return m


def _present(cache, S, H):
    out = np.zeros((S, H), dtype=np.uint8)
    for d in cache.packed_data.values():
        for t, h in d["indices"]:
            out[t, h] = 1
    return out


def _manager(skv, arrays, layers, group, *, dense=(), packed_only=(), no_importance=()):
    mgr = skv.KVCacheManager(num_layers=layers)
    caches = []
    for L in range(layers):
        k = torch.from_numpy(arrays[f"L{L}.k"])
        v = torch.from_numpy(arrays[f"L{L}.v"])
        plan = skv.PrecisionPlan.from_codes(torch.from_numpy(arrays[f"L{L}.codes"]).cuda())
        cache = skv.PackedKVCache.pack(k.cuda(), v.cuda(), None, group, plan=plan)["packed_kv"]
        if L in packed_only:
            mgr.store_packed(L, cache)
        else:
            mgr.store(L, skv.KVCacheEntry(k_tensor=k if L in dense else None, v_tensor=v if L in dense else None,
                                          precision="mixed", packed_kv=cache))
        if L not in no_importance:
            mgr.set_importance_matrix(L, torch.from_numpy(arrays[f"L{L}.imp"]).cuda())
        caches.append(cache)
    return mgr, caches


@pytest.mark.parametrize("case", sorted(c for c, v in load_pins()["cases"].items() if v["kind"] == "global_budget"))
def test_global_budget_matches_reference_fixture(case, skv, golden_small):
    pin = load_pins()["cases"][case]
    a = case_arrays(golden_small, case)
    mgr, caches = _manager(skv, a, pin["layers"], pin["group"], dense=pin["dense"], packed_only=pin["packed_only"],
                           no_importance=pin["no_importance"])
    assert mgr.get_memory_usage() == pin["usage_before"]
    assert mgr.enforce_global_budget(pin["budget"], pin["sink"]) == pin["evicted"]
    assert mgr.get_memory_usage() == pin["usage_after"]
    for L, cache in enumerate(caches):
        assert cache.resident_bytes() == pin["resident_after"][L]
        np.testing.assert_array_equal(_present(cache, pin["S"], pin["H"]), a[f"L{L}.remaining"])


@pytest.mark.parametrize("layers,S,H,D,B,frac,sink,ties", [
    (4, 384, 8, 128, 1, 0.5, 4, False),
    (3, 200, 6, 64, 2, 0.3, 0, True),       # many equal importances: stable list order decides
    (6, 257, 4, 128, 1, 0.05, 8, False),    # deep cut, near the floor
])
def test_global_budget_matches_oracle(skv, layers, S, H, D, B, frac, sink, ties):
    rng = np.random.default_rng(S * 7 + layers)
    arrays, olayers = {}, []
    for L in range(layers):
        k = rng.standard_normal((B, H, S, D)).astype(np.float32)
        v = rng.standard_normal((B, H, S, D)).astype(np.float32)
        codes = rng.choice(5, size=(S, H), p=(0.05, 0.3, 0.3, 0.3, 0.05)).astype(np.int8)
        imp = rng.random((S, H)).astype(np.float32)
        if ties:
            imp = np.round(imp * 8) / 8
        arrays.update({f"L{L}.k": k, f"L{L}.v": v, f"L{L}.codes": codes, f"L{L}.imp": imp})
        olayers.append({"cache": O.pack(k, v, O.plan_from_codes(codes), 16), "importance": imp, "counted": True})
    mgr, caches = _manager(skv, arrays, layers, 16)
    before = mgr.get_memory_usage()
    assert before == O.manager_usage(olayers)
    budget = int(before * frac)
    assert mgr.enforce_global_budget(budget, sink) == O.enforce_global_budget(olayers, budget, sink)
    assert mgr.get_memory_usage() == O.manager_usage(olayers)
    for L, cache in enumerate(caches):
        np.testing.assert_array_equal(_present(cache, S, H), _present(olayers[L]["cache"], S, H))
    # packed data of the survivors is untouched by the compaction
    k_u, _ = caches[0].unpack()
    k_o, _ = O.unpack(olayers[0]["cache"])
    np.testing.assert_array_equal(k_u.cpu().numpy(), k_o)


def test_global_budget_no_candidates_and_no_budget(skv):
    rng = np.random.default_rng(3)
    k = torch.from_numpy(rng.standard_normal((1, 2, 8, 64)).astype(np.float32)).cuda()
    plan = skv.PrecisionPlan.from_codes(torch.ones(8, 2, dtype=torch.int8).cuda())
    cache = skv.PackedKVCache.pack(k, k, None, 16, plan=plan)["packed_kv"]
    mgr = skv.KVCacheManager(num_layers=1)
    mgr.store(0, skv.KVCacheEntry(k_tensor=None, v_tensor=None, precision="fp16", packed_kv=cache))
    assert mgr.enforce_global_budget(None) == 0
    assert mgr.enforce_global_budget(0) == 0
    assert mgr.enforce_global_budget(1) == 0                  # no importance matrix: no candidates
    mgr.set_importance_matrix(0, torch.rand(8, 2))
    assert mgr.enforce_global_budget(1, sink_tokens=8) == 0   # every token is a sink
    before = cache.resident_bytes()
    assert mgr.enforce_global_budget(1, sink_tokens=2) == 12  # floor: every non-sink processed
    assert cache.resident_bytes() < before


@pytest.mark.parametrize("policy_name,ties", [("least", False), ("least", True), ("age", False)])
def test_per_layer_budget_device_selection(policy_name, ties):
    """KVCacheManager._enforce_budget with the built-in policies selects on the GPU (or by a float64
    argsort when float32 cannot hold the keys) exactly the entries the policy's stable sort picks."""
    import copy
    import numpy as np
    from shadow_infer_b200.shadowkv import (ImportanceAgeEvictionPolicy, KVCacheEntry, KVCacheManager,
                                            LeastImportantEvictionPolicy, PackedKVCache, PrecisionPlan,
                                            TokenHeadScore)
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    rng = np.random.default_rng(31 + ties)
    B, H, S, D = 1, 4, 300, 64
    k = torch.from_numpy(rng.standard_normal((B, H, S, D)).astype(np.float32)).cuda()
    codes = torch.from_numpy(rng.integers(1, 4, size=(S, H)).astype(np.int8)).cuda()
    imp = rng.random((S, H)).astype(np.float32)
    if ties:
        imp = np.round(imp * 8) / 8                      # many equal keys: list order decides
    policy = (LeastImportantEvictionPolicy() if policy_name == "least" else ImportanceAgeEvictionPolicy(0.03))

    def build():
        cache = PackedKVCache.pack(k, k, None, 16, plan=PrecisionPlan.from_codes(codes))["packed_kv"]
        meta = {(t, h): TokenHeadScore(0, t, h, importance=float(imp[t, h]), age=int((t * 7 + h) % 11))
                for t in range(S) for h in range(H)}
        m = KVCacheManager(num_layers=1, eviction_policy=policy)
        m.store(0, KVCacheEntry(k_tensor=None, v_tensor=None, precision="mixed", packed_kv=cache))
        m.set_token_head_meta(0, meta)
        return m, cache, meta

    m, cache, meta = build()
    usage = m.get_memory_usage()
    est = max(1, int(cache.memory_bytes()) // (S * H))
    want = policy.select_for_eviction(list(copy.deepcopy(meta).values()), int(usage * 0.6), usage, est)
    m.memory_budget_bytes = int(usage * 0.6)
    m._enforce_budget(0)
    got = {(0, t, h) for (t, h), e in meta.items() if e.importance == -1.0}
    assert got == want and len(want) > 0
    ref = PackedKVCache.pack(k, k, None, 16, plan=PrecisionPlan.from_codes(codes))["packed_kv"]
    ref.evict({(t, h) for _, t, h in want})
    assert cache.memory_bytes() == ref.memory_bytes()
    ku, _ = cache.unpack()
    kr, _ = ref.unpack()
    assert torch.equal(ku, kr)
