"""Pin the CPU oracle to the reference: every golden fixture must be reproduced.

The fixtures were produced by the reference implementation itself
(``tests/golden/make_golden.py``); these tests run on the CPU only.
"""

import numpy as np
import pytest

from golden_lib import array_digest, case_arrays, packed_summary
from oracle import shadowkv_oracle as O

PRECISIONS = ("fp32", "fp16", "int8", "int4")


def _cases(pins, kind):
    return sorted(c for c, v in pins["cases"].items() if v["kind"] == kind)


def _pins():
    from golden_lib import load_pins
    return load_pins()


@pytest.mark.parametrize("case", _cases(_pins(), "pack"))
def test_pack_plan_unpack_dense(case, golden_small, golden_pins):
    a = case_arrays(golden_small, case)
    p = golden_pins["cases"][case]
    plan = O.plan_from_codes(a["codes"], a["reuse"])
    for prec in PRECISIONS:
        assert np.array_equal(plan["flat_indices"][prec], a[f"plan.flat.{prec}"]), prec
    assert np.array_equal(np.array(plan["evicted_entries"], dtype=np.int64).reshape(-1, 2), a["plan.evicted"])
    assert np.array_equal(plan["reuse_flat"], a["plan.reuse_flat"])
    assert plan["fingerprint"] == p["fingerprint"]
    cache = O.pack(a["k"], a["v"], plan, p["group"])
    assert packed_summary(cache.packed_data, cache.memory_bytes()) == p["summary"]
    assert cache.memory_bytes() == p["memory_bytes"]
    assert cache.data_plane_bytes() == p["data_plane_bytes"]
    assert cache.resident_bytes() == p["resident_bytes"]
    ku, vu = O.unpack(cache)
    assert np.array_equal(ku, a["unpack.k"]) and np.array_equal(vu, a["unpack.v"])
    kd, vd = O.compress_dense(a["k"], a["v"], plan, p["group"])
    assert np.array_equal(kd, a["dense.k"]) and np.array_equal(vd, a["dense.v"])
    kd, vd = O.compress_dense(a["k"], a["v"], plan, p["group"], a["k_prev"], a["v_prev"])
    assert np.array_equal(kd, a["dense_reuse.k"]) and np.array_equal(vd, a["dense_reuse.v"])


@pytest.mark.parametrize("case", _cases(_pins(), "reuse"))
def test_reuse(case, golden_small, golden_pins):
    a = case_arrays(golden_small, case)
    p = golden_pins["cases"][case]
    cur = O.pack(a["k"], a["v"], O.plan_from_codes(a["codes"]), p["group"])
    prev = O.pack(a["k_prev"], a["v_prev"], O.plan_from_codes(a["prev_codes"]), p["group"])
    stats = O.apply_reuse_mask(cur, prev, a["mask"])
    assert stats == p["stats"]
    assert packed_summary(cur.packed_data, cur.memory_bytes()) == p["summary"]
    ku, vu = O.unpack(cur)
    assert np.array_equal(ku, a["unpack.k"]) and np.array_equal(vu, a["unpack.v"])


@pytest.mark.parametrize("case", _cases(_pins(), "evict"))
def test_evict(case, golden_small, golden_pins):
    a = case_arrays(golden_small, case)
    p = golden_pins["cases"][case]
    cache = O.pack(a["k"], a["v"], O.plan_from_codes(a["codes"]), p["group"])
    assert O.evict(cache, a["mask"]) == p["removed"]
    assert O.evict(cache, a["mask"]) == p["removed_again"] == 0
    ku, vu = O.unpack(cache)
    assert np.array_equal(ku, a["unpack.k"]) and np.array_equal(vu, a["unpack.v"])
    assert O.evict(cache, a["whole_mask"]) == p["removed_whole"]
    assert "int8" not in cache.packed_data
    assert packed_summary(cache.packed_data, cache.memory_bytes()) == p["summary_after_whole"]
    assert cache.resident_bytes() == p["resident_after_whole"]


@pytest.mark.parametrize("case", _cases(_pins(), "admit"))
def test_admit(case, golden_small, golden_pins):
    a = case_arrays(golden_small, case)
    p = golden_pins["cases"][case]
    out, pred, ev = O.admit_codes(
        a["codes"], a["importance"], a["sensitivity"], p["budget"], p["B"], p["D"],
        sink_tokens=p["sink"], rd_allocation=p["rd"], allow_eviction=p["evict"],
        protected_mask=a.get("protected"), group_size=p["group"])
    assert np.array_equal(out, a["out"])
    assert (pred, ev) == (p["predicted"], p["evicted"])
    assert O.predict_codes_bytes(a["codes"], p["B"], p["D"], p["group"]) == p["predicted0"]


def test_allocate(golden_small):
    a = case_arrays(golden_small, "allocate")
    for mode in ("aggressive", "balanced", "conservative", "unknown"):
        assert np.array_equal(O.allocate_precision_codes(a["importance"], mode), a[f"codes.{mode}"]), mode


def test_sensitivity(golden_small):
    a = case_arrays(golden_small, "sensitivity")
    assert np.array_equal(O.kv_sensitivity(a["k"], a["v"]), a["sens"])


@pytest.mark.parametrize("case", _cases(_pins(), "attention"))
def test_attention(case, golden_small):
    a = case_arrays(golden_small, case)
    cache = O.pack(a["k"], a["v"], O.plan_from_codes(a["codes"]), 16)
    out = O.packed_attention(a["q"].astype(np.float32), cache)
    ref = a["out"].astype(np.float64)
    rel = np.linalg.norm(out - ref) / np.linalg.norm(ref)
    assert rel < 1e-5, rel


def test_entry_bytes_table():
    # rd_allocator.py:26-44 values at B=1 and B=8, D=128 (fp32/fp16/int8/int4)
    assert list(O.code_costs(1, 128, 16)) == [1024, 512, 264, 192, 0]
    assert list(O.code_costs(8, 128, 16)) == [8192, 4096, 2112, 1536, 0]


def test_full_cfg1_pins(golden_pins):
    from shadow_infer_b200 import workloads as W
    pin = golden_pins["full"]["cfg1"]
    c = W.CONFIGS["cfg1"]
    k, v = W.kv_tensors(c["B"], c["H"], c["S"], c["D"], c["seed"])
    imp = W.importance_map(c["S"], c["H"], c["seed"], c["fractions"])
    assert array_digest(k) == pin["k"] and array_digest(imp) == pin["importance"]
    codes = O.allocate_precision_codes(imp.numpy(), "balanced")
    assert array_digest(codes) == pin["codes"]
    plan = O.plan_from_codes(codes)
    assert plan["fingerprint"] == pin["fingerprint"]
    cache = O.pack(k.numpy(), v.numpy(), plan, 16)
    assert packed_summary(cache.packed_data, cache.memory_bytes()) == pin["packed"]
    ku, vu = O.unpack(cache)
    assert array_digest(ku) == pin["unpack_k"] and array_digest(vu) == pin["unpack_v"]
    kd, vd = O.compress_dense(k.numpy(), v.numpy(), plan, 16)
    assert array_digest(kd) == pin["dense_k"] and array_digest(vd) == pin["dense_v"]


def test_full_cfg2_pins(golden_pins):
    import torch
    from shadow_infer_b200 import workloads as W
    pin = golden_pins["full"]["cfg2"]
    I = W.cfg2_inputs()
    k, v = I["k"].numpy(), I["v"].numpy()
    assert array_digest(I["k"]) == pin["k"] and array_digest(I["reuse"]) == pin["reuse"]
    sens = O.kv_sensitivity(k, v)
    assert array_digest(sens) == pin["sensitivity"]
    codes0 = O.allocate_precision_codes(I["importance"].numpy(), "balanced")
    assert array_digest(codes0) == pin["codes0"]
    adm, pred, ev = O.admit_codes(codes0, I["importance"].numpy(), sens, I["budget"], 1, 128,
                                  sink_tokens=I["sink_tokens"], rd_allocation=True, allow_eviction=True)
    assert array_digest(adm) == pin["admitted"] and (pred, ev) == (pin["predicted"], pin["evicted"])
    reuse = I["reuse"].numpy()
    plan = O.plan_from_codes(adm, reuse)
    assert plan["fingerprint"] == pin["fingerprint"]
    cache = O.pack(k, v, plan, 16)
    assert packed_summary(cache.packed_data, cache.memory_bytes()) == pin["packed"]
    prev = O.pack(I["k_prev"].numpy(), I["v_prev"].numpy(), O.plan_from_codes(adm), 16)
    assert O.apply_reuse_mask(cache, prev, reuse) == pin["reuse_stats"]
    assert packed_summary(cache.packed_data, cache.memory_bytes()) == pin["after_reuse"]
    ku, vu = O.unpack(cache)
    assert array_digest(ku) == pin["unpack_k"] and array_digest(vu) == pin["unpack_v"]
    g = torch.Generator().manual_seed(pin["evict_seed"])
    emask = (torch.rand(adm.shape, generator=g) < pin["evict_frac"]).numpy()
    assert O.evict(cache, emask) == pin["removed"]
    assert packed_summary(cache.packed_data, cache.memory_bytes()) == pin["after_evict"]
    assert cache.resident_bytes() == pin["resident_after_evict"]


def _gb_layers(pin, arrays):
    """Oracle layer list of a global-budget fixture (the manager's layer order)."""
    layers = []
    for L in range(pin["layers"]):
        k, v = arrays[f"L{L}.k"], arrays[f"L{L}.v"]
        cache = O.pack(k, v, O.plan_from_codes(arrays[f"L{L}.codes"]), pin["group"])
        layers.append({
            "cache": cache, "importance": arrays[f"L{L}.imp"],
            "counted": L not in pin["packed_only"], "candidate": L not in pin["no_importance"],
            "dense_bytes": (k.nbytes + v.nbytes) if L in pin["dense"] else 0,
        })
    return layers


@pytest.mark.parametrize("case", _cases(_pins(), "global_budget"))
def test_global_budget(case, golden_small):
    """KVCacheManager.enforce_global_budget: processed count, usage and surviving entries."""
    pin = _pins()["cases"][case]
    a = case_arrays(golden_small, case)
    layers = _gb_layers(pin, a)
    assert O.manager_usage(layers) == pin["usage_before"]
    assert O.enforce_global_budget(layers, pin["budget"], pin["sink"]) == pin["evicted"]
    assert O.manager_usage(layers) == pin["usage_after"]
    for L, layer in enumerate(layers):
        present = np.zeros_like(a[f"L{L}.remaining"])
        for d in layer["cache"].packed_data.values():
            for t, h in d["indices"]:
                present[t, h] = 1
        np.testing.assert_array_equal(present, a[f"L{L}.remaining"])
        assert layer["cache"].resident_bytes() == pin["resident_after"][L]


@pytest.mark.parametrize("case", _cases(_pins(), "paged"))
def test_paged_store(case):
    """PagedKVStore scripts: return values / ValueErrors, page layout, slot pool, counters,
    ledgers, page-tensor digests and gather digests after every operation."""
    from golden_lib import array_digest as dig, paged_apply, state_digest
    from oracle.paged_store_oracle import OraclePagedStore, store_state
    pin = _pins()["cases"][case]
    B, H, D = pin["B"], pin["H"], pin["D"]
    store = OraclePagedStore(B, H, D, page_size=pin["P"], int4_group_size=pin["G"])
    for i, (op, want) in enumerate(zip(pin["ops"], pin["results"])):
        try:
            ret, err = paged_apply(store, op, B, H, D, lambda x: x), False
        except ValueError:
            ret, err = None, True
        assert (ret, err) == (want["ret"], want["error"]), (i, op)
        st = store_state(store)
        st["pages_digest"] = state_digest(st.pop("page_digests"))
        assert st == want["state"], (i, op)
        k, v = store.gather()
        assert [dig(k), dig(v)] == want["gather"] and k.shape[2] == want["S_out"], (i, op)


@pytest.mark.parametrize("case", _cases(_pins(), "reuse_decision"))
def test_reuse_decision(case, golden_small):
    """decide_reuse_per_token: drift within 1e-6 relative of the reference's float32 drift; the
    mask equal wherever the reference's drift is not within that band of its threshold."""
    from golden_lib import reuse_inputs
    from oracle import decision_oracle as DO
    pin = _pins()["cases"][case]
    a = case_arrays(golden_small, case)
    k, v, kp, vp, imp = reuse_inputs(pin["seed"], pin["B"], pin["H"], pin["S"], pin["D"])
    mask, stats, delta = DO.decide_reuse_per_token(k, v, kp, vp, pin["step_id"], pin["total_steps"], pin["drift"],
                                                   pin["mode"], imp)
    np.testing.assert_allclose(delta.T.astype(np.float64), a["ref_delta"], rtol=1e-6, atol=0)
    near = np.abs(a["ref_delta"] - a["ref_thr"]) <= 1e-6 * a["ref_thr"]
    assert np.array_equal(mask[~near], a["mask"].astype(bool)[~near])
    if not near.any():
        assert stats == pin["stats"]


@pytest.mark.parametrize("case", _cases(_pins(), "irap"))
def test_irap_importance(case, golden_small):
    """compute_irap_importance (direct or through the agent's contract): importance within the
    reference's own 1e-6, EMA within 1e-6 relative, delta_a within 1e-5 relative."""
    from golden_lib import irap_scores
    from oracle import decision_oracle as DO
    pin = _pins()["cases"][case]
    a = case_arrays(golden_small, case)
    x = irap_scores(pin["seed"], pin["B"], pin["H"], pin["Sq"], pin["Sk"], kind=pin["score_kind"], bad=pin["bad"])
    if pin["contract"] is not None:
        x = DO.irap_inputs(x, pin["contract"] == "probs")
    imp, ema, da = DO.compute_irap_importance(x, a.get("prev"), pin["decay"], pin["beta"], pin["sink"],
                                              pin["layer_index"], pin["num_layers"])
    assert np.abs(imp - a["importance"]).max() <= 1e-6
    np.testing.assert_allclose(ema, a["ema"], rtol=1e-6, atol=1e-12)
    if pin["delta_a"] is None:
        assert da is None
    else:
        assert abs(da - pin["delta_a"]) <= 1e-5 * abs(pin["delta_a"])


@pytest.mark.parametrize("case", _cases(_pins(), "attention_gqa"))
def test_attention_gqa(case, golden_small):
    """Grouped-query attention over a packed past plus this step's K/V (DiffusionLlamaAttention)."""
    a = case_arrays(golden_small, case)
    cache = O.pack(a["k"], a["v"], O.plan_from_codes(a["codes"]), 16)
    out = O.packed_attention(a["q"].astype(np.float32), cache, k_new=a["k_new"], v_new=a["v_new"])
    ref = a["out"].astype(np.float64)
    rel = np.linalg.norm(out - ref) / np.linalg.norm(ref)
    assert rel < 1e-5, rel


def _sampled_oracle_attention(q_rows, cache):
    """Oracle attention of the query rows ``q_rows`` [B, H, n, D] over the whole packed cache."""
    return O.packed_attention(q_rows.astype(np.float32), cache)


def test_long_context_slice_pins(golden_pins, golden_small):
    """Heads 0-1 of the long-context layer (S=32768, codes 10/30/60, 4 outlier channels x10):
    the oracle reproduces the reference's plan, packed bytes, unpack and sampled attention."""
    from shadow_infer_b200 import workloads as W
    pin = golden_pins["full"]["cfg5_slice"]
    h0, h1 = pin["heads"]
    L = W.cfg5_layer(h0, h1)
    assert array_digest(L["k"]) == pin["k"] and array_digest(L["v"]) == pin["v"]
    assert array_digest(L["q"]) == pin["q"] and array_digest(L["importance"]) == pin["importance"]
    imp = np.ascontiguousarray(L["importance"][:, h0:h1].numpy())
    codes = O.allocate_precision_codes(imp, "balanced")
    assert array_digest(codes) == pin["codes"]
    plan = O.plan_from_codes(codes)
    assert plan["fingerprint"] == pin["fingerprint"]
    cache = O.pack(L["k"].numpy(), L["v"].numpy(), plan, 16)
    assert packed_summary(cache.packed_data, cache.memory_bytes()) == pin["packed"]
    assert cache.data_plane_bytes() == pin["data_plane_bytes"] and cache.resident_bytes() == pin["resident_bytes"]
    ku, vu = O.unpack(cache)
    assert array_digest(ku) == pin["unpack_k"] and array_digest(vu) == pin["unpack_v"]
    a = case_arrays(golden_small, "cfg5_slice")
    out = _sampled_oracle_attention(L["q"].numpy()[:, :, a["rows"]], cache)
    assert np.linalg.norm(out - a["out"]) / np.linalg.norm(out) < 1e-5


def test_batched_denoise_slice_pins(golden_pins, golden_small):
    """Heads 0-3 of a batched denoising layer (B=8, S=2048): one drift step, the reuse decision
    (drift < 0.05), re-pack, reuse from the previous cache, eviction of the 25 % lowest-importance
    entries and the unpack, against the reference's digests."""
    import torch
    from oracle import decision_oracle as DO
    from shadow_infer_b200 import workloads as W
    pin = golden_pins["full"]["cfg4_slice"]
    a = case_arrays(golden_small, "cfg4_slice")
    h0, h1 = pin["heads"]
    c = W.CONFIGS["cfg4"]
    L = W.cfg4_layer(h0, h1)
    nk, nv = W.drift_noise(c["B"], c["S"], c["D"], 10_000, 1, h0, h1)
    k1, v1 = W.apply_drift(L["k"], nk), W.apply_drift(L["v"], nv)
    assert array_digest(k1) == pin["k1"] and array_digest(v1) == pin["v1"] and array_digest(L["q"]) == pin["q"]
    imp = np.ascontiguousarray(L["importance"][:, h0:h1].numpy())
    codes = O.allocate_precision_codes(imp, "balanced")
    assert array_digest(codes) == pin["codes"]
    mask, stats, drift = DO.decide_reuse_per_token(k1.numpy(), v1.numpy(), L["k"].numpy(), L["v"].numpy(), 16, 16,
                                                   0.0, "conservative", np.zeros_like(imp))
    # equal wherever the drift is not within 1e-6 of the 0.05 threshold (float32 reduction order)
    far = np.abs(drift.T.astype(np.float64) - 0.05) > 1e-6
    assert np.array_equal(mask[far], a["reuse"][far])
    reuse = a["reuse"]
    prev = O.pack(L["k"].numpy(), L["v"].numpy(), O.plan_from_codes(codes), 16)
    plan = O.plan_from_codes(codes, reuse)
    assert plan["fingerprint"] == pin["fingerprint"]
    cache = O.pack(k1.numpy(), v1.numpy(), plan, 16)
    assert packed_summary(cache.packed_data, cache.memory_bytes()) == pin["packed"]
    assert O.apply_reuse_mask(cache, prev, reuse) == pin["reuse_stats"]
    assert packed_summary(cache.packed_data, cache.memory_bytes()) == pin["after_reuse"]
    emask = W.lowest_importance_mask(torch.from_numpy(imp), c["evict_frac"], 4).numpy()
    assert array_digest(emask) == pin["evict_mask"]
    assert O.evict(cache, emask) == pin["removed"]
    assert packed_summary(cache.packed_data, cache.memory_bytes()) == pin["after_evict"]
    assert cache.resident_bytes() == pin["resident_after_evict"]
    ku, vu = O.unpack(cache)
    assert array_digest(ku) == pin["unpack_k"] and array_digest(vu) == pin["unpack_v"]
    out = _sampled_oracle_attention(L["q"].numpy()[:, :, a["rows"]], cache)
    assert np.linalg.norm(out - a["out"]) / np.linalg.norm(out) < 1e-5


@pytest.mark.parametrize("case", _cases(_pins(), "block"))
def test_model_block_attention(case, golden_small):
    """The reference block forward over a packed past (kv_execution="packed"): the oracle's
    attention of the block's own queries over unpack() + this step's K/V equals the reference's."""
    a = case_arrays(golden_small, case)
    cache = O.pack(a["k"], a["v"], O.plan_from_codes(a["codes"]), 16)
    out = O.packed_attention(a["q"], cache, k_new=a["k_new"], v_new=a["v_new"])
    assert np.linalg.norm(out - a["attn_out"]) / np.linalg.norm(a["attn_out"]) < 1e-5
