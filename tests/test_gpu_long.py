"""The long-context (cfg5) and batched denoising (cfg4) workloads on the GPU.

* Head slices pinned to the reference itself (``make_golden.py`` records its plan, packed
  bytes, reuse, eviction and unpack digests and its fp32 attention on sampled query rows):
  bit-exact for every byte, index and count; attention within relative L2 1e-3.
* Whole layers at their full size (cfg5: 32 heads x 32768 tokens, 17.6 TFLOP of attention;
  cfg4: batch 8) against the oracle through properties that do not need the oracle to run the
  whole layer: the plan's fingerprint and byte totals, per-head unpack equality (quantisation
  is per (token, head) row, so a head packed inside the layer unpacks exactly as the same head
  packed alone) and attention on sampled query rows of sampled heads.
"""

import numpy as np
import pytest
import torch

from golden_lib import array_digest, case_arrays, packed_summary
from oracle import shadowkv_oracle as O

pytestmark = pytest.mark.gpu

REL_L2_TOL = 1e-3


def rel_l2(a, b):
    a = np.asarray(a, dtype=np.float64)
    b = np.asarray(b, dtype=np.float64)
    return float(np.linalg.norm(a - b) / max(np.linalg.norm(b), 1e-30))


@pytest.fixture(scope="module")
def skv():
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    import shadow_infer_b200.shadowkv as m
    return m


@pytest.fixture(scope="module")
def W():
    from shadow_infer_b200 import workloads
    return workloads


def _summary(cache):
    return packed_summary(cache.packed_data, cache.memory_bytes())


def test_cfg5_slice_matches_reference(skv, W, golden_pins, golden_small):
    from shadow_infer_b200.shadowkv.shadowkv_agent import allocate_precision_codes
    pin = golden_pins["full"]["cfg5_slice"]
    a = case_arrays(golden_small, "cfg5_slice")
    h0, h1 = pin["heads"]
    L = W.cfg5_layer(h0, h1)
    codes = allocate_precision_codes(L["importance"][:, h0:h1].contiguous().cuda(), "balanced")
    assert array_digest(codes) == pin["codes"]
    plan = skv.PrecisionPlan.from_codes(codes)
    assert plan.fingerprint == pin["fingerprint"]
    cache = skv.PackedKVCache.pack(L["k"].cuda(), L["v"].cuda(), None, 16, plan=plan)["packed_kv"]
    assert _summary(cache) == pin["packed"]
    assert cache.data_plane_bytes() == pin["data_plane_bytes"] and cache.resident_bytes() == pin["resident_bytes"]
    ku, vu = cache.unpack()
    assert array_digest(ku) == pin["unpack_k"] and array_digest(vu) == pin["unpack_v"]
    rows = torch.from_numpy(a["rows"])
    out = skv.packed_attention(L["q"][:, :, rows].contiguous().cuda(), cache)
    assert rel_l2(out.cpu().numpy(), a["out"]) < REL_L2_TOL


def test_cfg5_full_layer(skv, W):
    """All 32 heads of a long-context layer: plan, byte totals, per-head unpack and the full
    attention (every query row computed, sampled rows of three heads checked)."""
    from shadow_infer_b200.shadowkv.shadowkv_agent import allocate_precision_codes
    c = W.CONFIGS["cfg5"]
    L = W.cfg5_layer()
    imp = L["importance"]
    codes = allocate_precision_codes(imp.cuda(), "balanced")
    codes_o = O.allocate_precision_codes(imp.numpy(), "balanced")
    assert np.array_equal(codes.cpu().numpy(), codes_o)
    frac = [float((codes_o == i).mean()) for i in range(4)]
    assert abs(frac[1] - 0.10) < 0.001 and abs(frac[2] - 0.30) < 0.001 and abs(frac[3] - 0.60) < 0.001
    plan = skv.PrecisionPlan.from_codes(codes)
    assert plan.fingerprint == O.plan_from_codes(codes_o)["fingerprint"]
    cache = skv.PackedKVCache.pack(L["k"].cuda(), L["v"].cuda(), None, 16, plan=plan)["packed_kv"]
    assert cache.memory_bytes() == O.predict_codes_bytes(codes_o, c["B"], c["D"])
    ku, vu = cache.unpack()
    q = L["q"].cuda()
    out = skv.packed_attention(q, cache)
    heads = (0, 11, 31)
    for h in heads:
        ch = O.pack(L["k"][:, h:h + 1].numpy(), L["v"][:, h:h + 1].numpy(),
                    O.plan_from_codes(np.ascontiguousarray(codes_o[:, h:h + 1])), 16)
        ko, vo = O.unpack(ch)
        assert np.array_equal(ku[:, h:h + 1].cpu().numpy(), ko) and np.array_equal(vu[:, h:h + 1].cpu().numpy(), vo)
        rows = W.sample_rows(c["S"], 48, h)
        want = O.packed_attention(L["q"][:, h:h + 1, rows].float().numpy(), ch)
        got = out[:, h:h + 1, rows.cuda()].cpu().numpy()
        assert rel_l2(got, want) < REL_L2_TOL, h


def test_cfg4_slice_matches_reference(skv, W, golden_pins, golden_small):
    """Batch 8: one denoising step of a 4-head slice -- drift, reuse decision, re-pack, reuse,
    eviction of the 25 % lowest-importance entries, unpack, attention on sampled rows."""
    from shadow_infer_b200.shadowkv.shadowkv_agent import allocate_precision_codes, decide_reuse_mask
    pin = golden_pins["full"]["cfg4_slice"]
    a = case_arrays(golden_small, "cfg4_slice")
    c = W.CONFIGS["cfg4"]
    h0, h1 = pin["heads"]
    L = W.cfg4_layer(h0, h1)
    nk, nv = W.drift_noise(c["B"], c["S"], c["D"], 10_000, 1, h0, h1)
    k1, v1 = W.apply_drift(L["k"], nk), W.apply_drift(L["v"], nv)
    assert array_digest(k1) == pin["k1"]
    imp = L["importance"][:, h0:h1].contiguous().cuda()
    codes = allocate_precision_codes(imp, "balanced")
    assert array_digest(codes) == pin["codes"]
    k0d, v0d, k1d, v1d = L["k"].cuda(), L["v"].cuda(), k1.cuda(), v1.cuda()
    mask, stats, drift = decide_reuse_mask(k1d, v1d, k0d, v0d, 16, 16, 0.0, "conservative", torch.zeros_like(imp),
                                           return_drift=True)
    far = (drift.double() - 0.05).abs().cpu().numpy() > 1e-6
    assert np.array_equal(mask.cpu().numpy()[far], a["reuse"][far])
    reuse = torch.from_numpy(a["reuse"]).cuda()
    prev = skv.PackedKVCache.pack(k0d, v0d, None, 16, plan=skv.PrecisionPlan.from_codes(codes))["packed_kv"]
    plan = skv.PrecisionPlan.from_codes(codes, reuse_mask=reuse)
    assert plan.fingerprint == pin["fingerprint"]
    cur = skv.PackedKVCache.pack(k1d, v1d, None, 16, plan=plan)["packed_kv"]
    assert _summary(cur) == pin["packed"]
    assert cur.apply_reuse_mask(prev, reuse, return_stats=True) == pin["reuse_stats"]
    assert _summary(cur) == pin["after_reuse"]
    emask = W.lowest_importance_mask(imp, c["evict_frac"], 4)
    assert array_digest(emask) == pin["evict_mask"]
    assert cur.evict(emask) == pin["removed"]
    assert _summary(cur) == pin["after_evict"] and cur.resident_bytes() == pin["resident_after_evict"]
    ku, vu = cur.unpack()
    assert array_digest(ku) == pin["unpack_k"] and array_digest(vu) == pin["unpack_v"]
    rows = torch.from_numpy(a["rows"])
    out = skv.packed_attention(L["q"][:, :, rows].contiguous().cuda(), cur)
    assert rel_l2(out.cpu().numpy(), a["out"]) < REL_L2_TOL


def test_cfg4_full_layer_attention(skv, W):
    """A whole batch-8 layer (32 heads) after a reuse step and the 25 % eviction: sampled rows of
    sampled heads against the oracle, every batch entry."""
    from shadow_infer_b200.shadowkv.shadowkv_agent import allocate_precision_codes
    c = W.CONFIGS["cfg4"]
    L = W.cfg4_layer()
    codes = allocate_precision_codes(L["importance"].cuda(), "balanced")
    cache = skv.PackedKVCache.pack(L["k"].cuda(), L["v"].cuda(), None, 16,
                                   plan=skv.PrecisionPlan.from_codes(codes))["packed_kv"]
    emask = W.lowest_importance_mask(L["importance"], c["evict_frac"], 4)
    n_ev = cache.evict(emask.cuda())
    assert n_ev == int(emask.sum())
    out = skv.packed_attention(L["q"].cuda(), cache)
    codes_o = codes.cpu().numpy()
    for h in (3, 17, 30):
        ch = O.pack(L["k"][:, h:h + 1].numpy(), L["v"][:, h:h + 1].numpy(),
                    O.plan_from_codes(np.ascontiguousarray(codes_o[:, h:h + 1])), 16)
        O.evict(ch, np.ascontiguousarray(emask[:, h:h + 1].numpy()))
        rows = W.sample_rows(c["S"], 32, h)
        want = O.packed_attention(L["q"][:, h:h + 1, rows].float().numpy(), ch)
        got = out[:, h:h + 1, rows.cuda()].cpu().numpy()
        assert rel_l2(got, want) < REL_L2_TOL, h
