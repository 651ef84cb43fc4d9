"""Parity of the CUDA data plane with the reference (golden fixtures) and the CPU oracle.

Integer/byte work (codes, plans, packed bytes, scales, index lists, byte
accounting) must be bit-exact; dequantised K/V are bit-exact as well because
the dequantisation is a single fp32 multiply.
"""

import numpy as np
import pytest
import torch

from golden_lib import array_digest, case_arrays, load_pins, packed_summary
from oracle import shadowkv_oracle as O

pytestmark = pytest.mark.gpu

PRECISIONS = ("fp32", "fp16", "int8", "int4")


def _cases(kind):
    return sorted(c for c, v in load_pins()["cases"].items() if v["kind"] == kind)


def cu(x):
    return torch.from_numpy(np.ascontiguousarray(x)).cuda()


def eq(t, a):
    return np.array_equal(t.detach().cpu().numpy(), a)


@pytest.fixture(scope="module")
def skv():
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    import shadow_infer_b200.shadowkv as m
    return m


@pytest.mark.parametrize("case", _cases("pack"))
def test_plan_pack_unpack(case, skv, golden_small, golden_pins):
    a = case_arrays(golden_small, case)
    p = golden_pins["cases"][case]
    codes = cu(a["codes"])
    plan = skv.PrecisionPlan.from_codes(codes, reuse_mask=cu(a["reuse"]))
    for prec in PRECISIONS:
        assert eq(plan.flat_indices[prec], a[f"plan.flat.{prec}"]), prec
    assert np.array_equal(np.array(plan.evicted_entries, dtype=np.int64).reshape(-1, 2), a["plan.evicted"])
    assert eq(plan.reuse_flat, a["plan.reuse_flat"])
    assert plan.fingerprint == p["fingerprint"]
    # dict reuse mask gives the same plan
    rm = a["reuse"]
    rdict = {(t, h): bool(rm[t, h]) for t in range(rm.shape[0]) for h in range(rm.shape[1])}
    assert skv.PrecisionPlan.from_codes(codes, reuse_mask=rdict).fingerprint == p["fingerprint"]

    k, v = cu(a["k"]), cu(a["v"])
    cache = skv.PackedKVCache.pack(k, v, None, group_size=p["group"], plan=plan)["packed_kv"]
    assert packed_summary(cache.packed_data, cache.memory_bytes()) == p["summary"]
    assert cache.memory_bytes() == p["memory_bytes"]
    assert cache.data_plane_bytes() == p["data_plane_bytes"]
    assert cache.resident_bytes() == p["resident_bytes"]
    ku, vu = cache.unpack()
    assert eq(ku, a["unpack.k"]) and eq(vu, a["unpack.v"])
    kr, vr = cache.unpack_reference()
    assert torch.allclose(kr, ku, atol=1e-6, rtol=1e-6) and torch.allclose(vr, vu, atol=1e-6, rtol=1e-6)
    # precision-map path is identical to the plan path
    cmap = skv.PackedKVCache.pack(k, v, skv.codes_to_map(codes.cpu()),
                                  group_size=p["group"])["packed_kv"]
    assert packed_summary(cmap.packed_data, cmap.memory_bytes()) == p["summary"]


@pytest.mark.parametrize("case", _cases("pack"))
def test_dense_working_copy(case, skv, golden_small, golden_pins):
    from shadow_infer_b200.shadowkv.packed_kv_cache import run_pack
    a = case_arrays(golden_small, case)
    p = golden_pins["cases"][case]
    plan = skv.PrecisionPlan.from_codes(cu(a["codes"]), reuse_mask=cu(a["reuse"]))
    _, dk, dv = run_pack(cu(a["k"]), cu(a["v"]), plan, p["group"], dense=True)
    assert eq(dk, a["dense.k"]) and eq(dv, a["dense.v"])
    _, dk, dv = run_pack(cu(a["k"]), cu(a["v"]), plan, p["group"], dense=True,
                         k_prev=cu(a["k_prev"]), v_prev=cu(a["v_prev"]))
    assert eq(dk, a["dense_reuse.k"]) and eq(dv, a["dense_reuse.v"])


def test_host_tensors_round_trip(skv, golden_small, golden_pins):
    """Host (CPU) tensors in -> GPU compute -> host tensors out, same bytes."""
    case = "pack_b2_d64"
    a = case_arrays(golden_small, case)
    p = golden_pins["cases"][case]
    k, v = torch.from_numpy(a["k"]), torch.from_numpy(a["v"])
    plan = skv.PrecisionPlan.from_codes(torch.from_numpy(a["codes"]))
    cache = skv.PackedKVCache.pack(k, v, None, group_size=p["group"], plan=plan)["packed_kv"]
    assert all(t.device.type == "cpu" for d in cache.packed_data.values() for t in (d["k"], d["v"]))
    assert packed_summary(cache.packed_data, cache.memory_bytes()) == p["summary"]
    ku, vu = cache.unpack()
    assert ku.device.type == "cpu" and np.array_equal(ku.numpy(), a["unpack.k"])


@pytest.mark.parametrize("case", _cases("reuse"))
def test_reuse(case, skv, golden_small, golden_pins):
    a = case_arrays(golden_small, case)
    p = golden_pins["cases"][case]
    P = skv.PackedKVCache
    cur = P.pack(cu(a["k"]), cu(a["v"]), None, p["group"], plan=skv.PrecisionPlan.from_codes(cu(a["codes"])))["packed_kv"]
    prev = P.pack(cu(a["k_prev"]), cu(a["v_prev"]), None, p["group"],
                  plan=skv.PrecisionPlan.from_codes(cu(a["prev_codes"])))["packed_kv"]
    m = a["mask"]
    mdict = {(t, h): bool(m[t, h]) for t in range(m.shape[0]) for h in range(m.shape[1])}
    stats = cur.apply_reuse_mask(prev, mdict, return_stats=True)
    assert stats == p["stats"]
    assert packed_summary(cur.packed_data, cur.memory_bytes()) == p["summary"]
    ku, vu = cur.unpack()
    assert eq(ku, a["unpack.k"]) and eq(vu, a["unpack.v"])
    assert cur.apply_reuse_mask(prev, {}, return_stats=True) == {"applied": 0, "skipped_precision": 0}
    assert cur.apply_reuse_mask(prev, cu(m)) is None


def test_reuse_errors(skv):
    P = skv.PackedKVCache
    k = torch.randn(1, 2, 8, 64, device="cuda")
    codes = torch.full((8, 2), 3, dtype=torch.int8, device="cuda")
    a = P.pack(k, k, None, 16, plan=skv.PrecisionPlan.from_codes(codes))["packed_kv"]
    b = P.pack(torch.randn(1, 2, 8, 32, device="cuda"), torch.randn(1, 2, 8, 32, device="cuda"), None, 16,
               plan=skv.PrecisionPlan.from_codes(codes))["packed_kv"]
    with pytest.raises(ValueError, match="shape mismatch"):
        a.apply_reuse_mask(b, {(0, 0): True})
    c = P.pack(k, k, None, 32, plan=skv.PrecisionPlan.from_codes(codes))["packed_kv"]
    with pytest.raises(ValueError, match="group_size mismatch"):
        a.apply_reuse_mask(c, {(0, 0): True})


@pytest.mark.parametrize("case", _cases("evict"))
def test_evict(case, skv, golden_small, golden_pins):
    a = case_arrays(golden_small, case)
    p = golden_pins["cases"][case]
    cache = skv.PackedKVCache.pack(cu(a["k"]), cu(a["v"]), None, p["group"],
                                   plan=skv.PrecisionPlan.from_codes(cu(a["codes"])))["packed_kv"]
    m = a["mask"]
    entries = set(zip(*[x.tolist() for x in np.nonzero(m)]))
    assert cache.evict(entries) == p["removed"]
    assert cache.evict(entries) == 0
    ku, vu = cache.unpack()
    assert eq(ku, a["unpack.k"]) and eq(vu, a["unpack.v"])
    assert cache.evict(cu(a["whole_mask"])) == p["removed_whole"]
    assert "int8" not in cache.packed_data
    assert packed_summary(cache.packed_data, cache.memory_bytes()) == p["summary_after_whole"]
    assert cache.resident_bytes() == p["resident_after_whole"]


@pytest.mark.parametrize("case", _cases("admit"))
def test_admit(case, skv, golden_small, golden_pins):
    a = case_arrays(golden_small, case)
    p = golden_pins["cases"][case]
    prot = cu(a["protected"]) if "protected" in a else None
    out, pred, ev = skv.admit_codes(cu(a["codes"]), cu(a["importance"]), cu(a["sensitivity"]), p["budget"],
                                    p["B"], p["D"], sink_tokens=p["sink"], rd_allocation=p["rd"],
                                    allow_eviction=p["evict"], protected_mask=prot, group_size=p["group"])
    assert eq(out, a["out"])
    assert (pred, ev) == (p["predicted"], p["evicted"])
    assert skv.predict_codes_bytes(cu(a["codes"]), p["B"], p["D"], p["group"]) == p["predicted0"]


def test_admit_does_not_mutate_input(skv):
    codes = torch.ones(64, 8, dtype=torch.int8, device="cuda")
    imp = torch.rand(64, 8, device="cuda")
    before = codes.clone()
    skv.admit_codes(codes, imp, None, 1000, 1, 128, allow_eviction=True)
    assert torch.equal(codes, before)


def test_allocate_and_sensitivity(skv, golden_small):
    from shadow_infer_b200.shadowkv.shadowkv_agent import allocate_precision_codes
    a = case_arrays(golden_small, "allocate")
    for mode in ("aggressive", "balanced", "conservative", "unknown"):
        assert eq(allocate_precision_codes(cu(a["importance"]), mode), a[f"codes.{mode}"]), mode
    s = case_arrays(golden_small, "sensitivity")
    assert eq(skv.kv_sensitivity(cu(s["k"]), cu(s["v"])), s["sens"])


def test_full_cfg1(skv, golden_pins):
    from shadow_infer_b200 import workloads as W
    from shadow_infer_b200.shadowkv.packed_kv_cache import run_pack
    from shadow_infer_b200.shadowkv.shadowkv_agent import allocate_precision_codes
    pin = golden_pins["full"]["cfg1"]
    c = W.CONFIGS["cfg1"]
    k, v = W.kv_tensors(c["B"], c["H"], c["S"], c["D"], c["seed"])
    imp = W.importance_map(c["S"], c["H"], c["seed"], c["fractions"])
    k, v, imp = k.cuda(), v.cuda(), imp.cuda()
    codes = allocate_precision_codes(imp, "balanced")
    assert array_digest(codes) == pin["codes"]
    plan = skv.PrecisionPlan.from_codes(codes)
    assert plan.fingerprint == pin["fingerprint"]
    cache = skv.PackedKVCache.pack(k, v, None, 16, plan=plan)["packed_kv"]
    assert packed_summary(cache.packed_data, cache.memory_bytes()) == pin["packed"]
    ku, vu = cache.unpack()
    assert array_digest(ku) == pin["unpack_k"] and array_digest(vu) == pin["unpack_v"]
    _, dk, dv = run_pack(k, v, plan, 16, dense=True)
    assert array_digest(dk) == pin["dense_k"] and array_digest(dv) == pin["dense_v"]


def test_full_cfg2(skv, golden_pins):
    from shadow_infer_b200 import workloads as W
    from shadow_infer_b200.shadowkv.shadowkv_agent import allocate_precision_codes
    pin = golden_pins["full"]["cfg2"]
    I = W.cfg2_inputs()
    k, v = I["k"].cuda(), I["v"].cuda()
    sens = skv.kv_sensitivity(k, v)
    assert array_digest(sens) == pin["sensitivity"]
    imp = I["importance"].cuda()
    codes0 = allocate_precision_codes(imp, "balanced")
    adm, pred, ev = skv.admit_codes(codes0, imp, sens, I["budget"], 1, 128, sink_tokens=I["sink_tokens"],
                                    rd_allocation=True, allow_eviction=True)
    assert array_digest(adm) == pin["admitted"] and (pred, ev) == (pin["predicted"], pin["evicted"])
    reuse = I["reuse"].cuda()
    plan = skv.PrecisionPlan.from_codes(adm, reuse_mask=reuse)
    assert plan.fingerprint == pin["fingerprint"]
    cache = skv.PackedKVCache.pack(k, v, None, 16, plan=plan)["packed_kv"]
    assert packed_summary(cache.packed_data, cache.memory_bytes()) == pin["packed"]
    prev = skv.PackedKVCache.pack(I["k_prev"].cuda(), I["v_prev"].cuda(), None, 16,
                                  plan=skv.PrecisionPlan.from_codes(adm))["packed_kv"]
    assert cache.apply_reuse_mask(prev, reuse, return_stats=True) == pin["reuse_stats"]
    assert packed_summary(cache.packed_data, cache.memory_bytes()) == pin["after_reuse"]
    ku, vu = cache.unpack()
    assert array_digest(ku) == pin["unpack_k"] and array_digest(vu) == pin["unpack_v"]
    g = torch.Generator().manual_seed(pin["evict_seed"])
    emask = torch.rand(adm.shape, generator=g) < pin["evict_frac"]
    assert cache.evict(emask.cuda()) == pin["removed"]
    assert packed_summary(cache.packed_data, cache.memory_bytes()) == pin["after_evict"]
    assert cache.resident_bytes() == pin["resident_after_evict"]
    ke, ve = cache.unpack()
    assert array_digest(ke) == pin["unpack_evict_k"] and array_digest(ve) == pin["unpack_evict_v"]


def test_oracle_agrees_at_random_shapes(skv):
    """Seeded random shapes against the CPU oracle (odd D, B>1, every precision)."""
    rng = np.random.default_rng(7)
    for trial in range(6):
        B = int(rng.integers(1, 4)); H = int(rng.integers(1, 6)); S = int(rng.integers(1, 70))
        D = int(rng.choice([8, 16, 24, 33, 64, 96, 128, 256])); group = int(rng.choice([4, 16, 32]))
        k = (rng.standard_normal((B, H, S, D)) * rng.choice([1e-3, 1.0, 50.0])).astype(np.float32)
        v = rng.standard_normal((B, H, S, D)).astype(np.float32)
        codes = rng.integers(0, 5, size=(S, H)).astype(np.int8)
        plan_o = O.plan_from_codes(codes)
        ref = O.pack(k, v, plan_o, group)
        plan = skv.PrecisionPlan.from_codes(cu(codes))
        cache = skv.PackedKVCache.pack(cu(k), cu(v), None, group, plan=plan)["packed_kv"]
        assert packed_summary(cache.packed_data, cache.memory_bytes()) == packed_summary(ref.packed_data, ref.memory_bytes()), trial
        ku, vu = cache.unpack()
        ko, vo = O.unpack(ref)
        assert eq(ku, ko) and eq(vu, vo), trial


def _bucket_bytes(cache):
    out = {}
    for p, d in cache.packed_data.items():
        for key in ("k", "v", "scale_k", "scale_v"):
            t = d[key]
            out[(p, key)] = None if t is None else (tuple(t.shape), t.dtype, t.cpu().numpy().tobytes())
    return out


def test_pack_before_counts_reach_host(skv):
    """Packing launched on the device layout (the plan's counts still in flight) equals packing
    on the host layout, also when the slab guessed from the previous pack is too small (the
    device writes nothing and the buckets are packed again)."""
    from shadow_infer_b200 import _lib
    from shadow_infer_b200.shadowkv import packed_kv_cache as PKC
    rng = np.random.default_rng(31)
    B, H, S, D = 2, 8, 300, 128
    k, v = cu(rng.standard_normal((B, H, S, D)).astype(np.float32)), cu(rng.standard_normal((B, H, S, D)).astype(np.float32))
    lib = _lib.load()
    PKC._SLAB_HINT.clear()
    for probs in ((0.0, 0.1, 0.3, 0.5, 0.1), (0.7, 0.2, 0.1, 0.0, 0.0), (0.7, 0.2, 0.1, 0.0, 0.0),
                  (0.0, 0.0, 0.0, 1.0, 0.0), (0.0, 0.0, 0.0, 0.0, 1.0)):
        codes = cu(rng.choice(5, size=(S, H), p=probs).astype(np.int8))
        exact_plan = skv.PrecisionPlan.from_codes(codes)
        exact_plan.counts                                  # counts on the host: host layout
        want = skv.PackedKVCache.pack(k, v, None, 16, plan=exact_plan)["packed_kv"]
        hint = PKC._SLAB_HINT.get((0, B, H, S, D, 16))
        lazy_plan = skv.PrecisionPlan.from_codes(codes)    # counts in flight: device layout
        n0 = lib.skv_launch_count()
        got = skv.PackedKVCache.pack(k, v, None, 16, plan=lazy_plan)["packed_kv"]
        launches = lib.skv_launch_count() - n0
        assert launches == 2                               # layout + pack, the hint fits (same counts)
        assert _bucket_bytes(got) == _bucket_bytes(want)
        assert got.memory_bytes() == want.memory_bytes()
        ku, vu = got.unpack()
        kw, vw = want.unpack()
        assert torch.equal(ku, kw) and torch.equal(vu, vw)
        # a slab that is too small: shrink the hint below this layout, then pack again
        PKC._SLAB_HINT[(0, B, H, S, D, 16)] = 256
        small_plan = skv.PrecisionPlan.from_codes(codes)
        n0 = lib.skv_launch_count()
        again = skv.PackedKVCache.pack(k, v, None, 16, plan=small_plan)["packed_kv"]
        launches = lib.skv_launch_count() - n0
        stored = sum(1 for p in again.packed_data)
        assert launches == (3 if stored else 2)            # layout + empty pack + exact pack
        assert _bucket_bytes(again) == _bucket_bytes(want)
        assert hint is not None


@pytest.mark.parametrize("case", ["one_bucket_touched", "bucket_emptied_others_touched",
                                  "bucket_emptied_other_untouched", "every_bucket_touched"])
def test_evict_fresh_pack_paths(case, skv, monkeypatch):
    """evict on a freshly packed cache takes the pack's own bucket array (fast path) unless a
    non-empty bucket loses no entry, when it hands over to the general path; both must equal the
    oracle: removed count, packed bytes and index lists, memory accounting and the unpack."""
    calls = []
    orig = skv.PackedKVCache._evict_pending

    def spy(self, entries):
        r = orig(self, entries)
        calls.append(r)
        return r

    monkeypatch.setattr(skv.PackedKVCache, "_evict_pending", spy)
    rng = np.random.default_rng(len(case))
    B, H, S, D = 2, 3, 40, 64
    k = rng.standard_normal((B, H, S, D)).astype(np.float32)
    v = rng.standard_normal((B, H, S, D)).astype(np.float32)
    codes = rng.integers(1, 4, size=(S, H)).astype(np.int8)       # fp16 / int8 / int4 buckets
    sel = {
        "one_bucket_touched": codes == 2,                         # int8 only
        "bucket_emptied_others_touched": (codes == 3) | ((codes != 3) & (rng.random((S, H)) < 0.3)),
        "bucket_emptied_other_untouched": (codes == 3) | ((codes == 1) & (rng.random((S, H)) < 0.5)),
        "every_bucket_touched": rng.random((S, H)) < 0.25,
    }[case]
    if case == "one_bucket_touched":
        sel = sel & (rng.random((S, H)) < 0.5)
    fast = case in ("bucket_emptied_others_touched", "every_bucket_touched")
    cache = skv.PackedKVCache.pack(cu(k), cu(v), None, 16, plan=skv.PrecisionPlan.from_codes(cu(codes)))["packed_kv"]
    ref = O.pack(k, v, O.plan_from_codes(codes), 16)
    removed = cache.evict(cu(sel))
    assert removed == O.evict(ref, sel) == int(sel.sum())
    assert calls == ([removed] if fast else [None])
    assert packed_summary(cache.packed_data, cache.memory_bytes()) == packed_summary(ref.packed_data,
                                                                                     ref.memory_bytes())
    assert cache.memory_bytes() == ref.memory_bytes() and cache.resident_bytes() == ref.resident_bytes()
    ku, vu = cache.unpack()
    ko, vo = O.unpack(ref)
    assert eq(ku, ko) and eq(vu, vo)
    # idempotent: the same set again removes nothing
    assert cache.evict(cu(sel)) == 0


def test_evict_chain_then_views_and_attention(skv):
    """Three evictions in a row on a freshly packed cache (each leaves the survivors' slab with its
    views still unmade), then reuse from the evicted cache, unpack, the bucket views and packed
    attention, each against the oracle after the same evictions."""
    rng = np.random.default_rng(31)
    B, H, S, D = 2, 4, 300, 128
    k = rng.standard_normal((B, H, S, D)).astype(np.float32)
    v = rng.standard_normal((B, H, S, D)).astype(np.float32)
    codes = rng.integers(0, 5, size=(S, H)).astype(np.int8)
    cache = skv.PackedKVCache.pack(cu(k), cu(v), None, 16, plan=skv.PrecisionPlan.from_codes(cu(codes)))["packed_kv"]
    ref = O.pack(k, v, O.plan_from_codes(codes), 16)
    for frac in (0.2, 0.3, 0.5):
        sel = rng.random((S, H)) < frac
        assert cache.evict(cu(sel)) == O.evict(ref, sel)
        assert cache.memory_bytes() == ref.memory_bytes()
    ku, vu = cache.unpack()
    ko, vo = O.unpack(ref)
    assert eq(ku, ko) and eq(vu, vo)
    q = rng.standard_normal((B, H, 70, D)).astype(np.float16)
    out = skv.packed_attention(torch.from_numpy(q).cuda(), cache).cpu().numpy()
    want = O.packed_attention(q.astype(np.float32), ref)
    assert float(np.linalg.norm(out - want) / np.linalg.norm(want)) < 1e-3
    assert packed_summary(cache.packed_data, cache.memory_bytes()) == packed_summary(ref.packed_data, ref.memory_bytes())
    assert cache.resident_bytes() == ref.resident_bytes()
