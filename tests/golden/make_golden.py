"""Generate the golden fixtures by running the reference implementation itself.

Usage::

    python tests/golden/make_golden.py --reference <path to the shadow-infer source tree>

The reference (``shadowinfer`` package, pure Python + torch CPU) is imported
from its source tree with a no-op ``structlog`` stand-in (``_stub/``).  It is
run on seeded inputs and its outputs are written to

* ``small_cases.npz`` -- inputs and full outputs of small edge cases;
* ``pins.json``       -- scalar outputs of those cases, plus SHA-256 digests of
  full-size outputs of the cfg1 / cfg2 pipelines (inputs regenerated from
  ``shadow_infer_b200.workloads`` at test time).

Nothing at test time imports the reference; only these files are read.
"""

from __future__ import annotations

import argparse
import json
import os
import sys
import types

import numpy as np
import torch

HERE = os.path.dirname(os.path.abspath(__file__))
REPO = os.path.dirname(os.path.dirname(HERE))
sys.path.insert(0, REPO)
sys.path.insert(0, HERE)

from golden_lib import (BLOCK_PARAM_ORDER, PINS_JSON, SMALL_NPZ, array_digest, block_params,  # noqa: E402
                        irap_scores, packed_summary, paged_apply, reuse_inputs, state_digest, to_numpy)

from shadow_infer_b200 import workloads as W  # noqa: E402

PRECISIONS = ("fp32", "fp16", "int8", "int4")


def _import_reference(path: str):
    sys.path.insert(0, os.path.join(HERE, "_stub"))
    sys.path.insert(0, path)
    from shadowinfer.shadowkv import rd_allocator, precision_plan, packed_kv_cache  # noqa
    from shadowinfer.shadowkv.shadowkv_agent import ShadowKVAgent  # noqa
    from shadowinfer.shadowkv import paged_kv_store, importance_model  # noqa
    from shadowinfer.models import diffusion_llama, simple_diffusion_llm  # noqa
    return types.SimpleNamespace(
        rd=rd_allocator, plan=precision_plan, pkc=packed_kv_cache, Agent=ShadowKVAgent, paged=paged_kv_store,
        imp=importance_model, llama=diffusion_llama, sdl=simple_diffusion_llm,
    )


ARR: dict = {}
PINS: dict = {"cases": {}, "full": {}}


def put(case: str, name: str, x) -> None:
    ARR[f"{case}/{name}"] = to_numpy(x)


def packed_arrays(case: str, prefix: str, packed) -> None:
    """Store every tensor and list of a reference packed cache."""
    for pname, d in packed.packed_data.items():
        for key in ("k", "v", "scale_k", "scale_v"):
            if d.get(key) is not None:
                put(case, f"{prefix}{pname}.{key}", d[key])
        put(case, f"{prefix}{pname}.indices", np.array(d["indices"], dtype=np.int64).reshape(-1, 2))
        if "byte_offsets" in d:
            put(case, f"{prefix}{pname}.byte_offsets", np.array(d["byte_offsets"], dtype=np.int64).reshape(-1, 4))


def codes_of(gen, S, H, probs):
    p = torch.tensor(probs, dtype=torch.float64)
    return torch.multinomial(p, S * H, replacement=True, generator=gen).reshape(S, H).to(torch.int8)


def kv(gen, B, H, S, D, zero_rows=0, big=False):
    k = torch.randn(B, H, S, D, generator=gen)
    v = torch.randn(B, H, S, D, generator=gen)
    m = torch.rand(B, H, S, D, generator=gen) < 0.01
    k = torch.where(m, k * 8, k)
    if zero_rows:
        for i in range(zero_rows):
            k[0, i % H, (3 * i) % S, :] = 0.0
            v[-1, (i + 1) % H, (5 * i + 1) % S, :] = 0.0
    if big:
        k[0, 0, 0, :4] = torch.tensor([7.0e4, -1.0e5, 65519.0, 65520.0])
    return k.contiguous(), v.contiguous()


def pack_case(R, case, gen, B, H, S, D, probs, group=16, reuse_p=0.3, zero_rows=0, big=False):
    k, v = kv(gen, B, H, S, D, zero_rows, big)
    codes = codes_of(gen, S, H, probs)
    reuse = torch.rand(S, H, generator=gen) < reuse_p
    reuse_dict = {(t, h): bool(reuse[t, h]) for t in range(S) for h in range(H)}
    plan = R.plan.PrecisionPlan.from_codes(codes, reuse_mask=reuse_dict)
    packed = R.pkc.PackedKVCache.pack(k, v, None, group_size=group, plan=plan)["packed_kv"]
    # the map path must agree with the plan path
    pmap = R.plan.codes_to_map(codes)
    packed_map = R.pkc.PackedKVCache.pack(k, v, pmap, group_size=group)["packed_kv"]
    assert packed_summary(packed.packed_data, packed.memory_bytes()) == packed_summary(
        packed_map.packed_data, packed_map.memory_bytes())
    ku, vu = packed.unpack()
    kr, vr = packed.unpack_reference()
    put(case, "k", k); put(case, "v", v); put(case, "codes", codes); put(case, "reuse", reuse)
    for p in PRECISIONS:
        put(case, f"plan.flat.{p}", plan.flat_indices[p])
    put(case, "plan.evicted", np.array(plan.evicted_entries, dtype=np.int64).reshape(-1, 2))
    put(case, "plan.reuse_flat", plan.reuse_flat)
    packed_arrays(case, "packed.", packed)
    put(case, "unpack.k", ku); put(case, "unpack.v", vu)
    assert torch.allclose(kr, ku, atol=1e-6, rtol=1e-6) and torch.allclose(vr, vu, atol=1e-6, rtol=1e-6)
    # dense working copy of compress_kv (no previous step, then with one)
    fake = types.SimpleNamespace(int4_group_size=group)
    core = R.Agent._compress_kv_with_plan(fake, k, v, None, None, plan, build_scale_map=False)
    put(case, "dense.k", core["k"]); put(case, "dense.v", core["v"])
    kp = k + 0.01 * torch.randn(k.shape, generator=gen)
    vp = v + 0.01 * torch.randn(v.shape, generator=gen)
    core2 = R.Agent._compress_kv_with_plan(fake, k, v, kp, vp, plan, build_scale_map=False)
    put(case, "k_prev", kp); put(case, "v_prev", vp)
    put(case, "dense_reuse.k", core2["k"]); put(case, "dense_reuse.v", core2["v"])
    PINS["cases"][case] = {
        "kind": "pack", "B": B, "H": H, "S": S, "D": D, "group": group,
        "fingerprint": plan.fingerprint,
        "summary": packed_summary(packed.packed_data, packed.memory_bytes()),
        "memory_bytes": packed.memory_bytes(),
        "data_plane_bytes": packed.data_plane_bytes(),
        "resident_bytes": packed.resident_bytes(),
    }
    return k, v, codes, packed


def reuse_case(R, case, gen, B, H, S, D, group=16):
    k, v = kv(gen, B, H, S, D)
    probs = (0.15, 0.3, 0.25, 0.2, 0.1)
    codes = codes_of(gen, S, H, probs)
    prev_codes = torch.where(torch.rand(S, H, generator=gen) < 0.6, codes, codes_of(gen, S, H, probs))
    kp = k + 0.01 * torch.randn(k.shape, generator=gen)
    vp = v + 0.01 * torch.randn(v.shape, generator=gen)
    mask = torch.rand(S, H, generator=gen) < 0.5
    mask_dict = {(t, h): bool(mask[t, h]) for t in range(S) for h in range(H)}
    P = R.pkc.PackedKVCache
    cur = P.pack(k, v, R.plan.codes_to_map(codes), group_size=group)["packed_kv"]
    prev = P.pack(kp, vp, R.plan.codes_to_map(prev_codes), group_size=group)["packed_kv"]
    stats = cur.apply_reuse_mask(prev, mask_dict, return_stats=True)
    put(case, "k", k); put(case, "v", v); put(case, "k_prev", kp); put(case, "v_prev", vp)
    put(case, "codes", codes); put(case, "prev_codes", prev_codes); put(case, "mask", mask)
    packed_arrays(case, "after.", cur)
    ku, vu = cur.unpack()
    put(case, "unpack.k", ku); put(case, "unpack.v", vu)
    PINS["cases"][case] = {
        "kind": "reuse", "B": B, "H": H, "S": S, "D": D, "group": group, "stats": stats,
        "summary": packed_summary(cur.packed_data, cur.memory_bytes()),
    }


def evict_case(R, case, gen, B, H, S, D, group=16, frac=0.25):
    k, v = kv(gen, B, H, S, D)
    codes = codes_of(gen, S, H, (0.2, 0.3, 0.3, 0.15, 0.05))
    cache = R.pkc.PackedKVCache.pack(k, v, R.plan.codes_to_map(codes), group_size=group)["packed_kv"]
    mask = torch.rand(S, H, generator=gen) < frac
    ts, hs = torch.nonzero(mask, as_tuple=True)
    entries = set(zip(ts.tolist(), hs.tolist()))
    removed = cache.evict(entries)
    again = cache.evict(entries)
    put(case, "k", k); put(case, "v", v); put(case, "codes", codes); put(case, "mask", mask)
    packed_arrays(case, "after.", cache)
    ku, vu = cache.unpack()
    put(case, "unpack.k", ku); put(case, "unpack.v", vu)
    # evicting a whole bucket deletes its key
    whole = torch.zeros(S, H, dtype=torch.bool)
    idx = cache.packed_data.get("int8", {}).get("indices", [])
    for t, h in idx:
        whole[t, h] = True
    removed_whole = cache.evict(set(idx))
    put(case, "whole_mask", whole)
    PINS["cases"][case] = {
        "kind": "evict", "B": B, "H": H, "S": S, "D": D, "group": group,
        "removed": removed, "removed_again": again, "removed_whole": removed_whole,
        "summary_after_whole": packed_summary(cache.packed_data, cache.memory_bytes()),
        "resident_after_whole": cache.resident_bytes(),
    }


def admit_case(R, case, gen, S, H, B, D, budget_frac, *, sink=0, rd=True, evict=False,
               protected_p=0.0, ties=False, group=16, signed_zero=False, nan=False,
               sens_mismatch=False, budget_abs=None):
    probs = (0.1, 0.4, 0.25, 0.2, 0.05)
    codes = codes_of(gen, S, H, probs)
    if ties:
        imp = (torch.randint(0, 3, (S, H), generator=gen).float() * 0.5)
        sens = torch.ones(S, H)
    else:
        imp = torch.rand(S, H, generator=gen)
        k, v = kv(gen, B, H, S, D)
        sens = R.rd.kv_sensitivity(k, v)
    if signed_zero:
        z = torch.rand(S, H, generator=gen) < 0.2
        imp = torch.where(z, torch.where(torch.rand(S, H, generator=gen) < 0.5, -0.0, 0.0), imp)
    if nan:
        imp[1, 0] = float("nan")
        imp[S // 2, H - 1] = float("nan")
    if sens_mismatch:
        sens = torch.ones(S + 1, H)
    protected = None
    if protected_p > 0:
        protected = torch.rand(S, H, generator=gen) < protected_p
    predicted0 = R.rd.predict_codes_bytes(codes, B, D, group_size=group)
    budget = budget_abs if budget_abs is not None else int(predicted0 * budget_frac)
    out, pred, ev = R.rd.admit_codes(
        codes, imp, sens, budget, batch=B, head_dim=D, sink_tokens=sink, rd_allocation=rd,
        allow_eviction=evict, protected_mask=protected, group_size=group)
    put(case, "codes", codes); put(case, "importance", imp); put(case, "sensitivity", sens)
    if protected is not None:
        put(case, "protected", protected)
    put(case, "out", out)
    PINS["cases"][case] = {
        "kind": "admit", "S": S, "H": H, "B": B, "D": D, "group": group, "budget": budget,
        "sink": sink, "rd": rd, "evict": evict, "predicted": pred, "evicted": ev,
        "predicted0": predicted0,
    }


def allocate_case(R, case):
    vals = []
    for base in (0.0, 0.1, 0.2, 0.3, 0.4, 0.5, 0.6, 0.7, 0.8, 0.9, 1.0):
        for d in (-1e-6, 0.0, 1e-6):
            vals.append(base + d)
    vals += [0.7000000000000001, 0.19999999, 0.20000001, -0.5, 2.0]
    imp = torch.tensor(vals, dtype=torch.float32).reshape(-1, 1).repeat(1, 3)
    put(case, "importance", imp)
    for mode in ("aggressive", "balanced", "conservative", "unknown"):
        put(case, f"codes.{mode}", R.Agent.allocate_precision_codes(None, imp, mode))
    PINS["cases"][case] = {"kind": "allocate"}


def sensitivity_case(R, case, gen):
    k, v = kv(gen, 2, 3, 17, 64)
    put(case, "k", k); put(case, "v", v); put(case, "sens", R.rd.kv_sensitivity(k, v))
    PINS["cases"][case] = {"kind": "sensitivity"}


def attention_case(R, case, gen, B, H, S, D):
    k, v = kv(gen, B, H, S, D)
    codes = codes_of(gen, S, H, (0.1, 0.3, 0.3, 0.25, 0.05))
    packed = R.pkc.PackedKVCache.pack(k, v, R.plan.codes_to_map(codes), group_size=16)["packed_kv"]
    q = torch.randn(B, H, S, D, generator=gen).to(torch.float16)
    ku, vu = packed.unpack()
    qf = q.float()
    scores = torch.matmul(qf, ku.transpose(-2, -1)) / (D ** 0.5)
    out = torch.matmul(torch.softmax(scores, dim=-1), vu)
    put(case, "k", k); put(case, "v", v); put(case, "codes", codes); put(case, "q", q)
    put(case, "out", out)
    PINS["cases"][case] = {"kind": "attention", "B": B, "H": H, "S": S, "D": D}


def attention_gqa_case(R, case, gen, B, H_kv, n_rep, S_past, S_new, S_q, D, probs=(0.1, 0.3, 0.3, 0.25, 0.05)):
    """The model attention over a packed past plus this step's own K/V, as DiffusionLlamaAttention
    runs it (diffusion_llama.py:376-390: cat(past, new), _repeat_kv, softmax(q k^T / sqrt(D)) v),
    with the past from the reference PackedKVCache (pack -> unpack)."""
    k, v = kv(gen, B, H_kv, S_past, D)
    codes = codes_of(gen, S_past, H_kv, probs)
    packed = R.pkc.PackedKVCache.pack(k, v, R.plan.codes_to_map(codes), group_size=16)["packed_kv"]
    k_new = torch.randn(B, H_kv, S_new, D, generator=gen)
    v_new = torch.randn(B, H_kv, S_new, D, generator=gen)
    q = torch.randn(B, H_kv * n_rep, S_q, D, generator=gen).to(torch.float16)
    past_k, past_v = packed.unpack()
    k_all = torch.cat((past_k, k_new), dim=2)
    v_all = torch.cat((past_v, v_new), dim=2)
    k_exp = R.llama._repeat_kv(k_all, n_rep)
    v_exp = R.llama._repeat_kv(v_all, n_rep)
    scores = torch.matmul(q.float(), k_exp.transpose(-2, -1)) / (D ** 0.5)
    out = torch.matmul(torch.softmax(scores, dim=-1), v_exp)
    for name, x in (("k", k), ("v", v), ("codes", codes), ("k_new", k_new), ("v_new", v_new), ("q", q),
                    ("out", out)):
        put(case, name, x)
    PINS["cases"][case] = {"kind": "attention_gqa", "B": B, "H_kv": H_kv, "n_rep": n_rep, "S_past": S_past,
                           "S_new": S_new, "S_q": S_q, "D": D}


def global_budget_case(R, case, gen, B, H, S, D, layers, budget_frac, sink, *, probs=(0.2, 0.3, 0.25, 0.2, 0.05),
                       group=16, dense=(), packed_only=(), no_importance=(), ties=False, budget_abs=None):
    """KVCacheManager.enforce_global_budget over several packed layers (kv_cache_manager.py:129-200)."""
    from shadowinfer.core.structs import KVCacheEntry
    from shadowinfer.shadowkv.kv_cache_manager import KVCacheManager
    mgr = KVCacheManager(num_layers=layers)
    packs = []
    for L in range(layers):
        k, v = kv(gen, B, H, S, D)
        codes = codes_of(gen, S, H, probs)
        imp = torch.rand(S, H, generator=gen)
        if ties:
            imp = torch.round(imp * 4) / 4
        imp[:sink] = 1.0
        plan = R.plan.PrecisionPlan.from_codes(codes)
        packed = R.pkc.PackedKVCache.pack(k, v, None, group_size=group, plan=plan)["packed_kv"]
        if L in packed_only:
            mgr.store_packed(L, packed)
        else:
            mgr.store(L, KVCacheEntry(k_tensor=k if L in dense else None, v_tensor=v if L in dense else None,
                                      precision="mixed", packed_kv=packed))
        if L not in no_importance:
            mgr.set_importance_matrix(L, imp)
        put(case, f"L{L}.k", k); put(case, f"L{L}.v", v); put(case, f"L{L}.codes", codes); put(case, f"L{L}.imp", imp)
        packs.append(packed)
    before = mgr.get_memory_usage()
    budget = budget_abs if budget_abs is not None else int(before * budget_frac)
    evicted = mgr.enforce_global_budget(budget, sink)
    for L, packed in enumerate(packs):
        remaining = np.zeros((S, H), dtype=np.uint8)
        for d in packed.packed_data.values():
            for t, h in d["indices"]:
                remaining[t, h] = 1
        put(case, f"L{L}.remaining", remaining)
    PINS["cases"][case] = {
        "kind": "global_budget", "B": B, "H": H, "S": S, "D": D, "group": group, "layers": layers,
        "sink": sink, "budget": budget, "dense": list(dense), "packed_only": list(packed_only),
        "no_importance": list(no_importance), "usage_before": before, "evicted": evicted,
        "usage_after": mgr.get_memory_usage(),
        "resident_after": [p.resident_bytes() for p in packs],
    }


def _paged_op(store, op, B, H, D):
    return paged_apply(store, op, B, H, D, torch.from_numpy)


def paged_state(store):
    from oracle.paged_store_oracle import store_state
    st = store_state(store, to_numpy)
    st["pages_digest"] = state_digest(st.pop("page_digests"))
    return st


def paged_case(R, case, B, H, D, P, G, ops):
    """Replay an operation script on the reference PagedKVStore (paged_kv_store.py) and pin its
    return values / ValueErrors, page layout, slot pool, counters, ledgers, page-tensor digests
    and gather digests after every operation."""
    store = R.paged.PagedKVStore(B, H, D, page_size=P, device="cpu", int4_group_size=G)
    results = []
    for op in ops:
        try:
            ret, err = _paged_op(store, op, B, H, D), False
        except ValueError:
            ret, err = None, True
        k, v = store.gather()
        results.append({"ret": ret, "error": err, "state": paged_state(store),
                        "gather": [array_digest(k), array_digest(v)], "S_out": int(k.shape[2])})
    PINS["cases"][case] = {"kind": "paged", "B": B, "H": H, "D": D, "P": P, "G": G, "ops": ops,
                           "results": results}


def paged_random_ops(R, B, H, D, P, G, n_ops, seed):
    """A seeded random script: appends of random lengths and precisions (sticky), evictions of
    full tokens / single heads / absent pairs, rewrites inside and across pages (many valid,
    some refused), invalid inputs and one clear.  Chosen against a live reference store."""
    rng = np.random.default_rng(seed)
    store = R.paged.PagedKVStore(B, H, D, page_size=P, device="cpu", int4_group_size=G)
    ops, prec = [], "fp16"
    for i in range(n_ops):
        r = rng.random()
        s = int(seed * 1000 + i)
        if r < 0.45 or store.max_seq == 0:
            if rng.random() < 0.4:
                prec = PRECISIONS[int(rng.integers(4))]
            T = int(rng.choice([0, 1, 2, P - 1, P, P + 1, 2 * P + 3, int(rng.integers(1, 3 * P))]))
            op = ["append", max(T, 0), prec, s]
        elif r < 0.68:
            S = store.max_seq
            pairs = set()
            for _ in range(int(rng.integers(1, 4))):
                t = int(rng.integers(0, S + 2))
                if rng.random() < 0.5:
                    pairs.update((t, h) for h in range(H))
                else:
                    pairs.add((t, int(rng.integers(0, H + 1))))
            op = ["evict", sorted([list(p) for p in pairs])]
        elif r < 0.92:
            live = [store.pages[sl] for sl in store._order]
            if live and rng.random() < 0.8:
                pg = live[int(rng.integers(len(live)))]
                a = pg.start_token + int(rng.integers(pg.num_tokens))
                span = pg.end_token - a + (int(rng.integers(0, P)) if rng.random() < 0.3 else 0)
                T = int(rng.integers(1, span + 1))
                p = pg.precision if rng.random() < 0.9 else PRECISIONS[int(rng.integers(4))]
                op = ["rewrite", a, T, p, s]
            else:
                op = ["rewrite", int(rng.integers(-1, store.max_seq + 2)), int(rng.integers(0, 4)), prec, s]
        elif r < 0.97:
            kind = ["precision", "heads", "dim", "batch", "ndim", "kv_mismatch"][int(rng.integers(6))]
            p = "bf16" if kind == "precision" else prec
            op = ["append_bad", kind, p, s] if rng.random() < 0.5 else ["rewrite_bad", 0, kind, p, s]
        else:
            op = ["clear"]
        try:
            _paged_op(store, op, B, H, D)
        except ValueError:
            pass
        ops.append(op)
    return ops


def paged_cases(R):
    full = lambda *ts: [[t, h] for t in ts for h in range(4)]  # noqa: E731  (H = 4 scripts)
    a = lambda T, p, s: ["append", T, p, s]  # noqa: E731
    paged_case(R, "paged_fp16_evict", 2, 4, 32, 8, 16, [
        a(5, "fp16", 1), a(5, "fp16", 2), a(5, "fp16", 3), a(4, "fp16", 4),
        ["evict", full(2, 4, 5, 17) + [[10, 0], [10, 1], [12, 2], [12, 3]]],
        ["evict", [[5, 0], [5, 3], [24, 0], [0, 7]]],
        ["evict", [[10, 2], [10, 3]]],
        ["rewrite", 0, 2, "fp16", 5], ["rewrite", 9, 3, "fp16", 6],
        a(2, "fp16", 7), ["evict", full(18, 19, 20)], a(3, "fp16", 8),
    ])
    paged_case(R, "paged_int8_rewrite", 2, 4, 32, 8, 16, [
        a(8, "int8", 11), a(8, "int8", 12), a(8, "int8", 13), a(2, "int8", 14),
        ["rewrite", 4, 16, "int8", 15], ["rewrite", 0, 4, "fp16", 16], ["rewrite", 20, 8, "int8", 17],
        ["rewrite", -1, 2, "int8", 18], ["rewrite", 3, 0, "int8", 19], ["rewrite", 26, 1, "int8", 20],
        a(3, "int4", 21), ["rewrite", 24, 3, "int8", 22], ["rewrite", 0, 29, "int8", 23],
        ["rewrite", 0, 26, "int8", 24], ["validate", 2, 4, 32], ["validate", 2, 5, 32],
        ["rewrite_bad", 0, "heads", "int8", 25], ["append_bad", "precision", "bf16", 26],
        ["append_bad", "kv_mismatch", "int8", 27], ["append", 0, "int8", 28],
    ])
    paged_case(R, "paged_mixed_pool", 2, 4, 32, 4, 16, [
        a(4, "fp16", 31), a(4, "int8", 32), a(3, "int4", 33), a(5, "fp32", 34), a(2, "fp16", 35),
        ["evict", full(4, 5, 6, 7)], a(3, "int8", 36), ["evict", full(0)],
        ["evict", [[9, 1], [9, 3]]], ["evict", full(21, 20)], a(6, "int4", 37),
        ["rewrite", 8, 3, "int4", 38], ["evict", [[8, 0], [9, 0], [9, 2], [10, 0]]],
        ["rewrite", 12, 4, "fp32", 39], ["clear"], a(5, "int4", 40),
    ])
    paged_case(R, "paged_tail_contiguous", 1, 4, 64, 8, 16, [
        a(19, "fp16", 41), ["evict", full(17, 18)], a(2, "fp16", 42), ["evict", full(19, 20)],
        ["evict", full(0, 1, 2, 3, 4, 5, 6, 7)], a(9, "int8", 43), ["evict", full(8, 9, 10)],
    ])
    paged_case(R, "paged_int4_d40_group_fallback", 2, 2, 40, 8, 16, [
        a(5, "int4", 51), a(7, "int4", 52), a(3, "int8", 53), ["rewrite", 2, 8, "int4", 54],
        ["evict", [[3, 1], [6, 0], [6, 1], [13, 0]]], a(4, "int4", 55),
    ])
    paged_case(R, "paged_int4_d33_odd", 1, 3, 33, 5, 16, [
        a(7, "int4", 61), a(4, "fp16", 62), a(6, "int4", 63), ["evict", [[1, 2], [12, 0], [12, 1], [12, 2], [14, 1]]],
        ["rewrite", 11, 1, "int4", 64], a(3, "int8", 65),
    ])
    paged_case(R, "paged_int4_d48_group24", 1, 2, 48, 6, 24, [
        a(10, "int4", 71), ["rewrite", 2, 5, "int4", 72], ["evict", [[4, 0], [7, 0], [7, 1]]], a(9, "int4", 73),
    ])
    paged_case(R, "paged_int4_d64_group4", 1, 2, 64, 16, 4, [
        a(20, "int4", 81), a(7, "int8", 82), ["rewrite", 5, 11, "int4", 83], ["evict", [[3, 1], [17, 0], [17, 1]]],
    ])
    for name, (B, H, D, P, G, n, seed) in {
        "paged_random_b2_d64": (2, 3, 64, 8, 16, 48, 7),
        "paged_random_b1_d128_g32": (1, 4, 128, 16, 32, 48, 8),
        "paged_random_b3_d32_p3": (3, 2, 32, 3, 8, 48, 9),
        "paged_random_b1_d96_p1": (1, 2, 96, 1, 16, 30, 10),
    }.items():
        paged_case(R, name, B, H, D, P, G, paged_random_ops(R, B, H, D, P, G, n, seed))


def reuse_decision_case(R, case, seed, B, H, S, D, step_id, total_steps, drift, mode):
    """ShadowKVAgent.decide_reuse_per_token (shadowkv_agent.py:1165-1256): the reuse dict as an
    array, the stats, and the drift / threshold the reference compares (replayed with the
    reference's own torch lines, to tell near-threshold entries)."""
    k, v, kp, vp, imp = (torch.from_numpy(x) for x in reuse_inputs(seed, B, H, S, D))
    mask, stats = R.Agent.decide_reuse_per_token(None, k, v, kp, vp, step_id, total_steps, drift, mode, imp)
    arr = np.zeros((S, H), dtype=np.uint8)
    for (t, h), on in mask.items():
        arr[t, h] = 1 if on else 0
    dk = torch.norm(k - kp, dim=(0, 3)) / (torch.norm(k, dim=(0, 3)) + 1e-8)
    dv = torch.norm(v - vp, dim=(0, 3)) / (torch.norm(v, dim=(0, 3)) + 1e-8)
    delta = ((dk + dv) / 2.0).t().double()
    progress = step_id / max(total_steps, 1)
    base = {"aggressive": 0.20, "balanced": 0.15, "conservative": 0.10}.get(mode, 0.15)
    eff = base * (1.0 - 0.5 * progress) * (1.0 - drift * 0.3)
    thr = torch.clamp(eff * (1.0 - 0.3 * imp.double().clamp(0.0, 1.0)), min=1e-5)
    put(case, "mask", arr)
    put(case, "ref_delta", delta)
    put(case, "ref_thr", thr)
    PINS["cases"][case] = {"kind": "reuse_decision", "seed": seed, "B": B, "H": H, "S": S, "D": D,
                           "step_id": step_id, "total_steps": total_steps, "drift": drift, "mode": mode,
                           "stats": stats}


def irap_case(R, case, seed, B, H, Sq, Sk, *, kind="probs", contract=None, prev_len=None, decay=0.9, beta=0.3,
              sink=4, layer_index=0, num_layers=1, bad=False):
    """compute_irap_importance (importance_model.py:37-134), called directly on probabilities
    (contract None) or through the agent's contract normalisation
    (_compute_importance_with_state, shadowkv_agent.py:940-965; contract 'probs' / 'logits').
    ``prev_len``: a previous EMA state of that many tokens (grown / truncated to Sk)."""
    scores = torch.from_numpy(irap_scores(seed, B, H, Sq, Sk, kind=kind, bad=bad))
    prev = None
    if prev_len is not None:
        g = np.random.default_rng(seed + 7)
        prev = torch.from_numpy((g.random((prev_len, H)) / Sk).astype(np.float32))
        put(case, "prev", prev)
    if contract is None:
        imp, ema, da = R.imp.compute_irap_importance(scores, received_ema_prev=prev, irap_decay=decay,
                                                     entropy_weight=beta, sink_tokens=sink,
                                                     layer_index=layer_index, num_layers=num_layers)
        w = torch.nan_to_num(scores, nan=0.0, posinf=0.0, neginf=0.0)
    else:
        imp, ema, da = R.Agent._compute_importance_with_state(
            R.Agent, scores, layer_index, num_layers, attn_is_probabilities=contract == "probs",
            received_ema=prev, irap_decay=decay, entropy_weight=beta, sink_tokens=sink)
        if contract == "probs":
            w = R.Agent._row_normalize(scores)
        else:
            w = torch.nn.functional.softmax(torch.nan_to_num(scores), dim=-1)
        w = torch.nan_to_num(w, nan=0.0, posinf=0.0, neginf=0.0)
    put(case, "importance", imp)
    put(case, "ema", ema)
    put(case, "ref_received", w.mean(dim=(0, 2)).t())
    PINS["cases"][case] = {"kind": "irap", "seed": seed, "B": B, "H": H, "Sq": Sq, "Sk": Sk, "score_kind": kind,
                           "contract": contract, "prev_len": prev_len, "decay": decay, "beta": beta,
                           "sink": sink, "layer_index": layer_index, "num_layers": num_layers, "bad": bad,
                           "delta_a": da}


def decision_cases(R):
    reuse_decision_case(R, "reuse_dec_b1_d128", 501, 1, 8, 256, 128, 3, 16, 0.2, "balanced")
    reuse_decision_case(R, "reuse_dec_b2_d64_aggr", 502, 2, 4, 200, 64, 0, 10, 0.0, "aggressive")
    reuse_decision_case(R, "reuse_dec_b1_d96_cons_late", 503, 1, 6, 150, 96, 9, 10, 0.9, "conservative")
    reuse_decision_case(R, "reuse_dec_b3_d32_unknown_mode", 504, 3, 3, 77, 32, 5, 0, 0.5, "custom")
    irap_case(R, "irap_probs_cold", 601, 1, 8, 128, 128)
    irap_case(R, "irap_probs_ema_grow", 602, 1, 8, 128, 128, prev_len=96, decay=0.8, layer_index=2, num_layers=4)
    irap_case(R, "irap_probs_ema_shrink", 603, 2, 4, 100, 100, prev_len=130, beta=0.0, sink=0)
    irap_case(R, "irap_nonsquare_q_lt_k", 604, 1, 4, 48, 160, beta=1.0, sink=200)
    irap_case(R, "irap_nonsquare_q_gt_k", 605, 2, 3, 90, 64, prev_len=64, layer_index=3, num_layers=3)
    irap_case(R, "irap_bad_values", 606, 1, 4, 64, 64, bad=True, prev_len=64)
    irap_case(R, "irap_contract_probs_raw", 607, 1, 8, 128, 128, kind="raw", contract="probs", prev_len=128)
    irap_case(R, "irap_contract_logits", 608, 2, 8, 128, 128, kind="logits", contract="logits", bad=True)
    irap_case(R, "irap_contract_logits_ema", 609, 1, 16, 256, 256, kind="logits", contract="logits",
              prev_len=200, decay=0.95, beta=0.5, layer_index=1, num_layers=2)


def full_pins(R):
    """cfg1 / cfg2 pipelines at full size: digests only."""
    c1 = W.CONFIGS["cfg1"]
    k, v = W.kv_tensors(c1["B"], c1["H"], c1["S"], c1["D"], c1["seed"])
    imp = W.importance_map(c1["S"], c1["H"], c1["seed"], c1["fractions"])
    codes = R.Agent.allocate_precision_codes(None, imp, "balanced")
    plan = R.plan.PrecisionPlan.from_codes(codes)
    packed = R.pkc.PackedKVCache.pack(k, v, None, group_size=16, plan=plan)["packed_kv"]
    ku, vu = packed.unpack()
    fake = types.SimpleNamespace(int4_group_size=16)
    core = R.Agent._compress_kv_with_plan(fake, k, v, None, None, plan, build_scale_map=False)
    counts = {p: len(plan.groups[p]) for p in PRECISIONS}
    PINS["full"]["cfg1"] = {
        "k": array_digest(k), "importance": array_digest(imp),
        "codes": array_digest(codes), "counts": counts, "fingerprint": plan.fingerprint,
        "packed": packed_summary(packed.packed_data, packed.memory_bytes()),
        "unpack_k": array_digest(ku), "unpack_v": array_digest(vu),
        "dense_k": array_digest(core["k"]), "dense_v": array_digest(core["v"]),
    }
    print("cfg1 done", counts, packed.memory_bytes())

    I = W.cfg2_inputs()
    k, v = I["k"], I["v"]
    sens = R.rd.kv_sensitivity(k, v)
    codes0 = R.Agent.allocate_precision_codes(None, I["importance"], "balanced")
    admitted, pred, ev = R.rd.admit_codes(
        codes0, I["importance"], sens, I["budget"], batch=1, head_dim=128,
        sink_tokens=I["sink_tokens"], rd_allocation=True, allow_eviction=True, group_size=16)
    reuse = I["reuse"]
    ts, hs = torch.nonzero(reuse, as_tuple=True)
    reuse_dict = {(t, h): True for t, h in zip(ts.tolist(), hs.tolist())}
    plan = R.plan.PrecisionPlan.from_codes(admitted, reuse_mask=reuse_dict)
    packed = R.pkc.PackedKVCache.pack(k, v, None, group_size=16, plan=plan)["packed_kv"]
    summary_pack = packed_summary(packed.packed_data, packed.memory_bytes())
    plan_prev = R.plan.PrecisionPlan.from_codes(admitted)
    prev = R.pkc.PackedKVCache.pack(I["k_prev"], I["v_prev"], None, group_size=16, plan=plan_prev)["packed_kv"]
    stats = packed.apply_reuse_mask(prev, reuse_dict, return_stats=True)
    summary_reuse = packed_summary(packed.packed_data, packed.memory_bytes())
    ku, vu = packed.unpack()
    g = torch.Generator().manual_seed(424242)
    emask = torch.rand(admitted.shape, generator=g) < 0.25
    ts, hs = torch.nonzero(emask, as_tuple=True)
    removed = packed.evict(set(zip(ts.tolist(), hs.tolist())))
    ke, ve = packed.unpack()
    PINS["full"]["cfg2"] = {
        "k": array_digest(k), "importance": array_digest(I["importance"]),
        "reuse": array_digest(reuse), "k_prev": array_digest(I["k_prev"]),
        "budget": I["budget"], "sensitivity": array_digest(sens),
        "codes0": array_digest(codes0), "admitted": array_digest(admitted),
        "predicted": pred, "evicted": ev, "fingerprint": plan.fingerprint,
        "counts": {p: len(plan.groups[p]) for p in PRECISIONS},
        "packed": summary_pack, "reuse_stats": stats, "after_reuse": summary_reuse,
        "unpack_k": array_digest(ku), "unpack_v": array_digest(vu),
        "evict_seed": 424242, "evict_frac": 0.25, "removed": removed,
        "after_evict": packed_summary(packed.packed_data, packed.memory_bytes()),
        "resident_after_evict": packed.resident_bytes(),
        "unpack_evict_k": array_digest(ke), "unpack_evict_v": array_digest(ve),
    }
    print("cfg2 done", pred, ev, stats, removed)


def _sampled_attention(q, ku, vu, rows):
    """The reference model's attention lines (simple_diffusion_llm.py:165-169, fp32) on the query
    rows ``rows`` only: non-causal attention is row-independent, so these are exactly those rows
    of the full output."""
    qf = q[:, :, rows].float()
    scores = torch.matmul(qf, ku.transpose(-2, -1)) / (qf.shape[-1] ** 0.5)
    return torch.matmul(torch.softmax(scores, dim=-1), vu)


def long_pins(R):
    """Head slices of the long-context layer (cfg5: S=32768, codes 10/30/60, channel outliers) and
    of the batched denoising layer (cfg4: B=8, one drift step with reuse and eviction): digests
    of the reference's plan / pack / reuse / evict / unpack, and its attention on sampled rows."""
    c5 = W.CONFIGS["cfg5"]
    h0, h1 = 0, 2
    L = W.cfg5_layer(h0, h1)
    imp = L["importance"][:, h0:h1].contiguous()
    codes = R.Agent.allocate_precision_codes(None, imp, "balanced")
    plan = R.plan.PrecisionPlan.from_codes(codes)
    packed = R.pkc.PackedKVCache.pack(L["k"], L["v"], None, group_size=c5["group"], plan=plan)["packed_kv"]
    ku, vu = packed.unpack()
    rows = W.sample_rows(c5["S"], 64, 5)
    out = _sampled_attention(L["q"], ku, vu, rows)
    put("cfg5_slice", "rows", rows)
    put("cfg5_slice", "out", out)
    PINS["full"]["cfg5_slice"] = {
        "heads": [h0, h1], "k": array_digest(L["k"]), "v": array_digest(L["v"]), "q": array_digest(L["q"]),
        "importance": array_digest(L["importance"]), "codes": array_digest(codes),
        "counts": {p: len(plan.groups[p]) for p in PRECISIONS}, "fingerprint": plan.fingerprint,
        "packed": packed_summary(packed.packed_data, packed.memory_bytes()),
        "data_plane_bytes": packed.data_plane_bytes(), "resident_bytes": packed.resident_bytes(),
        "unpack_k": array_digest(ku), "unpack_v": array_digest(vu),
    }
    print("cfg5 slice done", PINS["full"]["cfg5_slice"]["counts"], packed.memory_bytes())

    c4 = W.CONFIGS["cfg4"]
    B, S, D = c4["B"], c4["S"], c4["D"]
    h0, h1 = 0, 4
    L = W.cfg4_layer(h0, h1)
    imp = L["importance"][:, h0:h1].contiguous()
    codes = R.Agent.allocate_precision_codes(None, imp, "balanced")
    prev = R.pkc.PackedKVCache.pack(L["k"], L["v"], None, group_size=16,
                                    plan=R.plan.PrecisionPlan.from_codes(codes))["packed_kv"]
    nk, nv = W.drift_noise(B, S, D, 10_000, 1, h0, h1)
    k1, v1 = W.apply_drift(L["k"], nk), W.apply_drift(L["v"], nv)
    # drift < 0.05: the conservative threshold at the last step, importance term off
    reuse_dict, rstats = R.Agent.decide_reuse_per_token(None, k1, v1, L["k"], L["v"], 16, 16, 0.0, "conservative",
                                                        torch.zeros(S, h1 - h0))
    reuse = torch.zeros(S, h1 - h0, dtype=torch.bool)
    for (t, h), f in reuse_dict.items():
        reuse[t, h] = f
    plan = R.plan.PrecisionPlan.from_codes(codes, reuse_mask=reuse_dict)
    cur = R.pkc.PackedKVCache.pack(k1, v1, None, group_size=16, plan=plan)["packed_kv"]
    summary_pack = packed_summary(cur.packed_data, cur.memory_bytes())
    stats = cur.apply_reuse_mask(prev, reuse_dict, return_stats=True)
    summary_reuse = packed_summary(cur.packed_data, cur.memory_bytes())
    emask = W.lowest_importance_mask(imp, c4["evict_frac"], 4)
    ts, hs = torch.nonzero(emask, as_tuple=True)
    removed = cur.evict(set(zip(ts.tolist(), hs.tolist())))
    ku, vu = cur.unpack()
    rows = W.sample_rows(S, 16, 4)
    out = _sampled_attention(L["q"], ku, vu, rows)
    put("cfg4_slice", "rows", rows)
    put("cfg4_slice", "out", out)
    put("cfg4_slice", "reuse", reuse)
    PINS["full"]["cfg4_slice"] = {
        "heads": [h0, h1], "k1": array_digest(k1), "v1": array_digest(v1), "q": array_digest(L["q"]),
        "codes": array_digest(codes), "reuse": array_digest(reuse), "reuse_decision": rstats,
        "fingerprint": plan.fingerprint, "packed": summary_pack, "reuse_stats": stats,
        "after_reuse": summary_reuse, "evict_mask": array_digest(emask), "removed": removed,
        "after_evict": packed_summary(cur.packed_data, cur.memory_bytes()),
        "resident_after_evict": cur.resident_bytes(),
        "unpack_k": array_digest(ku), "unpack_v": array_digest(vu),
    }
    print("cfg4 slice done", rstats, stats, removed)


def block_case(R, case, gen, B, H, D, S_past, S_new, inter, probs=(0.1, 0.3, 0.3, 0.25, 0.05), seed=77):
    """One reference DiffusionTransformerBlock._compute_block forward over a past KV cache that
    comes from the reference PackedKVCache (pack -> unpack, the kv_execution="packed" backend's
    path, pytorch_backend.py:302-304): this block's hidden output, its own K/V and the attention
    output (attention weights times the concatenated V)."""
    hidden_dim = H * D
    block = R.sdl.DiffusionTransformerBlock(hidden_dim, H, D, inter, torch.device("cpu"), torch.float32)
    params = block_params(seed, hidden_dim, inter)
    with torch.no_grad():
        named = dict(block.named_parameters())
        assert set(named) == set(BLOCK_PARAM_ORDER)
        for name in BLOCK_PARAM_ORDER:
            named[name].copy_(params[name])
    k, v = kv(gen, B, H, S_past, D)
    codes = codes_of(gen, S_past, H, probs)
    packed = R.pkc.PackedKVCache.pack(k, v, R.plan.codes_to_map(codes), group_size=16)["packed_kv"]
    past = packed.unpack()
    hidden = torch.randn(B, S_new, hidden_dim, generator=gen)
    with torch.no_grad():
        out, k_new, v_new, k_full, v_full, attn_w = block._compute_block(hidden, past)
        attn_out = torch.matmul(attn_w, v_full)
        q = block.q_proj(block.ln1(hidden)).view(B, S_new, H, D).transpose(1, 2)
    for name, x in (("k", k), ("v", v), ("codes", codes), ("hidden", hidden), ("out", out), ("k_new", k_new),
                    ("v_new", v_new), ("attn_out", attn_out), ("q", q)):
        put(case, name, x)
    PINS["cases"][case] = {"kind": "block", "B": B, "H": H, "D": D, "S_past": S_past, "S_new": S_new,
                           "inter": inter, "seed": seed,
                           "params": {n: array_digest(params[n]) for n in BLOCK_PARAM_ORDER}}


def block_cases(R):
    g3 = torch.Generator().manual_seed(20261203)
    block_case(R, "block_b2_h2_d64", g3, 2, 2, 64, 200, 80, 256)
    block_case(R, "block_b1_h2_d128", g3, 1, 2, 128, 300, 130, 512, seed=78)


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--reference", required=True, help="path of the shadow-infer source tree")
    ap.add_argument("--only-long", action="store_true",
                    help="keep the existing fixtures and (re)record only the cfg5 / cfg4 head-slice pins")
    ap.add_argument("--only-block", action="store_true",
                    help="keep the existing fixtures and (re)record only the model-block forward cases")
    args = ap.parse_args()
    torch.set_num_threads(os.cpu_count() or 1)
    R = _import_reference(args.reference)
    if args.only_long or args.only_block:
        with np.load(SMALL_NPZ, allow_pickle=False) as z:
            drop = (("cfg5_slice/", "cfg4_slice/") if args.only_long else ()) + (("block_",) if args.only_block else ())
            ARR.update({k: z[k] for k in z.files if not k.startswith(drop)})
        with open(PINS_JSON) as f:
            PINS.update(json.load(f))
        if args.only_long:
            long_pins(R)
        if args.only_block:
            block_cases(R)
        np.savez_compressed(SMALL_NPZ, **ARR)
        with open(PINS_JSON, "w") as f:
            json.dump(PINS, f, indent=1, sort_keys=True)
        print("wrote", SMALL_NPZ, os.path.getsize(SMALL_NPZ), PINS_JSON)
        return
    gen = torch.Generator().manual_seed(20261201)
    mixed = (0.15, 0.3, 0.25, 0.2, 0.1)
    pack_case(R, "pack_b1_d64", gen, 1, 4, 16, 64, mixed)
    pack_case(R, "pack_b2_d64", gen, 2, 3, 10, 64, mixed)
    pack_case(R, "pack_b1_d63_odd", gen, 1, 2, 7, 63, mixed)
    pack_case(R, "pack_b3_d40", gen, 3, 2, 9, 40, mixed)
    pack_case(R, "pack_b1_d128_g32_int4", gen, 1, 2, 8, 128, (0, 0, 0, 1.0, 0), group=32)
    pack_case(R, "pack_b2_d128_zero_rows", gen, 2, 3, 11, 128, mixed, zero_rows=6)
    pack_case(R, "pack_b1_d128_fp16_overflow", gen, 1, 2, 5, 128, (0.0, 1.0, 0, 0, 0), big=True)
    pack_case(R, "pack_b1_d256", gen, 1, 2, 12, 256, mixed)
    pack_case(R, "pack_b1_d32", gen, 1, 3, 11, 32, mixed)
    pack_case(R, "pack_b1_all_evicted_but_one", gen, 1, 2, 6, 64, (0, 0, 0, 0, 1.0))
    pack_case(R, "pack_b4_d128", gen, 4, 2, 9, 128, mixed)
    reuse_case(R, "reuse_b1_d64", gen, 1, 4, 24, 64)
    reuse_case(R, "reuse_b2_d128", gen, 2, 3, 12, 128)
    reuse_case(R, "reuse_b1_d63", gen, 1, 2, 9, 63)
    evict_case(R, "evict_b1_d64", gen, 1, 4, 24, 64)
    evict_case(R, "evict_b2_d128", gen, 2, 3, 16, 128)
    admit_case(R, "admit_basic", gen, 64, 8, 1, 128, 0.6)
    admit_case(R, "admit_evict_tiny", gen, 64, 8, 1, 128, 0.05, evict=True)
    admit_case(R, "admit_ties", gen, 48, 6, 1, 64, 0.5, ties=True, evict=True)
    admit_case(R, "admit_sink_protected", gen, 40, 4, 2, 64, 0.3, sink=3, protected_p=0.2, evict=True)
    admit_case(R, "admit_budget_none", gen, 16, 4, 1, 64, 0.5, budget_abs=-1)
    admit_case(R, "admit_budget_loose", gen, 16, 4, 1, 64, 2.0)
    admit_case(R, "admit_no_rd", gen, 64, 8, 1, 128, 0.55, rd=False)
    admit_case(R, "admit_signed_zero", gen, 64, 8, 1, 128, 0.5, signed_zero=True, evict=True)
    admit_case(R, "admit_nan", gen, 32, 4, 1, 64, 0.4, nan=True, evict=True)
    admit_case(R, "admit_sens_mismatch", gen, 32, 4, 1, 64, 0.45)
    admit_case(R, "admit_b2_g16", gen, 96, 8, 2, 64, 0.35, sink=4, evict=True)
    admit_case(R, "admit_boundary_mid", gen, 256, 8, 1, 128, 0.93)
    admit_case(R, "admit_all_sinks", gen, 8, 4, 1, 64, 0.1, sink=16, evict=True)
    allocate_case(R, "allocate")
    sensitivity_case(R, "sensitivity", gen)
    attention_case(R, "attention_b1", gen, 1, 2, 64, 64)
    attention_case(R, "attention_b2_d128", gen, 2, 1, 80, 128)
    global_budget_case(R, "gb_two_fp32_dense", gen, 1, 2, 16, 64, 2, 0.0, 2, probs=(1.0, 0, 0, 0, 0),
                       dense=(0, 1), budget_abs=20000)
    global_budget_case(R, "gb_mixed_ties", gen, 2, 3, 24, 64, 3, 0.55, 3, ties=True, packed_only=(2,))
    global_budget_case(R, "gb_noncandidate_layer", gen, 1, 4, 20, 128, 3, 0.6, 2, no_importance=(1,), dense=(0,))
    global_budget_case(R, "gb_floor", gen, 1, 2, 12, 64, 2, 0.02, 2)
    global_budget_case(R, "gb_no_pressure", gen, 1, 2, 12, 64, 2, 2.0, 0)
    global_budget_case(R, "gb_b2_group32", gen, 2, 2, 40, 128, 2, 0.4, 4, group=32, probs=(0.1, 0.3, 0.3, 0.25, 0.05))
    paged_cases(R)
    decision_cases(R)
    g2 = torch.Generator().manual_seed(20261202)
    attention_gqa_case(R, "attn_gqa_rep4_d64", g2, 1, 2, 4, 100, 40, 40, 64)
    attention_gqa_case(R, "attn_gqa_rep2_d128_b2", g2, 2, 2, 2, 96, 40, 40, 128)
    attention_gqa_case(R, "attn_new_rows_rep1", g2, 1, 3, 1, 70, 33, 50, 64)
    attention_gqa_case(R, "attn_gqa_past_all_evicted", g2, 1, 2, 2, 20, 17, 30, 64, probs=(0, 0, 0, 0, 1.0))
    full_pins(R)
    long_pins(R)
    block_cases(R)
    np.savez_compressed(SMALL_NPZ, **ARR)
    with open(PINS_JSON, "w") as f:
        json.dump(PINS, f, indent=1, sort_keys=True)
    print("wrote", SMALL_NPZ, os.path.getsize(SMALL_NPZ), PINS_JSON)


if __name__ == "__main__":
    main()
