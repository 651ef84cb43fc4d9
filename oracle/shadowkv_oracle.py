"""CPU oracle for the ShadowKV packed-KV data plane -- TEST INFRASTRUCTURE ONLY.

This module restates, in numpy, the reference algorithms of ShadowInfer's
ShadowKV data plane (reference project ``ShaneLiu04/shadow-infer``, package
``shadowinfer``).  It exists to *check* the CUDA product path and is imported
only by ``tests/``, ``__graft_entry__.smoke()`` and ``bench.py``'s
``cpu_baseline`` / ``--impl reference`` legs.  The product package
``shadow_infer_b200`` never imports it and has no CPU fallback.

Parity is pinned: ``tests/golden/make_golden.py`` runs the reference itself
(imported from its source tree) on seeded inputs and records its outputs (small
arrays plus SHA-256 digests of full-size outputs) under ``tests/golden/``;
``tests/test_oracle_golden.py`` checks every function here against them.

Arithmetic notes (all verified against the reference's torch CPU build):
  * ``x / 127.0`` and ``x / scale`` are IEEE-754 fp32 true divisions (torch CPU
    does not use a reciprocal multiply); numpy float32 division matches.
  * ``torch.round`` is round-half-to-even == ``np.rint``.
  * fp32 -> fp16 casts round to nearest even (``astype(np.float16)``).
  * ``argsort(stable=True)`` == ``np.argsort(kind="stable")`` (NaN last,
    -0.0 == +0.0 with index order kept).
"""

from __future__ import annotations

import hashlib
import struct
from typing import Any, Dict, List, Optional, Sequence, Tuple

import numpy as np

PRECISION_ORDER: Tuple[str, ...] = ("fp32", "fp16", "int8", "int4")
EVICTED = "evicted"
PRECISION_CODES: Dict[str, int] = {"fp32": 0, "fp16": 1, "int8": 2, "int4": 3, EVICTED: 4}
CODE_PRECISIONS: Dict[int, str] = {c: p for p, c in PRECISION_CODES.items()}


# --------------------------------------------------------------------------------------
# cost model  (shadowinfer/shadowkv/rd_allocator.py:26-44, :170-187)
# --------------------------------------------------------------------------------------
def entry_bytes(precision: str, batch: int, head_dim: int, group_size: int = 16) -> float:
    """Stored K+V bytes of one token-head, incl. scales (rd_allocator.py:26-44)."""
    p = precision.lower() if isinstance(precision, str) else precision
    if p == EVICTED:
        return 0.0
    if p == "int4":
        group = group_size if group_size > 0 and head_dim % group_size == 0 else head_dim
        per_tensor = batch * head_dim / 2.0 + batch * (head_dim // group) * 4
    elif p == "int8":
        per_tensor = batch * head_dim + batch * 4
    elif p == "fp32":
        per_tensor = batch * head_dim * 4
    else:
        per_tensor = batch * head_dim * 2
    return per_tensor * 2.0


def code_costs(batch: int, head_dim: int, group_size: int = 16) -> np.ndarray:
    """int64 cost per code 0..4, truncated with ``int()`` (rd_allocator.py:179-186)."""
    return np.array(
        [int(entry_bytes(CODE_PRECISIONS[c], batch, head_dim, group_size)) for c in range(5)],
        dtype=np.int64,
    )


def predict_codes_bytes(codes: np.ndarray, batch: int, head_dim: int, group_size: int = 16) -> int:
    """Sum of per-entry costs (rd_allocator.py:170-187)."""
    costs = code_costs(batch, head_dim, group_size)
    return int(costs[np.asarray(codes).astype(np.int64)].sum())


# --------------------------------------------------------------------------------------
# precision coding  (shadowinfer/shadowkv/shadowkv_agent.py:1028-1059)
# --------------------------------------------------------------------------------------
def allocate_precision_codes(importance: np.ndarray, mode: str) -> np.ndarray:
    """Threshold bands compared in float64 (shadowkv_agent.py:1028-1059)."""
    adj = {"aggressive": -0.1, "balanced": 0.0, "conservative": 0.1}.get(mode, 0.0)
    t_fp32 = max(0.0, 0.8 + adj)
    t_fp16 = max(0.0, 0.5 + adj)
    t_int8 = max(0.0, 0.2 + adj)
    s = np.asarray(importance).astype(np.float64)
    out = np.where(s >= t_fp32, 0, np.where(s >= t_fp16, 1, np.where(s >= t_int8, 2, 3)))
    return out.astype(np.int8)


def kv_sensitivity(k: np.ndarray, v: np.ndarray) -> np.ndarray:
    """``(amax|k|^2 + amax|v|^2)/2`` over batch and head_dim, as [S,H] (rd_allocator.py:47-61)."""
    if k.shape != v.shape:
        raise ValueError("k and v must have identical shapes")
    ka = np.abs(k).max(axis=(0, 3)).astype(np.float32)  # [H, S]
    va = np.abs(v).max(axis=(0, 3)).astype(np.float32)
    sens = (ka * ka + va * va) / np.float32(2.0)
    return np.ascontiguousarray(sens.T.astype(np.float32))


# --------------------------------------------------------------------------------------
# budget admission  (shadowinfer/shadowkv/rd_allocator.py:190-318)
# --------------------------------------------------------------------------------------
def admit_codes(
    codes: np.ndarray,
    importance: np.ndarray,
    sensitivity: np.ndarray,
    budget_bytes: Optional[int],
    batch: int,
    head_dim: int,
    sink_tokens: int = 0,
    rd_allocation: bool = True,
    allow_eviction: bool = False,
    protected_mask: Optional[np.ndarray] = None,
    group_size: int = 16,
) -> Tuple[np.ndarray, int, int]:
    """Closed-form greedy downgrade ladder + optional hard eviction (rd_allocator.py:190-318)."""
    codes = np.asarray(codes)
    if codes.ndim != 2:
        raise ValueError(f"codes must be 2-D [seq, heads], got shape {tuple(codes.shape)}")
    out = codes.astype(np.int8).copy()
    seq_len, num_heads = out.shape
    flat = out.reshape(-1)
    costs = code_costs(batch, head_dim, group_size)
    predicted = int(costs[flat.astype(np.int64)].sum())
    if budget_bytes is None or budget_bytes < 0:
        return out, predicted, 0

    imp = np.asarray(importance, dtype=np.float32)[:seq_len, :num_heads]
    sens = np.asarray(sensitivity, dtype=np.float32)[:seq_len, :num_heads]
    if sens.shape != imp.shape:
        sens = np.ones_like(imp)
    score = (imp * sens) if rd_allocation else imp

    eligible = np.ones((seq_len, num_heads), dtype=bool)
    if sink_tokens > 0:
        eligible[: min(int(sink_tokens), seq_len)] = False
    if protected_mask is not None:
        eligible &= ~np.asarray(protected_mask).astype(bool)[:seq_len, :num_heads]

    order = np.argsort(score.reshape(-1), kind="stable")
    candidates = order[eligible.reshape(-1)[order]]
    n = candidates.size
    if n == 0:
        return out, predicted, 0

    deltas = np.array([costs[c] - costs[c + 1] for c in (0, 1, 2)], dtype=np.int64)

    def _apply_downgrades(cur: np.ndarray, excess: int) -> Tuple[np.ndarray, int]:
        base = cur[candidates].astype(np.int64)
        step1 = np.where(base < 3, deltas[np.minimum(base, 2)], 0)
        next1 = np.where(base < 3, base + 1, base)
        step2 = np.where(next1 < 3, deltas[np.minimum(next1, 2)], 0)
        next2 = np.where(next1 < 3, next1 + 1, next1)
        step3 = np.where(next2 < 3, deltas[np.minimum(next2, 2)], 0)
        cumulative = np.cumsum(step1 + step2 + step3)
        boundary = int(np.searchsorted(cumulative, excess, side="left"))
        if boundary >= n:
            boundary = n
        new = base.copy()
        if boundary > 0:
            new[:boundary] = np.where(base[:boundary] != 4, 3, base[:boundary])
        if boundary < n:
            consumed = int(cumulative[boundary - 1]) if boundary > 0 else 0
            remaining = excess - consumed
            if int(base[boundary]) != 4:
                if remaining <= int(step1[boundary]):
                    new[boundary] = next1[boundary]
                elif remaining <= int(step1[boundary]) + int(step2[boundary]):
                    new[boundary] = next2[boundary]
                else:
                    new[boundary] = 3
        cur[candidates] = new.astype(np.int8)
        return cur, int(costs[cur.astype(np.int64)].sum())

    if predicted > budget_bytes:
        flat, predicted = _apply_downgrades(flat, predicted - budget_bytes)

    evicted = 0
    if allow_eviction and predicted > budget_bytes:
        excess = predicted - budget_bytes
        cumulative = np.cumsum(costs[flat[candidates].astype(np.int64)])
        boundary = int(np.searchsorted(cumulative, excess, side="left"))
        if boundary >= n:
            boundary = n - 1
        target = candidates[: boundary + 1]
        evicted = int((flat[target] != 4).sum())
        flat[target] = 4
        predicted = int(costs[flat.astype(np.int64)].sum())
    return flat.reshape(out.shape), int(predicted), evicted


# --------------------------------------------------------------------------------------
# plan  (shadowinfer/shadowkv/precision_plan.py:113-190)
# --------------------------------------------------------------------------------------
def reuse_mask_to_array(reuse_mask: Any, seq_len: int, num_heads: int) -> np.ndarray:
    """Dict ``(t,h)->bool`` or array -> bool [S,H]; out-of-range keys dropped (precision_plan.py:153-159)."""
    out = np.zeros((seq_len, num_heads), dtype=bool)
    if reuse_mask is None:
        return out
    if isinstance(reuse_mask, dict):
        for (t, h), flag in reuse_mask.items():
            if flag and 0 <= t < seq_len and 0 <= h < num_heads:
                out[int(t), int(h)] = True
        return out
    arr = np.asarray(reuse_mask).astype(bool)
    return arr[:seq_len, :num_heads].copy()


def plan_from_codes(codes: np.ndarray, reuse_mask: Any = None) -> Dict[str, Any]:
    """Per-code token-major buckets, flat ``h*S+t`` indices, reuse list, SHA-256 (precision_plan.py:113-190)."""
    codes = np.asarray(codes)
    if codes.ndim != 2:
        raise ValueError(f"codes must be 2-D [seq, heads], got shape {tuple(codes.shape)}")
    seq_len, num_heads = int(codes.shape[0]), int(codes.shape[1])
    if seq_len <= 0 or num_heads <= 0:
        raise ValueError(f"seq_len and num_heads must be positive, got {seq_len}, {num_heads}")
    c8 = np.ascontiguousarray(codes.astype(np.int8))
    flat = c8.reshape(-1).astype(np.int64)
    flat_indices: Dict[str, np.ndarray] = {}
    groups: Dict[str, List[Tuple[int, int]]] = {p: [] for p in PRECISION_ORDER}
    evicted: List[Tuple[int, int]] = []
    evicted_flat = np.zeros(0, dtype=np.int64)
    for code, precision in CODE_PRECISIONS.items():
        sel = np.nonzero(flat == code)[0]
        t = sel // num_heads
        h = sel % num_heads
        if sel.size == 0:
            if precision != EVICTED:
                flat_indices[precision] = np.zeros(0, dtype=np.int64)
            continue
        entries = list(zip(t.tolist(), h.tolist()))
        if precision == EVICTED:
            evicted = entries
            evicted_flat = (h * seq_len + t).astype(np.int64)
        else:
            groups[precision] = entries
            flat_indices[precision] = (h * seq_len + t).astype(np.int64)
    rmask = reuse_mask_to_array(reuse_mask, seq_len, num_heads) if reuse_mask is not None else None
    if rmask is not None and rmask.any():
        rt, rh = np.nonzero(rmask)  # row-major == sorted (t, h)
        reuse_entries = list(zip(rt.tolist(), rh.tolist()))
        reuse_flat = (rh * seq_len + rt).astype(np.int64)
    else:
        reuse_entries = []
        reuse_flat = np.zeros(0, dtype=np.int64)
    digest = hashlib.sha256()
    digest.update(struct.pack("<QQ", seq_len, num_heads))
    digest.update(c8.tobytes())
    digest.update(reuse_flat.astype("<i8").tobytes())
    return {
        "seq_len": seq_len,
        "num_heads": num_heads,
        "codes": c8,
        "groups": groups,
        "flat_indices": flat_indices,
        "evicted_entries": evicted,
        "evicted_flat": evicted_flat,
        "reuse_entries": reuse_entries,
        "reuse_flat": reuse_flat,
        "fingerprint": digest.hexdigest(),
    }


# --------------------------------------------------------------------------------------
# quantisers  (shadowinfer/utils/quantization.py:121-219)
# --------------------------------------------------------------------------------------
def quantize_int8(x: np.ndarray) -> Tuple[np.ndarray, np.ndarray]:
    """Row absmax/127, 0 -> 1, RNE, clamp [-128,127] (quantization.py:121-142)."""
    scale = np.abs(x).max(axis=-1, keepdims=True).astype(np.float32) / np.float32(127.0)
    scale = np.where(scale == 0, np.float32(1.0), scale).astype(np.float32)
    q = np.clip(np.rint(x / scale), -128, 127).astype(np.int8)
    return q, scale


def quantize_int4(x: np.ndarray, group_size: int) -> Tuple[np.ndarray, np.ndarray]:
    """Group absmax/7, 0 -> 1, RNE, clamp [-8,7]; q [...,G,g], scale [...,G,1] (quantization.py:145-178)."""
    last = x.shape[-1]
    if last % group_size != 0:
        raise ValueError(f"last dim {last} not divisible by group_size {group_size}")
    g = last // group_size
    xr = x.reshape(*x.shape[:-1], g, group_size)
    scale = np.abs(xr).max(axis=-1, keepdims=True).astype(np.float32) / np.float32(7.0)
    scale = np.where(scale == 0, np.float32(1.0), scale).astype(np.float32)
    q = np.clip(np.rint(xr / scale), -8, 7).astype(np.int8)
    return q, scale


def pack_int4_rows(q: np.ndarray) -> Tuple[np.ndarray, int]:
    """Row-wise nibble pack: ``(v+8)`` high nibble first, odd rows padded (packed_kv_cache.py:367-388)."""
    if q.shape[0] == 0:
        return np.zeros((0, 0), dtype=np.uint8), 0
    rows = q.reshape(q.shape[0], -1)
    off = (rows.astype(np.int16) + 8).astype(np.uint8)
    if off.shape[1] % 2:
        off = np.concatenate([off, np.zeros((off.shape[0], 1), dtype=np.uint8)], axis=1)
    packed = ((off[:, 0::2] << 4) & 0xF0) | (off[:, 1::2] & 0x0F)
    return packed.astype(np.uint8), packed.shape[1]


def int4_group(head_dim: int, group_size: int) -> int:
    """Effective int4 group: ``group_size`` when it divides head_dim, else head_dim (packed_kv_cache.py:307)."""
    return group_size if head_dim % group_size == 0 else head_dim


# --------------------------------------------------------------------------------------
# packed cache  (shadowinfer/shadowkv/packed_kv_cache.py)
# --------------------------------------------------------------------------------------
class OraclePackedKV:
    """numpy mirror of ``PackedKVCache`` state: ``packed_data`` with numpy arrays."""

    def __init__(self, batch: int, heads: int, seq: int, dim: int):
        self.batch_size, self.num_heads, self.seq_len, self.head_dim = batch, heads, seq, dim
        self.packed_data: Dict[str, Dict[str, Any]] = {}
        self._memory_bytes = 0

    def compute_data_bytes(self) -> int:
        """packed_kv_cache.py:856-863."""
        total = 0
        for data in self.packed_data.values():
            for key in ("k", "v", "scale_k", "scale_v"):
                arr = data.get(key)
                if arr is not None:
                    total += arr.size * arr.itemsize
        return total

    def memory_bytes(self) -> int:
        return self._memory_bytes

    def data_plane_bytes(self) -> int:
        return self.compute_data_bytes()

    def resident_bytes(self) -> int:
        """data + 48 B per entry (packed_kv_cache.py:869-878)."""
        if not self.packed_data:
            return 0
        n = sum(len(d["indices"]) for d in self.packed_data.values())
        return self.compute_data_bytes() + 48 * n


def pack(k: np.ndarray, v: np.ndarray, plan: Dict[str, Any], group_size: int = 16) -> OraclePackedKV:
    """Plan-driven gather + quantise + pack (packed_kv_cache.py:222-365)."""
    B, H, S, D = k.shape
    if plan["seq_len"] != S or plan["num_heads"] != H:
        raise ValueError(
            "PrecisionPlan shape mismatch: plan "
            f"(seq_len={plan['seq_len']}, num_heads={plan['num_heads']}) vs "
            f"tensor (seq_len={S}, num_heads={H})"
        )
    if v.shape != k.shape:
        raise ValueError("k_tensor and v_tensor must have identical shapes")
    cache = OraclePackedKV(B, H, S, D)
    kf = np.ascontiguousarray(k, dtype=np.float32).reshape(B, H * S, D)
    vf = np.ascontiguousarray(v, dtype=np.float32).reshape(B, H * S, D)
    total = 0
    for precision in PRECISION_ORDER:
        entries = plan["groups"][precision]
        if not entries:
            continue
        flat = plan["flat_indices"][precision]
        kg = kf[:, flat, :].transpose(1, 0, 2)
        vg = vf[:, flat, :].transpose(1, 0, 2)
        if precision in ("fp32", "fp16"):
            dt = np.float32 if precision == "fp32" else np.float16
            d = {"k": np.ascontiguousarray(kg.astype(dt)), "v": np.ascontiguousarray(vg.astype(dt)),
                 "scale_k": None, "scale_v": None}
        elif precision == "int8":
            qk, sk = quantize_int8(kg)
            qv, sv = quantize_int8(vg)
            d = {"k": qk, "v": qv, "scale_k": sk, "scale_v": sv}
        else:
            g = int4_group(D, group_size)
            ng = D // g
            qk, sk = quantize_int4(kg, g)
            qv, sv = quantize_int4(vg, g)
            krows, rb = pack_int4_rows(qk)
            vrows, _ = pack_int4_rows(qv)
            d = {
                "k": krows.reshape(-1), "v": vrows.reshape(-1),
                "scale_k": sk.reshape(-1, ng, 1), "scale_v": sv.reshape(-1, ng, 1),
                "byte_offsets": [(n * rb, (n + 1) * rb, n * rb, (n + 1) * rb) for n in range(len(entries))],
                "group_size": g, "num_groups": ng,
            }
        d["indices"] = list(entries)
        d["flat"] = flat.copy()
        for key in ("k", "v", "scale_k", "scale_v"):
            if d[key] is not None:
                total += d[key].size * d[key].itemsize
        cache.packed_data[precision] = d
    cache._memory_bytes = total
    return cache


def dequantize_bucket(cache: OraclePackedKV, precision: str, which: str) -> np.ndarray:
    """One bucket -> float32 [N,B,D] (packed_kv_cache.py:555-575, :636-656)."""
    d = cache.packed_data[precision]
    B, D = cache.batch_size, cache.head_dim
    n = len(d["indices"])
    if precision in ("fp32", "fp16"):
        return d[which].astype(np.float32)
    scale = d["scale_" + which]
    if precision == "int8":
        return d[which].astype(np.float32) * scale
    rows = d[which].reshape(n, -1)
    inter = np.stack([(rows >> 4) & 0x0F, rows & 0x0F], axis=-1).reshape(n, -1)
    codes = (inter[:, : B * D].astype(np.int16) - 8).astype(np.int8)
    g, ng = d["group_size"], d["num_groups"]
    vals = codes.reshape(n, B, ng, g).astype(np.float32) * scale.reshape(n, B, ng, 1)
    return vals.reshape(n, B, D)


def unpack(cache: OraclePackedKV) -> Tuple[np.ndarray, np.ndarray]:
    """Zero-filled fp32 [B,H,S,D] K and V; buckets scattered back (packed_kv_cache.py:535-577)."""
    B, H, S, D = cache.batch_size, cache.num_heads, cache.seq_len, cache.head_dim
    ko = np.zeros((B, H, S, D), dtype=np.float32)
    vo = np.zeros_like(ko)
    for precision, d in cache.packed_data.items():
        if not d["indices"]:
            continue
        t = np.array([e[0] for e in d["indices"]], dtype=np.int64)
        h = np.array([e[1] for e in d["indices"]], dtype=np.int64)
        ko[:, h, t, :] = dequantize_bucket(cache, precision, "k").transpose(1, 0, 2)
        vo[:, h, t, :] = dequantize_bucket(cache, precision, "v").transpose(1, 0, 2)
    return ko, vo


def evict(cache: OraclePackedKV, entries: Any) -> int:
    """Stable in-bucket removal; empty buckets deleted (packed_kv_cache.py:666-740).

    ``entries``: a set of (t,h) or a bool [S,H] mask.
    """
    if isinstance(entries, np.ndarray):
        ts, hs = np.nonzero(entries)
        entries = set(zip(ts.tolist(), hs.tolist()))
    if not entries or not cache.packed_data:
        return 0
    B = cache.batch_size
    removed = 0
    for precision in list(cache.packed_data.keys()):
        d = cache.packed_data[precision]
        idx = d["indices"]
        keep_pos = [i for i, e in enumerate(idx) if e not in entries]
        removed += len(idx) - len(keep_pos)
        if len(keep_pos) == len(idx):
            continue
        if not keep_pos:
            del cache.packed_data[precision]
            continue
        keep = np.array(keep_pos, dtype=np.int64)
        if precision in ("fp32", "fp16", "int8"):
            d["k"], d["v"] = d["k"][keep], d["v"][keep]
            if precision == "int8":
                d["scale_k"], d["scale_v"] = d["scale_k"][keep], d["scale_v"][keep]
        else:
            n = len(idx)
            rb = d["k"].size // n
            ng = d["num_groups"]
            d["k"] = d["k"].reshape(n, rb)[keep].reshape(-1)
            d["v"] = d["v"].reshape(n, rb)[keep].reshape(-1)
            d["scale_k"] = d["scale_k"].reshape(n, B, ng, 1)[keep].reshape(-1, ng, 1)
            d["scale_v"] = d["scale_v"].reshape(n, B, ng, 1)[keep].reshape(-1, ng, 1)
            d["byte_offsets"] = [(i * rb, (i + 1) * rb, i * rb, (i + 1) * rb) for i in range(len(keep_pos))]
        d["indices"] = [idx[i] for i in keep_pos]
        if "flat" in d:
            d["flat"] = d["flat"][keep]
    cache._memory_bytes = cache.compute_data_bytes()
    return removed


def apply_reuse_mask(cache: OraclePackedKV, prev: OraclePackedKV, reuse_mask: Any) -> Dict[str, int]:
    """Same-precision row copy from ``prev``; cross-precision counted (packed_kv_cache.py:753-854)."""
    if (cache.batch_size, cache.num_heads, cache.head_dim) != (prev.batch_size, prev.num_heads, prev.head_dim):
        raise ValueError(
            "packed cache shape mismatch for reuse: "
            f"current=({cache.batch_size},{cache.num_heads},{cache.head_dim}) "
            f"previous=({prev.batch_size},{prev.num_heads},{prev.head_dim})"
        )
    if "int4" in cache.packed_data:
        cur, pv = cache.packed_data["int4"], prev.packed_data.get("int4")
        if pv is not None and cur["group_size"] != pv["group_size"]:
            raise ValueError(
                "INT4 group_size mismatch for reuse: "
                f"current={cur['group_size']} previous={pv['group_size']}"
            )
    stats = {"applied": 0, "skipped_precision": 0}
    if isinstance(reuse_mask, np.ndarray):
        ts, hs = np.nonzero(reuse_mask)
        reuse_mask = {(t, h): True for t, h in zip(ts.tolist(), hs.tolist())}
    if not reuse_mask or not prev.packed_data:
        return stats
    prev_prec: Dict[Tuple[int, int], str] = {}
    prev_pos: Dict[Tuple[int, int], int] = {}
    for p, pd in prev.packed_data.items():
        for i, e in enumerate(pd["indices"]):
            prev_prec[e] = p
            prev_pos[e] = i
    B = cache.batch_size
    for p, d in cache.packed_data.items():
        tgt, src = [], []
        for i, e in enumerate(d["indices"]):
            if not reuse_mask.get(e, False):
                continue
            if prev_prec.get(e) == p:
                tgt.append(i)
                src.append(prev_pos[e])
            elif e in prev_prec:
                stats["skipped_precision"] += 1
        if not tgt:
            continue
        pd = prev.packed_data[p]
        t_a, s_a = np.array(tgt), np.array(src)
        if p in ("fp32", "fp16", "int8"):
            d["k"][t_a] = pd["k"][s_a]
            d["v"][t_a] = pd["v"][s_a]
            if p == "int8":
                d["scale_k"][t_a] = pd["scale_k"][s_a]
                d["scale_v"][t_a] = pd["scale_v"][s_a]
        else:
            n, pn = len(d["indices"]), len(pd["indices"])
            rb = d["k"].size // n
            ng = d["num_groups"]
            d["k"].reshape(n, rb)[t_a] = pd["k"].reshape(pn, rb)[s_a]
            d["v"].reshape(n, rb)[t_a] = pd["v"].reshape(pn, rb)[s_a]
            d["scale_k"].reshape(n, B, ng, 1)[t_a] = pd["scale_k"].reshape(pn, B, ng, 1)[s_a]
            d["scale_v"].reshape(n, B, ng, 1)[t_a] = pd["scale_v"].reshape(pn, B, ng, 1)[s_a]
        stats["applied"] += len(tgt)
    return stats


def compress_dense(
    k: np.ndarray, v: np.ndarray, plan: Dict[str, Any], group_size: int = 16,
    k_prev: Optional[np.ndarray] = None, v_prev: Optional[np.ndarray] = None,
) -> Tuple[np.ndarray, np.ndarray]:
    """Dense working copy of ``_compress_kv_with_plan`` (shadowkv_agent.py:1698-1809).

    fp32 value / fp16-rounded value / raw int8 / raw int4 integer codes as fp32;
    evicted entries 0; reuse entries overwritten with ``k_prev`` when present.
    """
    B, H, S, D = k.shape
    ko = np.zeros_like(k, dtype=np.float32).reshape(B, H * S, D)
    vo = np.zeros_like(ko)
    kf = k.reshape(B, H * S, D)
    vf = v.reshape(B, H * S, D)
    for precision in PRECISION_ORDER:
        if not plan["groups"][precision]:
            continue
        flat = plan["flat_indices"][precision]
        for src, dst in ((kf, ko), (vf, vo)):
            grp = src[:, flat, :].transpose(1, 0, 2)
            if precision == "fp32":
                q = grp
            elif precision == "fp16":
                q = grp.astype(np.float16)
            elif precision == "int8":
                q, _ = quantize_int8(grp)
            else:
                q, _ = quantize_int4(grp, int4_group(D, group_size))
                q = q.reshape(q.shape[0], B, D)
            dst[:, flat, :] = q.astype(np.float32).transpose(1, 0, 2)
    if k_prev is not None and plan["reuse_flat"].size > 0:
        rf = plan["reuse_flat"]
        ko[:, rf, :] = k_prev.reshape(B, H * S, D)[:, rf, :]
        vo[:, rf, :] = v_prev.reshape(B, H * S, D)[:, rf, :]
    return ko.reshape(B, H, S, D), vo.reshape(B, H, S, D)


# --------------------------------------------------------------------------------------
# attention over the packed cache  (shadowinfer/models/simple_diffusion_llm.py:165-169)
# --------------------------------------------------------------------------------------
def attention(q: np.ndarray, k: np.ndarray, v: np.ndarray, scale: Optional[float] = None) -> np.ndarray:
    """Non-causal ``softmax(q k^T * scale) v`` in float64 (simple_diffusion_llm.py:165-169)."""
    D = q.shape[-1]
    if scale is None:
        scale = 1.0 / np.sqrt(D)
    q64 = q.astype(np.float64)
    out = np.empty(q.shape, dtype=np.float64)
    B, H = q.shape[0], q.shape[1]
    for b in range(B):
        for h in range(H):
            s = (q64[b, h] @ k[b, h].astype(np.float64).T) * scale
            s -= s.max(axis=-1, keepdims=True)
            p = np.exp(s)
            p /= p.sum(axis=-1, keepdims=True)
            out[b, h] = p @ v[b, h].astype(np.float64)
    return out


def attention_f32(q: np.ndarray, k: np.ndarray, v: np.ndarray, scale: Optional[float] = None) -> np.ndarray:
    """The same attention in the reference's own float32 arithmetic (simple_diffusion_llm.py:165-169:
    fp32 matmuls and softmax).  The CPU baselines time this one -- it runs at the speed of the
    reference's torch CPU path -- while the float64 ``attention`` above is the parity checker."""
    D = q.shape[-1]
    if scale is None:
        scale = 1.0 / np.sqrt(D)
    s = np.matmul(q.astype(np.float32), np.swapaxes(k.astype(np.float32), -1, -2)) * np.float32(scale)
    s -= s.max(axis=-1, keepdims=True)
    np.exp(s, out=s)
    s /= s.sum(axis=-1, keepdims=True)
    return np.matmul(s, v.astype(np.float32))


def repeat_kv(x: np.ndarray, n_rep: int) -> np.ndarray:
    """``[B, H_kv, S, D] -> [B, H_kv * n_rep, S, D]``, head h of the result = head h // n_rep
    (diffusion_llama.py:300-308)."""
    return np.repeat(x, n_rep, axis=1)


def packed_attention(q: np.ndarray, cache: OraclePackedKV, scale: Optional[float] = None,
                     k_new: Optional[np.ndarray] = None, v_new: Optional[np.ndarray] = None) -> np.ndarray:
    """Oracle for attention read from the packed cache: ``unpack()``, this step's own K/V appended
    (``cat((past, new), dim=2)``), KV heads repeated to the query heads, then dense attention
    (diffusion_llama.py:376-390, simple_diffusion_llm.py:160-169)."""
    k, v = unpack(cache)
    if k_new is not None:
        k = np.concatenate([k, k_new.astype(np.float32)], axis=2)
        v = np.concatenate([v, v_new.astype(np.float32)], axis=2)
    n_rep = q.shape[1] // k.shape[1]
    return attention(q, repeat_kv(k, n_rep), repeat_kv(v, n_rep), scale)


# --------------------------------------------------------------------------------------
# cross-layer budget enforcement  (shadowinfer/shadowkv/kv_cache_manager.py:129-200, 301-322)
# --------------------------------------------------------------------------------------
def manager_usage(layers: Sequence[Dict[str, Any]]) -> int:
    """``KVCacheManager.get_memory_usage`` (kv_cache_manager.py:301-322) for layers that hold a
    cache entry (``counted``): packed resident bytes plus the retained dense shadow bytes."""
    total = 0
    for L in layers:
        if L.get("counted", True):
            total += L["cache"].resident_bytes() + int(L.get("dense_bytes", 0))
    return total


def enforce_global_budget(layers: Sequence[Dict[str, Any]], budget_bytes: Optional[int], sink_tokens: int = 0) -> int:
    """Cross-layer eviction by ascending importance (kv_cache_manager.py:129-200).

    ``layers`` in the manager's importance-matrix insertion order, each a dict with
    ``cache`` (OraclePackedKV, evicted in place), ``importance`` (float [S, H]), ``counted``
    (the layer holds a cache entry, so its bytes count in the usage), ``candidate`` (it has
    an importance matrix; default True) and ``dense_bytes`` (retained dense shadow, released
    first under pressure).  Returns the number of candidates processed, as the reference does.
    """
    if budget_bytes is None or budget_bytes <= 0 or not layers:
        return 0
    target = int(budget_bytes * 0.9)
    if manager_usage(layers) > target:                 # _release_dense_shadows (:202-222)
        for L in layers:
            if L.get("counted", True):
                L["dense_bytes"] = 0
    if manager_usage(layers) <= target:
        return 0
    # candidates in (layer order, token, head) order, stably sorted by importance (:152-165)
    values, owner, token, head = [], [], [], []
    for li, L in enumerate(layers):
        if not L.get("candidate", True):
            continue
        imp = np.asarray(L["importance"], dtype=np.float32)
        S, H = imp.shape
        for t in range(sink_tokens, S):
            values.append(imp[t])
            owner.append(np.full(H, li))
            token.append(np.full(H, t))
            head.append(np.arange(H))
    if not values:
        return 0
    values = np.concatenate(values)
    owner, token, head = np.concatenate(owner), np.concatenate(token), np.concatenate(head)
    order = np.argsort(values, kind="stable")
    n = len(order)
    idx = 0
    evicted_total = 0
    while manager_usage(layers) > target and idx < n:   # batched eviction loop (:167-194)
        usage = manager_usage(layers)
        remaining = usage - target
        avg_entry = max(1, usage // max(1, n))
        batch = max(1, min(n - idx, remaining // avg_entry + 1))
        chunk = order[idx: idx + batch]
        idx += batch
        for li, L in enumerate(layers):
            sel = chunk[owner[chunk] == li]
            if len(sel) == 0:
                continue
            evict(L["cache"], set(zip(token[sel].tolist(), head[sel].tolist())))
            evicted_total += len(sel)
    return evicted_total
