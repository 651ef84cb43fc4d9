"""Data-plane methods of ``ShadowKVAgent`` (shadowinfer/shadowkv/shadowkv_agent.py).

Only the data-plane methods of the reference agent are provided --
``allocate_precision_codes`` (:1028-1059), ``_admit_precision_codes``
(:679-743), ``compress_kv`` (:1445-1584), ``_compress_kv_with_plan``
(:1698-1809), and the decision inputs ``decide_reuse_per_token`` (:1165-1256),
``_compute_importance_matrix`` / ``_compute_importance_with_state`` (:899-965,
IRAP importance) and ``_row_normalize`` (:893-897) -- with the reference's
signatures and return values.  The agent's policy logic (stats, prefetch,
``on_step`` orchestration) is outside this package.

``compress_kv`` builds the plan on the GPU and runs ONE fused kernel that
writes both the packed buckets and the dense working copy (``k``/``v`` of the
result: fp32 values, fp16-rounded values, raw int8/int4 integer codes as fp32,
zeros for evicted entries, previous-step rows for reused entries).
"""

from __future__ import annotations

from collections.abc import Mapping
from typing import Any, Dict, List, Optional, Set, Tuple

import torch

from .. import _lib
from .._device import back, compute_device, on, device_ctx
from .importance_model import INPUT_LOGITS, INPUT_UNNORMALISED, irap_importance
from .packed_kv_cache import PackedKVCache, run_pack
from .precision_plan import PRECISION_ORDER, PrecisionPlan
from .rd_allocator import admit_codes, kv_sensitivity, predict_codes_bytes

_MODES = {"aggressive": 0, "balanced": 1, "conservative": 2}


def allocate_precision_codes(importance_map: torch.Tensor, mode: str) -> torch.Tensor:
    """Threshold bands (float64 compares) -> ``int8 [seq, heads]`` codes (shadowkv_agent.py:1028-1059)."""
    dev = compute_device(importance_map)
    imp = on(importance_map, dev, torch.float32)
    out = torch.empty(imp.shape, dtype=torch.int8, device=dev)
    lib = _lib.load()
    with device_ctx(dev):
        st = lib.skv_allocate_codes(_lib.ptr(imp), imp.numel(), _MODES.get(mode, -1), _lib.ptr(out),
                                    _lib.stream_of(dev))
    _lib.check(st, "allocate_precision_codes")
    return back(out, importance_map.device)


_REUSE_BASE = {"aggressive": 0.20, "balanced": 0.15, "conservative": 0.10}


def reuse_threshold(step_id: int, total_steps: int, qdrift_drift_score: float, mode: str) -> float:
    """Effective drift threshold before the importance term (shadowkv_agent.py:1222-1231)."""
    progress = step_id / max(total_steps, 1)
    adaptive = _REUSE_BASE.get(mode, 0.15) * (1.0 - 0.5 * progress)
    return adaptive * (1.0 - qdrift_drift_score * 0.3)


def decide_reuse_mask(
    kv_current_k: torch.Tensor,
    kv_current_v: torch.Tensor,
    kv_previous_k: torch.Tensor,
    kv_previous_v: torch.Tensor,
    step_id: int,
    total_steps: int,
    qdrift_drift_score: float,
    mode: str,
    importance_map: torch.Tensor,
    return_drift: bool = False,
):
    """``decide_reuse_per_token`` as a device mask: (bool ``[seq, heads]``, stats[, drift ``[seq,
    heads]``]) on the compute device, without building the ``{(t, h): bool}`` dict.

    drift = (|k - k_prev| / (|k| + 1e-8) + |v - v_prev| / (|v| + 1e-8)) / 2 per (token, head),
    norms over (batch, head_dim); reuse where drift < max(thr * (1 - 0.3 * clamp(imp, 0, 1)), 1e-5).
    """
    B, H, S, D = (int(x) for x in kv_current_k.shape)
    for t in (kv_current_v, kv_previous_k, kv_previous_v):
        if tuple(t.shape) != (B, H, S, D):
            raise ValueError("current and previous K/V must have the same [batch, heads, seq, head_dim] shape")
    if tuple(importance_map.shape) != (S, H):
        raise ValueError(f"importance_map must be [seq, heads] = [{S}, {H}], got {tuple(importance_map.shape)}")
    dev = compute_device(kv_current_k, kv_current_v, kv_previous_k, kv_previous_v, importance_map)
    kc, vc, kp, vp = (on(t, dev, torch.float32) for t in (kv_current_k, kv_current_v, kv_previous_k,
                                                                   kv_previous_v))
    imp = on(importance_map, dev, torch.float32)
    mask = torch.empty(S, H, dtype=torch.bool, device=dev)
    drift = torch.empty(S, H, dtype=torch.float32, device=dev) if return_drift else None
    counts = torch.empty(4, dtype=torch.int64, device=dev)
    eff = reuse_threshold(step_id, total_steps, qdrift_drift_score, mode)
    lib = _lib.load()
    with device_ctx(dev):
        st = lib.skv_reuse_decide(_lib.ptr(kc), _lib.ptr(vc), _lib.ptr(kp), _lib.ptr(vp), B, H, S, D, _lib.ptr(imp),
                                  eff, _lib.ptr(mask), _lib.ptr(drift), _lib.ptr(counts), _lib.stream_of(dev))
    _lib.check(st, "decide_reuse_per_token")
    stats = ReuseStats(counts, S * H)
    return (mask, stats, drift) if return_drift else (mask, stats)


class ReuseStats(Mapping):
    """The stats dict of ``decide_reuse_per_token`` (full / partial / no reuse counts, reuse ratio),
    read from the device on first access: a caller that does not look at them does not wait for
    the decision kernel."""

    _KEYS = ("full_reuse_count", "partial_reuse_count", "no_reuse_count", "reuse_ratio")

    def __init__(self, counts: torch.Tensor, entries: int):
        self._counts, self._entries, self._d = counts, entries, None

    def _get(self) -> Dict[str, float]:
        if self._d is None:
            full, partial, none, reused = self._counts.tolist()
            self._d = {"full_reuse_count": float(full), "partial_reuse_count": float(partial),
                       "no_reuse_count": float(none), "reuse_ratio": float(reused / max(self._entries, 1))}
        return self._d

    def __getitem__(self, key):
        return self._get()[key]

    def __iter__(self):
        return iter(self._KEYS)

    def __len__(self):
        return len(self._KEYS)

    def __eq__(self, other):
        return dict(self._get()) == (dict(other) if isinstance(other, Mapping) else other)

    def __repr__(self):
        return repr(self._get())


class ShadowKVAgent:
    """Hot-path subset of the reference ``ShadowKVAgent``.

    Config keys (same names and defaults as the reference, shadowkv_agent.py:70-211):
    ``num_layers`` (32), ``num_heads`` (32), ``head_dim`` (128),
    ``use_packed_cache`` (True), ``int4_group_size`` (16, must be >= 1),
    ``rd_allocation_enabled`` (True), ``hard_eviction_enabled`` (False),
    ``sink_tokens`` (4, must be >= 0), ``memory_budget_mb`` (None).
    """

    def __init__(self, config: Optional[Dict[str, Any]] = None):
        self.config = dict(config or {})
        c = self.config
        self.num_layers = c.get("num_layers", 32)
        self.num_heads = c.get("num_heads", 32)
        self.head_dim = c.get("head_dim", 128)
        self.use_packed_cache = c.get("use_packed_cache", True)
        self.int4_group_size = int(c.get("int4_group_size", 16))
        if self.int4_group_size < 1:
            raise ValueError(f"int4_group_size must be >= 1, got {self.int4_group_size}")
        self.rd_allocation_enabled = bool(c.get("rd_allocation_enabled", True))
        self.hard_eviction_enabled = bool(c.get("hard_eviction_enabled", False))
        self.sink_tokens = int(c.get("sink_tokens", 4))
        if self.sink_tokens < 0:
            raise ValueError(f"sink_tokens must be >= 0, got {self.sink_tokens}")
        mb = c.get("memory_budget_mb")
        self.memory_budget_bytes = int(mb * 1024 * 1024) if mb is not None else None
        self._compression_stats = {"total_original_bytes": 0, "total_compressed_bytes": 0, "step_count": 0}
        self.last_admission: Dict[str, int] = {}

    def allocate_precision_codes(self, importance_map: torch.Tensor, mode: str) -> torch.Tensor:
        return allocate_precision_codes(importance_map, mode)

    # ---------------------------------------------------------------- decision inputs
    def decide_reuse_per_token(
        self,
        kv_current_k: torch.Tensor,
        kv_current_v: torch.Tensor,
        kv_previous_k: torch.Tensor,
        kv_previous_v: torch.Tensor,
        step_id: int,
        total_steps: int,
        qdrift_drift_score: float,
        mode: str,
        importance_map: torch.Tensor,
    ) -> Tuple[Dict[Tuple[int, int], bool], Dict[str, float]]:
        """Per-(token, head) KV reuse decision (shadowkv_agent.py:1165-1256): the drift and the
        threshold comparison run on the GPU (``decide_reuse_mask``); the returned dict and stats
        are the reference's."""
        mask, stats = decide_reuse_mask(kv_current_k, kv_current_v, kv_previous_k, kv_previous_v, step_id,
                                        total_steps, qdrift_drift_score, mode, importance_map)
        S, H = mask.shape
        flags: List[bool] = mask.reshape(-1).tolist()
        keys = [(t, h) for t in range(S) for h in range(H)]
        return dict(zip(keys, flags)), dict(stats)

    @staticmethod
    def _row_normalize(tensor: torch.Tensor) -> torch.Tensor:
        """Row-sum correction of probability inputs (shadowkv_agent.py:893-897)."""
        return tensor / tensor.sum(dim=-1, keepdim=True).clamp(min=1e-10)

    def _compute_importance_with_state(
        self,
        attention_scores: torch.Tensor,
        layer_index: int,
        num_layers: int,
        attn_is_probabilities: bool = False,
        received_ema=None,
        irap_decay: float = 0.9,
        entropy_weight: float = 0.3,
        sink_tokens: int = 4,
    ) -> Tuple[torch.Tensor, torch.Tensor, Optional[float]]:
        """Importance + new EMA state + delta A (shadowkv_agent.py:940-965): probabilities get the
        row-sum correction, logits a softmax of the NaN-cleaned rows, both fused into the IRAP
        pass on the GPU."""
        mode = INPUT_UNNORMALISED if attn_is_probabilities else INPUT_LOGITS
        return irap_importance(attention_scores, mode, received_ema, irap_decay, entropy_weight, sink_tokens,
                               layer_index, num_layers)

    def _compute_importance_matrix(
        self,
        attention_scores: torch.Tensor,
        layer_index: int,
        num_layers: int,
        attn_is_probabilities: bool = False,
        received_ema=None,
        irap_decay: float = 0.9,
        entropy_weight: float = 0.3,
        sink_tokens: int = 4,
    ) -> torch.Tensor:
        """Importance ``[seq_k, heads]`` only (shadowkv_agent.py:899-938)."""
        return self._compute_importance_with_state(attention_scores, layer_index, num_layers, attn_is_probabilities,
                                                   received_ema, irap_decay, entropy_weight, sink_tokens)[0]

    def _admit_precision_codes(
        self,
        codes: torch.Tensor,
        importance_map: torch.Tensor,
        kv_current: Dict[str, torch.Tensor],
        protected: Optional[Any] = None,
    ) -> torch.Tensor:
        """Per-layer budget admission (shadowkv_agent.py:679-743).

        ``protected``: set of ``(t, h)`` or a bool ``[seq, heads]`` tensor.
        """
        budget = self.memory_budget_bytes
        if not budget or budget <= 0:
            return codes
        layer_budget = max(1, int(budget) // max(1, self.num_layers))
        k, v = kv_current["k"], kv_current["v"]
        batch, _, _, head_dim = k.shape
        if predict_codes_bytes(codes, batch, head_dim, group_size=self.int4_group_size) <= layer_budget:
            return codes
        sens = kv_sensitivity(k, v)
        prot = None
        if protected is not None:
            if torch.is_tensor(protected):
                prot = protected
            elif protected:
                prot = torch.zeros(codes.shape[0], codes.shape[1], dtype=torch.bool)
                for t, h in protected:
                    if 0 <= t < codes.shape[0] and 0 <= h < codes.shape[1]:
                        prot[t, h] = True
        out, predicted, evicted = admit_codes(
            codes, importance_map, sens, layer_budget, batch=batch, head_dim=head_dim,
            sink_tokens=self.sink_tokens, rd_allocation=self.rd_allocation_enabled,
            allow_eviction=self.hard_eviction_enabled, protected_mask=prot, group_size=self.int4_group_size)
        self.last_admission = {"layer_budget": layer_budget, "predicted": predicted, "evicted": evicted}
        return out

    def compress_kv(
        self,
        kv_current: Dict[str, torch.Tensor],
        precision_map: Optional[Dict[int, Dict[int, str]]],
        reuse_decision: Optional[Dict[str, Any]] = None,
        reuse_mask: Any = None,
        kv_previous: Optional[Dict[str, torch.Tensor]] = None,
        build_scale_map: bool = True,
        precision_codes: Optional[torch.Tensor] = None,
    ) -> Dict[str, Any]:
        """Quantise K/V per the plan; returns the reference's result dict (shadowkv_agent.py:1445-1584)."""
        k, v = kv_current["k"], kv_current["v"]
        batch_size, num_heads, seq_len, head_dim = k.shape
        mask = reuse_mask
        if mask is None and reuse_decision is not None and "reuse_mask" in reuse_decision:
            mask = reuse_decision["reuse_mask"]
        if mask is None and reuse_decision is not None and reuse_decision.get("should_reuse", False):
            heads = set(reuse_decision.get("reused_heads", []))
            if heads:
                m = torch.zeros(seq_len, num_heads, dtype=torch.bool)
                m[:, sorted(h for h in heads if 0 <= h < num_heads)] = True
                mask = m
        k_prev = kv_previous["k"] if kv_previous is not None else None
        v_prev = kv_previous["v"] if kv_previous is not None else None
        plan_mask = mask if k_prev is not None else None
        if precision_codes is not None:
            plan = PrecisionPlan.from_codes(precision_codes, reuse_mask=plan_mask, device=k.device)
        else:
            plan = PrecisionPlan.build(precision_map or {}, seq_len, num_heads, reuse_mask=plan_mask, device=k.device)
        core = self._compress_kv_with_plan(k, v, k_prev, v_prev, plan, build_scale_map)
        original = k.numel() * k.element_size() + v.numel() * v.element_size()
        result: Dict[str, Any] = {"k": core["k"], "v": core["v"], "scale_k_map": core["scale_k_map"],
                                  "scale_v_map": core["scale_v_map"]}
        packed = core["packed_kv"]
        compressed = packed.memory_bytes()
        if self.use_packed_cache:
            result["packed_kv"] = packed
            result["memory_bytes"] = compressed
        result["compression_ratio"] = 1.0 - compressed / original if original > 0 else 0.0
        result["memory_mb"] = (original - compressed) / (1024.0 * 1024.0)
        result["uncompressed_bytes"] = original
        result["compressed_bytes"] = compressed
        self._compression_stats["total_original_bytes"] += original
        self._compression_stats["total_compressed_bytes"] += compressed
        self._compression_stats["step_count"] += 1
        return result

    def _compress_kv_with_plan(
        self,
        k_tensor: torch.Tensor,
        v_tensor: torch.Tensor,
        k_prev: Optional[torch.Tensor],
        v_prev: Optional[torch.Tensor],
        plan: PrecisionPlan,
        build_scale_map: bool,
    ) -> Dict[str, Any]:
        """Fused quantise + pack + dense working copy for one plan (shadowkv_agent.py:1698-1809)."""
        batch_size, num_heads, seq_len, head_dim = k_tensor.shape
        if plan.seq_len != seq_len or plan.num_heads != num_heads or v_tensor.shape != k_tensor.shape:
            raise ValueError(
                "PrecisionPlan shape mismatch: plan "
                f"(seq_len={plan.seq_len}, num_heads={plan.num_heads}) vs "
                f"tensor (seq_len={seq_len}, num_heads={num_heads})"
            )
        reuse_active = k_prev is not None and plan.reuse_mask_device is not None
        if reuse_active and v_prev is None:
            raise ValueError("v_prev is required when reuse entries are active")
        if reuse_active and (k_prev.shape != k_tensor.shape or v_prev.shape != v_tensor.shape):
            raise ValueError("previous KV tensors must match the current KV shape")
        if plan.codes.device.type != k_tensor.device.type:
            raise ValueError(
                f"PrecisionPlan device ({plan.codes.device}) does not match KV device ({k_tensor.device})"
            )
        buckets, dk, dv = run_pack(k_tensor, v_tensor, plan, self.int4_group_size, dense=True,
                                   k_prev=k_prev if reuse_active else None, v_prev=v_prev if reuse_active else None)
        cache = PackedKVCache(batch_size, num_heads, seq_len, head_dim, device=k_tensor.device)
        cache._adopt(buckets, plan.slot, shared_slot=True, group_size=self.int4_group_size)
        scale_k_map = scale_v_map = None
        if build_scale_map:
            scale_k_map, scale_v_map = {}, {}
            reuse = plan.reuse_set() if reuse_active else set()
            for p, data in cache.packed_data.items():
                entries = data["indices"]
                sk, sv = data["scale_k"], data["scale_v"]
                if p == "int4":
                    ng = data["num_groups"]
                    sk = sk.reshape(len(entries), batch_size, ng, 1)
                    sv = sv.reshape(len(entries), batch_size, ng, 1)
                for i, e in enumerate(entries):
                    if e in reuse:
                        continue
                    scale_k_map[e] = None if sk is None else sk[i:i + 1]
                    scale_v_map[e] = None if sv is None else sv[i:i + 1]
        return {"k": back(dk, k_tensor.device), "v": back(dv, v_tensor.device), "scale_k_map": scale_k_map,
                "scale_v_map": scale_v_map, "packed_kv": cache}
