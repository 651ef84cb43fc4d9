"""KV cache manager (drop-in for ``shadowinfer/shadowkv/kv_cache_manager.py``).

Same class, methods and semantics as the reference ``KVCacheManager``: per-layer
store/retrieve of ``KVCacheEntry`` objects and packed caches, usage accounting
(packed ``resident_bytes`` plus retained dense shadows), dense-shadow release, the
per-layer policy eviction (``_enforce_budget`` with an ``EvictionPolicy`` over
``TokenHeadScore`` records), the prefetch buffer and reuse statistics.

``enforce_global_budget`` (kv_cache_manager.py:129-200) runs on the GPU.  The
reference lists every non-sink (layer, token, head) of the layers with an importance
matrix, sorts the list stably by importance (a Python sort of L*S*H tuples) and
evicts it from the front in batches, re-reading the usage after each batch.  Here the
candidates are written by ``skv_budget_candidates`` (score + resident bytes freed),
the bytes freed by the first ``k`` candidates come from ``skv_rank_select`` for each
``k`` the batch loop visits (the loop itself is the reference's arithmetic, on the
host), and the final ``k`` candidates are marked by ``skv_mark_smallest`` and evicted
from each layer with the in-place ``PackedKVCache.evict``.  The returned count, the
surviving entries and the final usage equal the reference's.
"""

from __future__ import annotations

import abc
import ctypes
import logging
from dataclasses import dataclass
from typing import Any, Dict, List, Optional, Set, Tuple

import torch

from .. import _lib
from .._device import compute_device, device_ctx, scratch

_LOG = logging.getLogger("kv_cache_manager")
_RESIDENT_ENTRY_OVERHEAD = 48        # bytes of metadata per token-head (packed_kv_cache.py:869-878)


@dataclass
class KVCacheEntry:
    """One layer's KV cache entry (shadowinfer/core/structs.py:37-62)."""

    k_tensor: Optional[torch.Tensor]
    v_tensor: Optional[torch.Tensor]
    precision: str
    scale_k: Optional[torch.Tensor] = None
    scale_v: Optional[torch.Tensor] = None
    importance_score: float = 0.0
    is_reused: bool = False
    reuse_step: int = -1
    packed_kv: Optional[Any] = None
    paged_kv: Optional[Any] = None


@dataclass
class TokenHeadScore:
    """Metadata of one (layer, token, head) entry (shadowinfer/shadowkv/importance_model.py:25-34)."""

    layer_id: int
    token_idx: int
    head_idx: int
    importance: float
    drift: float = 0.0
    age: int = 0
    access_count: int = 1


class EvictionPolicy(abc.ABC):
    """Chooses (layer, token, head) entries to drop (shadowinfer/shadowkv/eviction_policy.py:17-38)."""

    @abc.abstractmethod
    def select_for_eviction(self, entries: List[TokenHeadScore], budget_bytes: int, current_usage_bytes: int,
                            estimated_entry_bytes: int) -> Set[Tuple[int, int, int]]:
        ...


def _select_lowest(entries: List[TokenHeadScore], key, budget_bytes: int, current_usage_bytes: int,
                   estimated_entry_bytes: int) -> Set[Tuple[int, int, int]]:
    if current_usage_bytes <= budget_bytes or not entries:
        return set()
    target_reduction = current_usage_bytes - budget_bytes
    num_to_evict = min(len(entries), max(1, int(target_reduction // max(1, estimated_entry_bytes))))
    chosen = sorted(entries, key=key)[:num_to_evict]
    return {(e.layer_id, e.token_idx, e.head_idx) for e in chosen}


class LeastImportantEvictionPolicy(EvictionPolicy):
    """Lowest importance first (eviction_policy.py:40-64)."""

    def select_for_eviction(self, entries, budget_bytes, current_usage_bytes, estimated_entry_bytes):
        return _select_lowest(entries, lambda e: e.importance, budget_bytes, current_usage_bytes,
                              estimated_entry_bytes)


class ImportanceAgeEvictionPolicy(EvictionPolicy):
    """Lowest ``importance * (1 - age_decay) ** age`` first (eviction_policy.py:67-98)."""

    def __init__(self, age_decay: float = 0.01):
        self.age_decay = age_decay

    def _score(self, entry: TokenHeadScore) -> float:
        return entry.importance * (1.0 - self.age_decay) ** entry.age

    def select_for_eviction(self, entries, budget_bytes, current_usage_bytes, estimated_entry_bytes):
        return _select_lowest(entries, self._score, budget_bytes, current_usage_bytes, estimated_entry_bytes)


def _policy_keys(entries: List[TokenHeadScore], policy: EvictionPolicy):
    """float64 sort keys of the built-in policies, the same IEEE values the reference computes
    (``importance`` or ``importance * (1 - age_decay) ** age``, the power taken by Python per
    distinct age)."""
    import numpy as np
    n = len(entries)
    imp = np.fromiter((e.importance for e in entries), dtype=np.float64, count=n)
    if isinstance(policy, ImportanceAgeEvictionPolicy):
        ages = np.fromiter((e.age for e in entries), dtype=np.int64, count=n)
        uniq, inv = np.unique(ages, return_inverse=True)
        factor = np.array([(1.0 - policy.age_decay) ** int(a) for a in uniq], dtype=np.float64)
        imp = imp * factor[inv]
    return imp


def _select_lowest_device(entries: List[TokenHeadScore], policy: EvictionPolicy, budget_bytes: int,
                          current_usage_bytes: int, estimated_entry_bytes: int, packed: Any) -> List[TokenHeadScore]:
    """The built-in policies' selection (eviction_policy.py:40-98: the ``num_to_evict`` entries
    of smallest key in a stable sort) without the Python sort, and the in-place eviction of the
    chosen entries from ``packed``.  Keys that float32 holds exactly (finite, no -0.0) are
    selected on the GPU by the rank select of ``enforce_global_budget`` (score = key, position =
    list order, the stable sort's tie order); other keys by a float64 stable argsort.  Returns the
    chosen entries."""
    import numpy as np
    if current_usage_bytes <= budget_bytes or not entries:
        return []
    n = len(entries)
    target_reduction = current_usage_bytes - budget_bytes
    k = min(n, max(1, int(target_reduction // max(1, estimated_entry_bytes))))
    keys = _policy_keys(entries, policy)
    dev = packed._ensure_state() if packed.packed_data else compute_device()
    k32 = keys.astype(np.float32)
    exact = bool(np.all(np.isfinite(keys)) and np.array_equal(k32.astype(np.float64), keys) and
                 not np.any((keys == 0) & np.signbit(keys)))
    if exact and n < (1 << 31):
        lib = _lib.load()
        score = torch.from_numpy(k32).to(dev)
        weight = torch.ones(n, dtype=torch.int64, device=dev)
        res = torch.empty(2, dtype=torch.int64, device=dev)
        mask = torch.empty(n, dtype=torch.uint8, device=dev)
        scr = scratch(lib.skv_rank_select_scratch_bytes(n), dev)
        stream = _lib.stream_of(dev)
        with device_ctx(dev):
            _lib.check(lib.skv_rank_select(_lib.ptr(score), _lib.ptr(weight), n, k, _lib.ptr(scr), scr.numel(),
                                           _lib.ptr(res), stream), "_enforce_budget")
            _lib.check(lib.skv_mark_smallest(_lib.ptr(score), n, _lib.ptr(res), _lib.ptr(mask), stream),
                       "_enforce_budget")
        chosen_idx = torch.nonzero(mask, as_tuple=True)[0].cpu().numpy()
        if int(res[0].item()) < 0:
            raise RuntimeError("_enforce_budget: the selection kernel's grid barrier timed out")
    else:
        chosen_idx = np.sort(np.argsort(keys, kind="stable")[:k])
    chosen = [entries[i] for i in chosen_idx.tolist()]
    S, H = int(packed.seq_len), int(packed.num_heads)
    tok = np.fromiter((e.token_idx for e in chosen), dtype=np.int64, count=len(chosen))
    head = np.fromiter((e.head_idx for e in chosen), dtype=np.int64, count=len(chosen))
    inside = (tok >= 0) & (tok < S) & (head >= 0) & (head < H)
    ev = torch.zeros(S * H, dtype=torch.bool)
    ev[torch.from_numpy(tok[inside] * H + head[inside])] = True
    packed.evict(ev.view(S, H).to(dev))
    return chosen


def _resident_entry_cost(packed: Any) -> List[int]:
    """Resident bytes one stored entry of each precision takes in ``packed``: its K/V payload,
    its scales and the per-entry metadata (the quantities ``resident_bytes`` sums)."""
    B, D = int(packed.batch_size), int(packed.head_dim)
    G = packed._int4_group_of() if hasattr(packed, "_int4_group_of") else D
    G = G if G > 0 and D % G == 0 else D
    return [
        2 * B * D * 4 + _RESIDENT_ENTRY_OVERHEAD,
        2 * B * D * 2 + _RESIDENT_ENTRY_OVERHEAD,
        2 * (B * D + 4 * B) + _RESIDENT_ENTRY_OVERHEAD,
        2 * ((B * D + 1) // 2 + 4 * B * (D // G)) + _RESIDENT_ENTRY_OVERHEAD,
    ]


class KVCacheManager:
    """Per-layer KV storage with budget enforcement (kv_cache_manager.py:24-371)."""

    def __init__(self, num_layers: int, memory_budget_bytes: Optional[int] = None,
                 eviction_policy: Optional[EvictionPolicy] = None):
        self.num_layers = num_layers
        self.memory_budget_bytes = memory_budget_bytes
        self.eviction_policy = eviction_policy or LeastImportantEvictionPolicy()
        self.cache: Dict[int, Any] = {}
        self._packed_cache: Dict[int, Any] = {}
        self._reuse_count = 0
        self._total_access = 0
        self._reuse_history: Dict[int, List[bool]] = {}
        self._token_head_meta: Dict[int, Dict[Tuple[int, int], TokenHeadScore]] = {}
        self._importance_matrices: Dict[int, torch.Tensor] = {}
        self._importance_cpu: Dict[int, torch.Tensor] = {}
        self._prefetch_buffer: Dict[Tuple[int, str], Any] = {}

    # ------------------------------------------------------------------ store / retrieve
    def store(self, layer_id: int, entry: Any) -> None:
        """Store an entry, then enforce the per-layer budget (kv_cache_manager.py:61-76)."""
        self.cache[layer_id] = entry
        if entry.packed_kv is not None:
            self._packed_cache[layer_id] = entry.packed_kv
        self._reuse_history.setdefault(layer_id, []).append(entry.is_reused)
        self._total_access += 1
        if entry.is_reused:
            self._reuse_count += 1
        self._enforce_budget(layer_id)

    def retrieve(self, layer_id: int) -> Optional[Any]:
        return self.cache.get(layer_id, None)

    def store_packed(self, layer_id: int, packed_kv: Any) -> None:
        if isinstance(packed_kv, dict):
            packed_kv = packed_kv.get("packed_kv", packed_kv)
        self._packed_cache[layer_id] = packed_kv

    def retrieve_packed(self, layer_id: int) -> Optional[Any]:
        return self._packed_cache.get(layer_id, None)

    # ---------------------------------------------------------------- metadata & eviction
    def set_token_head_meta(self, layer_id: int, meta: Dict[Tuple[int, int], TokenHeadScore]) -> None:
        self._token_head_meta[layer_id] = meta

    def get_token_head_meta(self, layer_id: int) -> Dict[Tuple[int, int], TokenHeadScore]:
        return dict(self._token_head_meta.get(layer_id, {}))

    def set_importance_matrix(self, layer_id: int, importance: torch.Tensor) -> None:
        """Importance ``[seq, heads]`` of a layer, kept where it lives (kv_cache_manager.py:103-123).

        ``get_importance_matrix`` returns a CPU copy, as the reference stores one.
        """
        previous = self._importance_matrices.get(layer_id)
        if previous is not None and tuple(previous.shape) != tuple(importance.shape):
            _LOG.warning("importance matrix shape changed for layer %s: %s -> %s", layer_id,
                         tuple(previous.shape), tuple(importance.shape))
        self._importance_matrices[layer_id] = importance.detach()
        self._importance_cpu.pop(layer_id, None)

    def get_importance_matrix(self, layer_id: int) -> Optional[torch.Tensor]:
        m = self._importance_matrices.get(layer_id)
        if m is None:
            return None
        if layer_id not in self._importance_cpu:
            self._importance_cpu[layer_id] = m.cpu()
        return self._importance_cpu[layer_id]

    def enforce_global_budget(self, budget_bytes: int, sink_tokens: int = 0) -> int:
        """Evict non-sink token-heads across layers by ascending importance until the usage is at
        most ``0.9 * budget_bytes`` (kv_cache_manager.py:129-200).

        Returns the number of candidates processed, as the reference counts them.
        """
        if budget_bytes is None or budget_bytes <= 0:
            return 0
        if not self._packed_cache:
            return 0
        target = int(budget_bytes * 0.9)
        if self.get_memory_usage() > target:
            self._release_dense_shadows()
        usage0 = self.get_memory_usage()
        if usage0 <= target:
            return 0
        layers = [(lid, m, self._packed_cache[lid]) for lid, m in self._importance_matrices.items()
                  if lid in self._packed_cache]
        sizes = [max(0, int(m.shape[0]) - sink_tokens) * int(m.shape[1]) for _, m, _ in layers]
        n = sum(sizes)
        if n == 0:
            _LOG.warning("global budget enforcement reached floor: usage=%s target=%s", usage0, target)
            return 0
        devs = [p._ensure_state() for _, _, p in layers if p.packed_data]
        dev = devs[0] if devs else compute_device()
        lib = _lib.load()
        stream = _lib.stream_of(dev)
        score = torch.empty(n, dtype=torch.float32, device=dev)
        weight = torch.empty(n, dtype=torch.int64, device=dev)
        spans = []
        off = 0
        with device_ctx(dev):
            for (lid, m, packed), size in zip(layers, sizes):
                spans.append((off, size))
                if size == 0:
                    continue
                imp = m.to(device=dev, dtype=torch.float32).contiguous()
                counted = lid in self.cache
                cost = _resident_entry_cost(packed) if counted else [0, 0, 0, 0]
                cost_arr = (ctypes.c_int64 * 4)(*cost)
                slot = packed._slot.to(dev) if (packed.packed_data and packed._slot is not None) else None
                st = lib.skv_budget_candidates(_lib.ptr(imp), int(m.shape[0]), int(m.shape[1]), _lib.ptr(slot),
                                               packed.seq_len, packed.num_heads, int(sink_tokens),
                                               ctypes.cast(cost_arr, ctypes.c_void_p),
                                               _lib.ptr(score[off:]), _lib.ptr(weight[off:]), stream)
                _lib.check(st, "enforce_global_budget")
                off += size
            # the reference's batch loop (kv_cache_manager.py:167-194); the bytes freed by the
            # first idx candidates come from the device selection
            res = torch.empty(2, dtype=torch.int64, device=dev)
            scr = scratch(lib.skv_rank_select_scratch_bytes(n), dev)
            idx, usage = 0, usage0
            while usage > target and idx < n:
                remaining = usage - target
                avg_entry = max(1, usage // max(1, n))
                batch = max(1, min(n - idx, remaining // avg_entry + 1))
                idx += batch
                st = lib.skv_rank_select(_lib.ptr(score), _lib.ptr(weight), n, idx, _lib.ptr(scr), scr.numel(),
                                         _lib.ptr(res), stream)
                _lib.check(st, "enforce_global_budget")
                freed = int(res[0].item())
                if freed < 0:
                    raise RuntimeError("enforce_global_budget: the selection kernel's grid barrier timed out")
                usage = usage0 - freed
            mask = torch.empty(n, dtype=torch.uint8, device=dev)
            st = lib.skv_mark_smallest(_lib.ptr(score), n, _lib.ptr(res), _lib.ptr(mask), stream)
            _lib.check(st, "enforce_global_budget")
        for (lid, m, packed), (o, size) in zip(layers, spans):
            if size == 0 or not packed.packed_data:
                continue
            S_m, H_m = int(m.shape[0]), int(m.shape[1])
            sel = mask[o:o + size].view(S_m - sink_tokens, H_m).bool()
            ev = torch.zeros(packed.seq_len, packed.num_heads, dtype=torch.bool, device=dev)
            rows = min(S_m, packed.seq_len) - sink_tokens
            cols = min(H_m, packed.num_heads)
            if rows > 0 and cols > 0:
                ev[sink_tokens:sink_tokens + rows, :cols] = sel[:rows, :cols]
                packed.evict(ev)
        if self.get_memory_usage() > target and idx >= n:
            _LOG.warning("global budget enforcement reached floor: usage=%s target=%s", self.get_memory_usage(),
                         target)
        return idx

    def _release_dense_shadows(self) -> bool:
        """Drop dense shadows of layers that have a packed cache (kv_cache_manager.py:202-222)."""
        released = False
        for layer_id, entry in self.cache.items():
            if self._packed_cache.get(layer_id) is None:
                continue
            if any(t is not None for t in (entry.k_tensor, entry.v_tensor, entry.scale_k, entry.scale_v)):
                entry.k_tensor = None
                entry.v_tensor = None
                entry.scale_k = None
                entry.scale_v = None
                released = True
        return released

    def _enforce_budget(self, layer_id: int) -> None:
        """Per-layer policy eviction over ``TokenHeadScore`` records (kv_cache_manager.py:224-272)."""
        if self.memory_budget_bytes is None or self.memory_budget_bytes <= 0:
            return
        current_usage = self.get_memory_usage()
        if current_usage > self.memory_budget_bytes and self._release_dense_shadows():
            current_usage = self.get_memory_usage()
        if current_usage <= self.memory_budget_bytes:
            return
        entry = self.cache.get(layer_id)
        if entry is None or entry.packed_kv is None:
            return
        meta = self._token_head_meta.get(layer_id, {})
        if not meta:
            return
        packed = entry.packed_kv
        seq_len = getattr(packed, "seq_len", 0) or 0
        num_heads = getattr(packed, "num_heads", 0) or 0
        total_entries = max(1, seq_len * num_heads)
        if hasattr(packed, "memory_bytes"):
            estimated_entry_bytes = max(1, int(packed.memory_bytes()) // total_entries)
        else:
            estimated_entry_bytes = (getattr(packed, "batch_size", 1) or 1) * (getattr(packed, "head_dim", 1) or 1)
        policy = self.eviction_policy
        if type(policy) in (LeastImportantEvictionPolicy, ImportanceAgeEvictionPolicy) and \
                getattr(packed, "_slot", None) is not None:
            chosen = _select_lowest_device(list(meta.values()), policy, self.memory_budget_bytes, current_usage,
                                           estimated_entry_bytes, packed)
            if chosen:
                for e in chosen:
                    e.importance = -1.0
            return
        to_evict = policy.select_for_eviction(
            list(meta.values()), budget_bytes=self.memory_budget_bytes, current_usage_bytes=current_usage,
            estimated_entry_bytes=estimated_entry_bytes)
        if to_evict:
            packed.evict({(t, h) for _, t, h in to_evict})
            for _, t, h in to_evict:
                if (t, h) in meta:
                    meta[(t, h)].importance = -1.0

    # ------------------------------------------------------------------- prefetch buffer
    def store_prefetched(self, layer_id: int, tag: str, entry: Any) -> None:
        self._prefetch_buffer[(layer_id, tag)] = entry

    def retrieve_prefetched(self, layer_id: int, tag: str) -> Optional[Any]:
        return self._prefetch_buffer.get((layer_id, tag), None)

    def clear_prefetch_buffer(self, tag: Optional[str] = None) -> None:
        if tag is None:
            self._prefetch_buffer.clear()
            return
        for key in [k for k in self._prefetch_buffer if k[1] == tag]:
            del self._prefetch_buffer[key]

    # ------------------------------------------------------------------------- lifecycle
    def clear(self) -> None:
        self.cache.clear()
        self._packed_cache.clear()
        self._reuse_count = 0
        self._total_access = 0
        self._reuse_history.clear()
        self._token_head_meta.clear()
        self._importance_matrices.clear()
        self._importance_cpu.clear()
        self._prefetch_buffer.clear()

    # ------------------------------------------------------------------------ statistics
    def get_memory_usage(self) -> int:
        """Packed resident bytes plus retained dense shadows (kv_cache_manager.py:301-322)."""
        total = 0
        for layer_id, entry in self.cache.items():
            packed = self._packed_cache.get(layer_id)
            if packed is not None and hasattr(packed, "resident_bytes"):
                total += packed.resident_bytes()
                for t in (entry.k_tensor, entry.v_tensor, entry.scale_k, entry.scale_v):
                    total += self._tensor_bytes(t)
            elif packed is not None and hasattr(packed, "memory_bytes"):
                total += packed.memory_bytes()
            else:
                total += self._tensor_bytes(entry.k_tensor) + self._tensor_bytes(entry.v_tensor)
                total += self._tensor_bytes(entry.scale_k) + self._tensor_bytes(entry.scale_v)
        return total

    def get_memory_usage_mb(self) -> float:
        return self.get_memory_usage() / (1024.0 * 1024.0)

    def get_reuse_stats(self) -> Dict[str, float]:
        stats: Dict[str, float] = {"global_reuse_rate": 0.0}
        if self._total_access > 0:
            stats["global_reuse_rate"] = self._reuse_count / self._total_access
        for layer_id, history in self._reuse_history.items():
            stats[f"layer_{layer_id}_reuse_rate"] = sum(history) / len(history) if history else 0.0
        return stats

    @staticmethod
    def _tensor_bytes(tensor: Optional[torch.Tensor]) -> int:
        return 0 if tensor is None else tensor.numel() * tensor.element_size()

    def __repr__(self) -> str:
        budget_mb = self.memory_budget_bytes / (1024.0 * 1024.0) if self.memory_budget_bytes else None
        return (f"KVCacheManager(num_layers={self.num_layers}, cached_layers={len(self.cache)}, "
                f"memory_mb={self.get_memory_usage_mb():.2f}, budget_mb={budget_mb})")
