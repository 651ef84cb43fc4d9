"""CPU oracle for the paged KV store -- TEST INFRASTRUCTURE ONLY.

numpy restatement of ``PagedKVStore`` (reference ``shadowinfer/shadowkv/paged_kv_store.py``):
per-precision pages of at most ``page_size`` tokens in token order, row-local
quantisation bit-aligned with ``PackedKVCache``, a slot pool with a free list,
token-granular eviction that splits pages into runs, in-place rewrites and the
byte ledgers.  Imported only by ``tests/`` and ``bench.py``'s CPU legs; the
product package never imports it.

Parity is pinned by ``tests/golden/make_golden.py``, which replays scripted
operation sequences on the reference store and records its page layout,
counters, byte ledgers and SHA-256 digests of every page tensor and gather
result after each step (``tests/test_oracle_golden.py::test_paged_store``).
"""

from __future__ import annotations

import hashlib
from typing import Any, Dict, Iterable, List, Optional, Set, Tuple

import numpy as np

from oracle.shadowkv_oracle import int4_group, quantize_int4, quantize_int8

PRECISIONS = ("fp32", "fp16", "int8", "int4")


class OraclePage:
    """One page (paged_kv_store.py:24-58): payload arrays ``[B,H,n,*]`` of one precision."""

    __slots__ = ("precision", "k", "v", "scale_k", "scale_v", "start_token", "num_tokens", "sealed")

    def __init__(self, precision, k, v, scale_k, scale_v, start_token, num_tokens, sealed):
        self.precision = precision
        self.k, self.v, self.scale_k, self.scale_v = k, v, scale_k, scale_v
        self.start_token, self.num_tokens, self.sealed = start_token, num_tokens, sealed

    @property
    def end_token(self) -> int:
        return self.start_token + self.num_tokens


def pack_rows_lastdim(codes: np.ndarray) -> np.ndarray:
    """int4 codes ``[..., G, g]`` -> bytes ``[..., ceil(D/2)]``, ``(q+8)`` high nibble first,
    a zero nibble after an odd last element (paged_kv_store.py:212-222)."""
    flat = codes.reshape(*codes.shape[:-2], -1)
    off = (flat.astype(np.int16) + 8).astype(np.uint8)
    if off.shape[-1] % 2:
        off = np.concatenate([off, np.zeros((*off.shape[:-1], 1), dtype=np.uint8)], axis=-1)
    return (((off[..., 0::2] << 4) & 0xF0) | (off[..., 1::2] & 0x0F)).astype(np.uint8)


class OraclePagedStore:
    """numpy mirror of ``PagedKVStore`` (paged_kv_store.py:61-717)."""

    def __init__(self, batch_size: int, num_heads: int, head_dim: int, page_size: int = 32,
                 int4_group_size: int = 16):
        if page_size < 1:
            raise ValueError(f"page_size must be >= 1, got {page_size}")
        if int4_group_size < 1:
            raise ValueError(f"int4_group_size must be >= 1, got {int4_group_size}")
        self.batch_size, self.num_heads, self.head_dim = int(batch_size), int(num_heads), int(head_dim)
        self.page_size, self.int4_group_size = int(page_size), int(int4_group_size)
        self.clear()

    def clear(self) -> None:
        """paged_kv_store.py:694-704."""
        self.pages: List[Optional[OraclePage]] = []
        self.order: List[int] = []
        self.free_slots: List[int] = []
        self.max_seq = 0
        self.appended_tokens = 0
        self.page_evictions = 0
        self.rewritten_tokens = 0
        self.rewritten_pages = 0
        self.evicted_pairs: Set[Tuple[int, int]] = set()

    # ---------------------------------------------------------------- statistics
    @property
    def page_count(self) -> int:
        return len(self.order)

    @property
    def open_pages(self) -> int:
        return sum(1 for s in self.order if self.pages[s] is not None and not self.pages[s].sealed)

    @property
    def group(self) -> int:
        return int4_group(self.head_dim, self.int4_group_size)

    # ---------------------------------------------------------------- quantisation
    def quantize_chunk(self, k: np.ndarray, v: np.ndarray, precision: str):
        """Row-local payloads of one chunk ``[B,H,T,D]`` (paged_kv_store.py:189-210)."""
        if precision == "fp32":
            return k.astype(np.float32).copy(), v.astype(np.float32).copy(), None, None
        if precision == "fp16":
            with np.errstate(over="ignore"):
                return k.astype(np.float16), v.astype(np.float16), None, None
        if precision == "int8":
            qk, sk = quantize_int8(k)
            qv, sv = quantize_int8(v)
            return qk, qv, sk, sv
        qk, sk = quantize_int4(k, self.group)
        qv, sv = quantize_int4(v, self.group)
        return pack_rows_lastdim(qk), pack_rows_lastdim(qv), sk, sv

    def decode(self, payload: np.ndarray, scale: Optional[np.ndarray], precision: str) -> np.ndarray:
        """One page payload -> fp32 ``[B,H,T,D]`` (paged_kv_store.py:376-402)."""
        if precision in ("fp32", "fp16"):
            return payload.astype(np.float32)
        if precision == "int8":
            return payload.astype(np.float32) * scale
        hi = (payload >> 4) & 0x0F
        lo = payload & 0x0F
        inter = np.stack([hi, lo], axis=-1).reshape(*payload.shape[:-1], -1)
        codes = inter[..., : self.head_dim].astype(np.int16) - 8
        g = self.group
        vals = codes.astype(np.float32).reshape(*codes.shape[:-1], self.head_dim // g, g) * scale
        return vals.reshape(*vals.shape[:-2], -1).astype(np.float32)

    # ---------------------------------------------------------------- validation
    def validate_against(self, batch: int, heads: int, head_dim: int) -> None:
        """paged_kv_store.py:141-147."""
        if batch != self.batch_size or heads != self.num_heads or head_dim != self.head_dim:
            raise ValueError("PagedKVStore shape mismatch")

    def _validate(self, k: np.ndarray, v: np.ndarray, precision: str, what: str) -> None:
        """paged_kv_store.py:149-183 / :450-487 (shape checks)."""
        if precision not in PRECISIONS:
            raise ValueError(f"Unsupported page precision: {precision}")
        if k.ndim != 4 or v.ndim != 4:
            raise ValueError("k_new/v_new must be 4-D")
        if k.shape != v.shape:
            raise ValueError("k_new/v_new shapes disagree")
        if k.shape[0] != self.batch_size or k.shape[1] != self.num_heads or k.shape[3] != self.head_dim:
            raise ValueError(f"PagedKVStore {what} shape mismatch")

    # ---------------------------------------------------------------- append
    def _open_slot(self, precision: str) -> Optional[int]:
        """Tail slot that still takes ``precision`` tokens; a precision change seals it (:309-320)."""
        if not self.order:
            return None
        slot = self.order[-1]
        page = self.pages[slot]
        if page is None or page.sealed:
            return None
        if page.precision != precision:
            page.sealed = True
            return None
        return slot

    def _alloc_slot(self) -> int:
        if self.free_slots:
            return self.free_slots.pop()
        self.pages.append(None)
        return len(self.pages) - 1

    def append(self, k: np.ndarray, v: np.ndarray, precision: str) -> None:
        """paged_kv_store.py:248-307."""
        self._validate(k, v, precision, "append")
        tokens = int(k.shape[2])
        if tokens == 0:
            return
        cursor = 0
        while cursor < tokens:
            slot = self._open_slot(precision)
            cap = self.page_size if slot is None else self.page_size - self.pages[slot].num_tokens
            take = min(cap, tokens - cursor)
            qk, qv, sk, sv = self.quantize_chunk(k[:, :, cursor:cursor + take], v[:, :, cursor:cursor + take],
                                                 precision)
            if slot is None:
                slot = self._alloc_slot()
                self.order.append(slot)
                self.pages[slot] = OraclePage(precision, qk, qv, sk, sv, self.max_seq, take, take == self.page_size)
            else:
                p = self.pages[slot]
                cat = lambda a, b: None if a is None or b is None else np.concatenate([a, b], axis=2)  # noqa: E731
                n = p.num_tokens + take
                self.pages[slot] = OraclePage(precision, cat(p.k, qk), cat(p.v, qv), cat(p.scale_k, sk),
                                              cat(p.scale_v, sv), p.start_token, n, n == self.page_size)
            cursor += take
            self.max_seq += take
        self.appended_tokens += tokens

    # ---------------------------------------------------------------- gather
    def gather(self) -> Tuple[np.ndarray, np.ndarray]:
        """Dense fp32 ``[B,H,S,D]``; S = last end when the pages tile [0, end), else max_seq
        with zero rows in the holes (paged_kv_store.py:326-374)."""
        B, H, D = self.batch_size, self.num_heads, self.head_dim
        if not self.order:
            z = np.zeros((B, H, 0, D), dtype=np.float32)
            return z, z.copy()
        pieces = []
        expected, contiguous = 0, True
        for slot in self.order:
            p = self.pages[slot]
            if p is None:
                contiguous = False
                continue
            if p.start_token != expected:
                contiguous = False
            expected = p.end_token
            pieces.append((p.start_token, self.decode(p.k, p.scale_k, p.precision),
                           self.decode(p.v, p.scale_v, p.precision)))
        if contiguous:
            return (np.concatenate([x[1] for x in pieces], axis=2),
                    np.concatenate([x[2] for x in pieces], axis=2))
        ko = np.zeros((B, H, self.max_seq, D), dtype=np.float32)
        vo = np.zeros_like(ko)
        for start, kp, vp in pieces:
            ko[:, :, start:start + kp.shape[2]] = kp
            vo[:, :, start:start + vp.shape[2]] = vp
        return ko, vo

    # ---------------------------------------------------------------- rewrite
    def rewrite_tokens(self, start_token: int, k: np.ndarray, v: np.ndarray, precision: str) -> int:
        """In-place re-quantisation of rows [start, start+T); all checks before any write
        (paged_kv_store.py:408-527)."""
        start = int(start_token)
        self._validate(k, v, precision, "rewrite")
        tokens = int(k.shape[2])
        if tokens < 1:
            raise ValueError("rewrite interval must cover at least one token")
        if start < 0 or start + tokens > self.max_seq:
            raise ValueError("rewrite interval exceeds stored range")
        end = start + tokens
        hits, covered = [], 0
        for slot in self.order:
            p = self.pages[slot]
            if p is None:
                continue
            a, b = max(start, p.start_token), min(end, p.end_token)
            if a >= b:
                continue
            if p.precision != precision:
                raise ValueError("rewrite precision does not match hit page")
            hits.append((p, a, b))
            covered += b - a
        if covered != end - start:
            raise ValueError("rewrite interval is not fully covered by pages")
        evicted_tokens = {t for t, _ in self.evicted_pairs}
        if any(t in evicted_tokens for t in range(start, end)):
            raise ValueError("rewrite interval contains an evicted token")
        payloads = [self.quantize_chunk(k[:, :, a - start:b - start], v[:, :, a - start:b - start], precision)
                    for _, a, b in hits]
        for (p, a, b), (qk, qv, sk, sv) in zip(hits, payloads):
            i, j = a - p.start_token, b - p.start_token
            p.k[:, :, i:j] = qk
            p.v[:, :, i:j] = qv
            if p.scale_k is not None and sk is not None:
                p.scale_k[:, :, i:j] = sk
            if p.scale_v is not None and sv is not None:
                p.scale_v[:, :, i:j] = sv
        self.rewritten_tokens += end - start
        self.rewritten_pages += len(hits)
        return end - start

    # ---------------------------------------------------------------- accounting
    def data_plane_bytes(self) -> int:
        """paged_kv_store.py:533-543."""
        total = 0
        for slot in self.order:
            p = self.pages[slot]
            if p is None:
                continue
            for a in (p.k, p.v, p.scale_k, p.scale_v):
                if a is not None:
                    total += a.size * a.itemsize
        return total

    def resident_bytes(self) -> int:
        """data + 48 bytes per (b, h, token) + 16 per slot of the pool (paged_kv_store.py:545-554)."""
        data = self.data_plane_bytes()
        if not self.order:
            return 0
        tokens = sum(self.pages[s].num_tokens for s in self.order if self.pages[s] is not None)
        return data + 48 * self.batch_size * self.num_heads * tokens + 16 * len(self.pages)

    # ---------------------------------------------------------------- eviction
    def evict_tokens(self, pairs: Iterable[Tuple[int, int]]) -> int:
        """Token-head eviction: fully evicted tokens leave their page (which splits into runs of
        survivors), partially evicted ones keep their position with the evicted heads' rows
        zeroed (int4: 0x88 bytes); absent or already evicted pairs are not counted
        (paged_kv_store.py:560-692)."""
        pairs = set(pairs)
        if not pairs or not self.order:
            return 0
        removed = 0
        runs_by_slot: Dict[int, List[OraclePage]] = {}
        retired: Set[int] = set()
        for slot in list(self.order):
            p = self.pages[slot]
            if p is None:
                continue
            n_removed, runs = self._plan_eviction(p, pairs)
            if n_removed == 0:
                continue
            removed += n_removed
            self.page_evictions += 1
            if runs:
                runs_by_slot[slot] = runs
            else:
                retired.add(slot)
        if removed == 0:
            return 0
        for slot in retired:
            self.pages[slot] = None
            self.free_slots.append(slot)
        order: List[int] = []
        for slot in self.order:
            if slot in retired:
                continue
            runs = runs_by_slot.get(slot)
            if runs is None:
                order.append(slot)
                continue
            for i, rp in enumerate(runs):
                if i == 0:
                    self.pages[slot] = rp
                    order.append(slot)
                else:
                    s = self._alloc_slot()
                    self.pages[s] = rp
                    order.append(s)
        self.order = order
        return removed

    def _plan_eviction(self, page: OraclePage, pairs: Set[Tuple[int, int]]):
        removed = 0
        kept: List[bool] = []
        partial: Dict[int, List[int]] = {}
        for i in range(page.num_tokens):
            t = page.start_token + i
            ev = [h for h in range(self.num_heads) if (t, h) in pairs and (t, h) not in self.evicted_pairs]
            removed += len(ev)
            self.evicted_pairs.update((t, h) for h in ev)
            if len(ev) == self.num_heads:
                kept.append(False)
            else:
                kept.append(True)
                if ev:
                    partial[i] = ev
        if removed == 0:
            return 0, []
        runs: List[Tuple[int, int]] = []
        i, n = 0, page.num_tokens
        while i < n:
            if not kept[i]:
                i += 1
                continue
            j = i
            while j < n and kept[j]:
                j += 1
            runs.append((i, j))
            i = j
        out = []
        for r, (a, b) in enumerate(runs):
            k, v = page.k[:, :, a:b].copy(), page.v[:, :, a:b].copy()
            sk = None if page.scale_k is None else page.scale_k[:, :, a:b].copy()
            sv = None if page.scale_v is None else page.scale_v[:, :, a:b].copy()
            for row, heads in partial.items():
                if a <= row < b:
                    for h in heads:
                        fill = 0x88 if page.precision == "int4" else 0
                        k[:, h, row - a] = fill
                        v[:, h, row - a] = fill
            sealed = page.sealed or r < len(runs) - 1 or (b - a) == self.page_size
            out.append(OraclePage(page.precision, k, v, sk, sv, page.start_token + a, b - a, sealed))
        return removed, out


# ------------------------------------------------------------------------------------ state
def _digest(a: Optional[np.ndarray]) -> Optional[str]:
    if a is None:
        return None
    a = np.ascontiguousarray(a)
    h = hashlib.sha256()
    h.update(str(a.dtype).encode())
    h.update(str(tuple(a.shape)).encode())
    h.update(a.tobytes())
    return h.hexdigest()


def store_state(store: Any, to_np=np.asarray) -> Dict[str, Any]:
    """Observable state of a store (this oracle's or any object with the reference's attribute
    names): page layout in token order, slot pool, counters, ledgers, page-tensor digests."""
    order = getattr(store, "order", None)
    if order is None:
        order = store._order
    free = getattr(store, "free_slots", None)
    if free is None:
        free = store._free_slots
    layout, digests = [], []
    for slot in order:
        p = store.pages[slot]
        layout.append([int(slot), int(p.start_token), int(p.num_tokens), bool(p.sealed), p.precision])
        digests.append([_digest(None if getattr(p, name) is None else to_np(getattr(p, name)))
                        for name in ("k", "v", "scale_k", "scale_v")])
    return {
        "layout": layout, "pool": len(store.pages), "free": [int(s) for s in free],
        "max_seq": int(store.max_seq), "page_count": int(store.page_count), "open_pages": int(store.open_pages),
        "appended_tokens": int(store.appended_tokens), "page_evictions": int(store.page_evictions),
        "rewritten_tokens": int(store.rewritten_tokens), "rewritten_pages": int(store.rewritten_pages),
        "data_plane_bytes": int(store.data_plane_bytes()), "resident_bytes": int(store.resident_bytes()),
        "page_digests": digests,
    }


def gather_digests(k: Any, v: Any, to_np=np.asarray) -> List[str]:
    return [_digest(to_np(k)), _digest(to_np(v))]
