"""Paged KV store (drop-in for ``shadowinfer/shadowkv/paged_kv_store.py``).

Same class, properties and semantics as the reference ``PagedKVStore``: one store per
layer, tokens kept in pages of at most ``page_size`` tokens of one precision, pages in
a slot pool (``pages``, with a free list) listed in token order, appends that only touch
the open tail page and new pages, ``gather`` back to dense fp32, in-place
``rewrite_tokens``, token-head ``evict_tokens`` that splits pages into runs of
survivors, and the reference's two byte ledgers.

Device layout.  A page's rows live in a slab ``[B, H, page_size, row]`` on the GPU that
is allocated once, when the page is opened (all pages one append opens share one
allocation), so appending to the open page writes the new rows in place instead of
concatenating.  ``skv_paged_write`` quantises the caller's rows straight into the
slabs (bit-identical to the reference's row-local ``Quantizer`` calls) and stores the
pages' descriptors into a device page table; ``gather`` is one ``skv_paged_gather``
launch over that table.  Eviction keeps survivor runs as views of their slab (no copy)
and zeroes partially evicted head rows with ``skv_paged_clear_heads``.  A page's
``k`` / ``v`` / ``scale_k`` / ``scale_v`` are views ``[B, H, num_tokens, ...]`` of its
slab, with the reference's dtypes and shapes.

The ledgers are the reference's: ``data_plane_bytes`` counts the rows the pages hold
(not the unused rows of an open slab, nor the rows of fully evicted tokens, whose slab
memory returns to the allocator when no page of that slab remains).
"""

from __future__ import annotations

import bisect
import ctypes
import operator
import struct
from typing import Any, Dict, List, Optional, Set, Tuple

import numpy as np
import torch

from .. import _lib
from .._device import as_device, compute_device, device_ctx, on

_PRECISIONS = ("fp32", "fp16", "int8", "int4")
_CODE = {"fp32": 0, "fp16": 1, "int8": 2, "int4": 3}
_PAYLOAD_DTYPE = {"fp32": torch.float32, "fp16": torch.float16, "int8": torch.int8, "int4": torch.uint8}
_PAYLOAD_BYTES = {"fp32": 4, "fp16": 2, "int8": 1, "int4": 1}
_RESIDENT_TOKEN_HEAD = 48          # metadata bytes per (batch, head, token) (paged_kv_store.py:545-554)
_RESIDENT_SLOT = 16                # page-table bytes per pool slot

_DESC = np.dtype([("k", "<u8"), ("v", "<u8"), ("scale_k", "<u8"), ("scale_v", "<u8"), ("start_token", "<i8"),
                  ("num_tokens", "<i4"), ("row_stride", "<i4"), ("precision", "<i4"), ("reserved", "<i4", (3,))])
_WRITE = np.dtype([("page", _DESC), ("src_token", "<i8"), ("dst_row", "<i4"), ("rows", "<i4"),
                   ("table_pos", "<i4"), ("reserved", "<i4")])
assert _DESC.itemsize == 64 and _WRITE.itemsize == 88
# the same records as flat structs (faster than numpy field access for a few records)
_DESC_S = struct.Struct("<QQQQqiiiiii")
_WRITE_S = struct.Struct("<QQQQqiiiiiiqiiii")
assert _DESC_S.size == 64 and _WRITE_S.size == 88


class _Chunk:
    """Slabs of the pages one append opens, in ONE device allocation: K and V payload
    ``[n, B, H, cap, row]`` and, for int8 / int4, fp32 scales ``[n, B, H, cap, 1]`` /
    ``[n, B, H, cap, G, 1]``, each part 256-byte aligned.  Base addresses and strides are
    kept on the host so page descriptors are plain arithmetic; the typed tensors are built
    only when a page's tensors are looked at."""

    __slots__ = ("buf", "parts", "ptr", "page_bytes", "row_bytes", "cap", "_t")

    def __init__(self, precision: str, n: int, B: int, H: int, P: int, D: int, groups: int,
                 dev: torch.device) -> None:
        dt = _PAYLOAD_DTYPE[precision]
        esz = _PAYLOAD_BYTES[precision]
        row = (D + 1) // 2 if precision == "int4" else D
        parts: List[Optional[Tuple[torch.dtype, Tuple[int, ...], int]]] = [(dt, (n, B, H, P, row), row * esz)] * 2
        if precision == "int8":
            parts += [(torch.float32, (n, B, H, P, 1), 4)] * 2
        elif precision == "int4":
            parts += [(torch.float32, (n, B, H, P, groups, 1), 4 * groups)] * 2
        else:
            parts += [None, None]
        offs, total = [], 0
        for part in parts:
            offs.append(total)
            if part is not None:
                total += -(-(n * B * H * P * part[2]) // 256) * 256
        self.buf = torch.empty(max(total, 256), dtype=torch.uint8, device=dev)
        base = self.buf.data_ptr()
        self.parts = [None if part is None else (part[0], part[1], off) for part, off in zip(parts, offs)]
        self.ptr = tuple(0 if part is None else base + off for part, off in zip(parts, offs))
        self.page_bytes = tuple(0 if part is None else B * H * P * part[2] for part in parts)
        self.row_bytes = tuple(0 if part is None else part[2] for part in parts)
        self.cap = P
        self._t: List[Optional[torch.Tensor]] = [None, None, None, None]

    def tensor(self, i: int) -> Optional[torch.Tensor]:
        """Part ``i`` (0 K, 1 V, 2 K scales, 3 V scales) as a typed tensor ``[n, B, H, cap, ...]``."""
        part = self.parts[i]
        if part is None:
            return None
        if self._t[i] is None:
            dt, shape, off = part
            nbytes = self.page_bytes[i] * shape[0]
            self._t[i] = self.buf[off:off + nbytes].view(dt).view(shape)
        return self._t[i]


class _Page:
    """One page of one precision (paged_kv_store.py:24-58).

    ``k`` / ``v`` / ``scale_k`` / ``scale_v`` are views of rows ``[row0, row0 + num_tokens)``
    of the page's slab (host copies, refreshed in place, when the store's device is the CPU).
    """

    __slots__ = ("precision", "start_token", "num_tokens", "sealed", "_chunk", "_idx", "_row0", "_host_device",
                 "_ver", "_host")


    def __init__(self, precision: str, chunk: _Chunk, idx: int, row0: int, start_token: int, num_tokens: int,
                 sealed: bool, host_device: Optional[torch.device]) -> None:
        self.precision = precision
        self._chunk = chunk
        self._idx = idx
        self._row0 = row0
        self.start_token = start_token
        self.num_tokens = num_tokens
        self.sealed = sealed
        self._host_device = host_device
        self._ver = 0
        self._host: Optional[List[Optional[Tuple[int, torch.Tensor]]]] = None

    @property
    def end_token(self) -> int:
        return self.start_token + self.num_tokens

    def _view(self, i: int) -> Optional[torch.Tensor]:
        t = self._chunk.tensor(i)
        if t is None:
            return None
        v = t[self._idx, :, :, self._row0:self._row0 + self.num_tokens]
        if self._host_device is None:
            return v
        if self._host is None:
            self._host = [None, None, None, None]
        cached = self._host[i]
        if cached is not None and cached[0] == self._ver:
            return cached[1]
        if cached is not None and cached[1].shape == v.shape:
            cached[1].copy_(v)                  # same buffer: data_ptr() stays put
            self._host[i] = (self._ver, cached[1])
        else:
            self._host[i] = (self._ver, v.to(self._host_device))
        return self._host[i][1]

    @property
    def k(self) -> torch.Tensor:
        return self._view(0)

    @property
    def v(self) -> torch.Tensor:
        return self._view(1)

    @property
    def scale_k(self) -> Optional[torch.Tensor]:
        return self._view(2)

    @property
    def scale_v(self) -> Optional[torch.Tensor]:
        return self._view(3)

    def _fields(self) -> Tuple[int, int, int, int, int, int, int, int]:
        """The ``skv_page_desc`` fields of the page's current rows: k, v, scale_k, scale_v,
        start_token, num_tokens, row_stride, precision."""
        c = self._chunk
        i, r = self._idx, self._row0
        p = c.ptr
        return (p[0] + i * c.page_bytes[0] + r * c.row_bytes[0], p[1] + i * c.page_bytes[1] + r * c.row_bytes[1],
                p[2] + i * c.page_bytes[2] + r * c.row_bytes[2] if p[2] else 0,
                p[3] + i * c.page_bytes[3] + r * c.row_bytes[3] if p[3] else 0,
                self.start_token, self.num_tokens, c.cap, _CODE[self.precision])


def _as_index(x: Any) -> Optional[int]:
    """``x`` as an int when it compares equal to one (the membership test of the reference)."""
    try:
        return operator.index(x)
    except TypeError:
        pass
    try:
        i = int(x)
    except (TypeError, ValueError, OverflowError):
        return None
    return i if i == x else None


class PagedKVStore:
    """Page-table-indirected KV storage with incremental appends (paged_kv_store.py:61-717)."""

    def __init__(
        self,
        batch_size: int,
        num_heads: int,
        head_dim: int,
        page_size: int = 32,
        device: Any = "cpu",
        int4_group_size: int = 16,
    ) -> None:
        if page_size < 1:
            raise ValueError(f"page_size must be >= 1, got {page_size}")
        if int4_group_size < 1:
            raise ValueError(f"int4_group_size must be >= 1, got {int4_group_size}")
        self.batch_size = int(batch_size)
        self.num_heads = int(num_heads)
        self.head_dim = int(head_dim)
        self.page_size = int(page_size)
        self.device = device
        self.int4_group_size = int(int4_group_size)
        self._dev = as_device(device)
        self._cdev: Optional[torch.device] = None      # compute (CUDA) device, fixed at first use
        self._table: Optional[torch.Tensor] = None     # device skv_page_desc [capacity] (uint8 view)
        self._flag: Optional[torch.Tensor] = None
        # optional (start, end) CUDA events recorded around each write / gather launch
        self._kernel_events: Optional[Tuple[Any, Any]] = None
        self._reset()

    def _reset(self) -> None:
        self.pages: List[Optional[_Page]] = []
        self._order: List[int] = []
        self._free_slots: List[int] = []
        self._max_seq = 0
        self._appended_tokens = 0
        self._page_evictions = 0
        self._rewritten_tokens = 0
        self._rewritten_pages = 0
        self._evicted_pairs: Set[Tuple[int, int]] = set()
        self._evicted_tokens: Set[int] = set()
        # gather geometry: do the pages tile [0, end) without holes, widest hole, longest page
        self._contiguous = True
        self._max_hole = 0
        self._max_rows = 0

    # ------------------------------------------------------------------ properties
    @property
    def max_seq(self) -> int:
        return self._max_seq

    @property
    def page_count(self) -> int:
        return len(self._order)

    @property
    def open_pages(self) -> int:
        return sum(1 for s in self._order if self.pages[s] is not None and not self.pages[s].sealed)

    @property
    def appended_tokens(self) -> int:
        return self._appended_tokens

    @property
    def page_evictions(self) -> int:
        return self._page_evictions

    @property
    def rewritten_tokens(self) -> int:
        return self._rewritten_tokens

    @property
    def rewritten_pages(self) -> int:
        return self._rewritten_pages

    @property
    def _int4_effective_group(self) -> int:
        return self.int4_group_size if self.head_dim % self.int4_group_size == 0 else self.head_dim

    # ------------------------------------------------------------------ validation
    def validate_against(self, batch: int, heads: int, head_dim: int) -> None:
        """Raise ValueError when the store shape does not match the model (paged_kv_store.py:141-147)."""
        if batch != self.batch_size or heads != self.num_heads or head_dim != self.head_dim:
            raise ValueError(
                "PagedKVStore shape mismatch: store="
                f"({self.batch_size},{self.num_heads},{self.head_dim}) vs "
                f"model=({batch},{heads},{head_dim})"
            )

    def _validate_rows(self, k_new: torch.Tensor, v_new: torch.Tensor, precision: str, what: str) -> None:
        """paged_kv_store.py:149-183 (append) / :450-487 (rewrite)."""
        if precision not in _PRECISIONS:
            raise ValueError(f"Unsupported page precision: {precision}")
        if k_new.dim() != 4 or v_new.dim() != 4:
            raise ValueError(
                "k_new/v_new must be 4-D [batch, heads, tokens, head_dim], got "
                f"k.dim={k_new.dim()}, v.dim={v_new.dim()}"
            )
        if k_new.shape != v_new.shape:
            raise ValueError(f"k_new/v_new shapes disagree: {tuple(k_new.shape)} vs {tuple(v_new.shape)}")
        if k_new.shape[0] != self.batch_size or k_new.shape[1] != self.num_heads or k_new.shape[3] != self.head_dim:
            raise ValueError(
                f"PagedKVStore {what} shape mismatch: expected "
                f"({self.batch_size},{self.num_heads},T,{self.head_dim}), got {tuple(k_new.shape)}"
            )

    # ------------------------------------------------------------------ device plumbing
    def _compute_device(self, *tensors: Optional[torch.Tensor]) -> torch.device:
        if self._cdev is None:
            if self._dev.type == "cuda":
                self._cdev = self._dev if self._dev.index is not None else compute_device()
            else:
                self._cdev = compute_device(*tensors)
        return self._cdev

    def _sources(self, k_new: torch.Tensor, v_new: torch.Tensor,
                 dev: torch.device) -> Tuple[torch.Tensor, torch.Tensor, int]:
        """K/V rows as the write kernel reads them: fp32 on ``dev`` with rows of D contiguous
        values and the (b, h) blocks at one common stride of ``T_src`` rows.  A token slice
        ``x[:, :, a:b]`` of a contiguous fp32 tensor qualifies as it is (no copy)."""
        D = self.head_dim
        B, H, T = int(k_new.shape[0]), int(k_new.shape[1]), int(k_new.shape[2])

        def rows_stride(t: torch.Tensor) -> Optional[int]:
            if t.dtype != torch.float32 or not t.is_cuda or t.get_device() != dev.index or t.data_ptr() % 16:
                return None
            st = t.stride()
            if st[3] != 1 or st[2] != D:
                return None
            if B * H == 1:
                return T
            s = st[0] if H == 1 else st[1]
            if H > 1 and B > 1 and st[0] != H * s:
                return None
            return s // D if s % D == 0 and s // D >= T else None

        k, v = k_new.detach(), v_new.detach()
        tk, tv = rows_stride(k), rows_stride(v)
        if tk is not None and tk == tv:
            return k, v, tk
        return on(k, dev, torch.float32), on(v, dev, torch.float32), T

    def _host_device(self) -> Optional[torch.device]:
        return None if self._dev.type == "cuda" else self._dev

    def _new_chunk(self, precision: str, n_pages: int, dev: torch.device) -> _Chunk:
        """Slabs of ``n_pages`` new pages (one allocation)."""
        return _Chunk(precision, n_pages, self.batch_size, self.num_heads, self.page_size, self.head_dim,
                      self.head_dim // self._int4_effective_group, dev)

    def _table_capacity(self, n: int, dev: torch.device) -> torch.Tensor:
        """The device page table, grown (contents kept) to hold ``n`` descriptors."""
        t = self._table
        if t is None or t.numel() < n * 64:
            cap = max(64, 1 << max(0, n - 1).bit_length())
            nt = torch.zeros(cap * 64, dtype=torch.uint8, device=dev)
            if t is not None:
                nt[:t.numel()].copy_(t)
            self._table = t = nt
        return t

    def _upload_table(self, dev: torch.device) -> None:
        """Rewrite the whole device page table from the page objects (after an eviction)."""
        n = len(self._order)
        table = self._table_capacity(max(n, 1), dev)
        if n == 0:
            return
        buf = bytearray(64 * n)
        for i, slot in enumerate(self._order):
            _DESC_S.pack_into(buf, 64 * i, *self.pages[slot]._fields(), 0, 0, 0)
        table[:n * 64].copy_(torch.frombuffer(buf, dtype=torch.uint8))

    def _launch_writes(self, k: torch.Tensor, v: torch.Tensor, t_src: int, writes: bytearray, dev: torch.device,
                       update_table: bool) -> None:
        """One ``skv_paged_write`` over ``writes`` (packed ``skv_page_write`` records)."""
        n = len(writes) // 88
        rec = (ctypes.c_char * len(writes)).from_buffer(writes)
        lib = _lib.load()
        table = self._table_capacity(len(self._order), dev) if update_table else None
        ev = self._kernel_events
        with device_ctx(dev):
            if ev is not None:
                ev[0].record()
            st = lib.skv_paged_write(_lib.ptr(k), _lib.ptr(v), self.batch_size, self.num_heads, t_src,
                                     self.head_dim, self.int4_group_size, ctypes.addressof(rec), n,
                                     _lib.ptr(table), _lib.stream_of(dev))
            if ev is not None:
                ev[1].record()
        _lib.check(st, "PagedKVStore write")

    def _recompute_geometry(self) -> None:
        self._contiguous, self._max_hole, self._max_rows = True, 0, 0
        end = 0
        for slot in self._order:
            p = self.pages[slot]
            hole = p.start_token - end
            if hole:
                self._contiguous = False
                self._max_hole = max(self._max_hole, hole)
            self._max_rows = max(self._max_rows, p.num_tokens)
            end = p.end_token

    # ------------------------------------------------------------------ append
    def _open_slot(self, precision: str) -> Optional[int]:
        """Tail slot that can still absorb ``precision`` tokens; a precision change seals it
        (paged_kv_store.py:309-320)."""
        if not self._order:
            return None
        slot = self._order[-1]
        page = self.pages[slot]
        if page is None or page.sealed:
            return None
        if page.precision != precision:
            page.sealed = True
            return None
        return slot

    def _alloc_slot(self) -> int:
        if self._free_slots:
            return self._free_slots.pop()
        self.pages.append(None)
        return len(self.pages) - 1

    def append(self, k_new: torch.Tensor, v_new: torch.Tensor, precision: str) -> None:
        """Append new tokens incrementally; sealed pages are never touched (paged_kv_store.py:248-307).

        The open tail page (same precision) takes what fits, then new pages of
        ``page_size`` tokens are opened at ``max_seq``; one write launch fills them all.
        """
        self._validate_rows(k_new, v_new, precision, "append")
        tokens = int(k_new.shape[2])
        if tokens == 0:
            return
        dev = self._compute_device(k_new, v_new)
        k, v, t_src = self._sources(k_new, v_new, dev)
        P = self.page_size
        slot = self._open_slot(precision)
        first = 0
        if slot is not None:
            page = self.pages[slot]
            first = min(P - page.num_tokens, tokens)
            if page._row0 + page.num_tokens + first > page._chunk.cap:
                self._relocate(page, dev)
        n_new = -(-(tokens - first) // P)
        writes = bytearray(88 * ((1 if first else 0) + n_new))
        if first:
            page = self.pages[slot]
            dst_row = page.num_tokens
            page.num_tokens += first
            page.sealed = page.num_tokens == P
            page._ver += 1
            _WRITE_S.pack_into(writes, 0, *page._fields(), 0, 0, 0, 0, dst_row, first, len(self._order) - 1, 0)
            self._max_rows = max(self._max_rows, page.num_tokens)
            self._max_seq += first
        if n_new:
            chunk = self._new_chunk(precision, n_new, dev)
            prev_end = self.pages[self._order[-1]].end_token if self._order else 0
            start0, pos0, code = self._max_seq, len(self._order), _CODE[precision]
            (pk, pv, psk, psv), (bk, bv, bsk, bsv) = chunk.ptr, chunk.page_bytes
            host = self._host_device()
            off = 88 if first else 0
            for i in range(n_new):
                take = min(P, tokens - first - i * P)
                s = self._alloc_slot()
                self._order.append(s)
                self.pages[s] = _Page(precision, chunk, i, 0, start0 + i * P, take, take == P, host)
                _WRITE_S.pack_into(writes, off + 88 * i, pk + i * bk, pv + i * bv, psk + i * bsk if psk else 0,
                                   psv + i * bsv if psv else 0, start0 + i * P, take, P, code, 0, 0, 0,
                                   first + i * P, 0, take, pos0 + i, 0)
            if start0 != prev_end:
                self._contiguous = False
                self._max_hole = max(self._max_hole, start0 - prev_end)
            self._max_rows = max(self._max_rows, min(P, tokens - first))
            self._max_seq += tokens - first
        self._launch_writes(k, v, t_src, writes, dev, update_table=True)
        self._appended_tokens += tokens

    def _relocate(self, page: _Page, dev: torch.device) -> None:
        """Give an open page (a survivor run that starts inside its slab) a slab of its own."""
        chunk = self._new_chunk(page.precision, 1, dev)
        n = page.num_tokens
        for i in range(4):
            src, dst = page._chunk.tensor(i), chunk.tensor(i)
            if src is not None:
                dst[0, :, :, :n].copy_(src[page._idx, :, :, page._row0:page._row0 + n])
        page._chunk, page._idx, page._row0 = chunk, 0, 0
        page._ver += 1

    # ------------------------------------------------------------------ gather
    def gather(self) -> Tuple[torch.Tensor, torch.Tensor]:
        """Rebuild dense float32 (k, v) in one pass over the page table (paged_kv_store.py:326-374).

        The result spans the last page's end when the pages tile ``[0, end)`` without a
        hole, else ``max_seq`` tokens with zeros where no page holds a token.
        """
        B, H, D = self.batch_size, self.num_heads, self.head_dim
        if not self._order:
            empty = torch.zeros(B, H, 0, D, dtype=torch.float32, device=self.device)
            return empty, empty.clone()
        dev = self._cdev
        last_end = self.pages[self._order[-1]].end_token
        s_out = last_end if self._contiguous else self._max_seq
        span = max(self._max_hole + self._max_rows, s_out - last_end)
        k_out = torch.empty(B, H, s_out, D, dtype=torch.float32, device=dev)
        v_out = torch.empty(B, H, s_out, D, dtype=torch.float32, device=dev)
        lib = _lib.load()
        ev = self._kernel_events
        with device_ctx(dev):
            if ev is not None:
                ev[0].record()
            st = lib.skv_paged_gather(_lib.ptr(self._table), len(self._order), B, H, D, self.int4_group_size, s_out,
                                      span, _lib.ptr(k_out), _lib.ptr(v_out), _lib.stream_of(dev))
            if ev is not None:
                ev[1].record()
        _lib.check(st, "PagedKVStore.gather")
        if self._dev.type != "cuda":
            return k_out.to(self._dev), v_out.to(self._dev)
        return k_out, v_out

    # ------------------------------------------------------------------ rewrite
    def rewrite_tokens(self, start_token: int, k_new: torch.Tensor, v_new: torch.Tensor, precision: str) -> int:
        """Overwrite token rows ``[start_token, start_token+T)`` in place (paged_kv_store.py:408-448).

        Rows are re-quantised exactly like an append of the same values; page layout and
        untouched rows never change; every check runs before the single write launch, so a
        refused call leaves the store untouched.  Returns the number of rewritten tokens.
        """
        start = int(start_token)
        self._validate_rows(k_new, v_new, precision, "rewrite")
        tokens = int(k_new.shape[2])
        if tokens < 1:
            raise ValueError(f"rewrite interval must cover at least one token, got {tokens}")
        if start < 0 or start + tokens > self._max_seq:
            raise ValueError(
                f"rewrite interval [{start},{start + tokens}) exceeds stored range [0,{self._max_seq})"
            )
        end = start + tokens
        hits = self._plan_rewrite(start, end, precision)
        dev = self._compute_device(k_new, v_new)
        k, v, t_src = self._sources(k_new, v_new, dev)
        writes = bytearray(88 * len(hits))
        for i, (page, a, b) in enumerate(hits):
            _WRITE_S.pack_into(writes, 88 * i, *page._fields(), 0, 0, 0, a - start, a - page.start_token, b - a, -1, 0)
            page._ver += 1
        self._launch_writes(k, v, t_src, writes, dev, update_table=False)
        self._rewritten_tokens += end - start
        self._rewritten_pages += len(hits)
        return end - start

    def _plan_rewrite(self, start: int, end: int, precision: str) -> List[Tuple[_Page, int, int]]:
        """Hit pages of ``[start, end)`` with the reference's refusals (paged_kv_store.py:489-527)."""
        hits: List[Tuple[_Page, int, int]] = []
        covered = 0
        for slot in self._order:
            page = self.pages[slot]
            if page is None:
                continue
            a, b = max(start, page.start_token), min(end, page.end_token)
            if a >= b:
                continue
            if page.precision != precision:
                raise ValueError(
                    f"rewrite precision does not match hit page: requested {precision}, page holds {page.precision}"
                )
            hits.append((page, a, b))
            covered += b - a
        if covered != end - start:
            raise ValueError(
                f"rewrite interval [{start},{end}) is not fully covered by pages "
                f"({covered} of {end - start} tokens); evicted holes cannot be rewritten"
            )
        if self._evicted_tokens:
            for token in range(start, end):
                if token in self._evicted_tokens:
                    raise ValueError(
                        f"rewrite interval [{start},{end}) contains evicted token {token}; "
                        "evicted positions cannot be rewritten"
                    )
        return hits

    # ------------------------------------------------------------------ accounting
    def _page_bytes(self, page: _Page) -> int:
        B, H, D = self.batch_size, self.num_heads, self.head_dim
        n = B * H * page.num_tokens
        p = page.precision
        if p == "fp32":
            return 2 * n * D * 4
        if p == "fp16":
            return 2 * n * D * 2
        if p == "int8":
            return 2 * n * D + 2 * n * 4
        return 2 * n * ((D + 1) // 2) + 2 * n * (D // self._int4_effective_group) * 4

    def data_plane_bytes(self) -> int:
        """Page tensor storage bytes (payload + scales) (paged_kv_store.py:533-543)."""
        return sum(self._page_bytes(self.pages[s]) for s in self._order if self.pages[s] is not None)

    def resident_bytes(self) -> int:
        """Data-plane bytes plus metadata and page-table overhead (paged_kv_store.py:545-554)."""
        if not self._order:
            return 0
        tokens = sum(self.pages[s].num_tokens for s in self._order if self.pages[s] is not None)
        return (self.data_plane_bytes() + _RESIDENT_TOKEN_HEAD * self.batch_size * self.num_heads * tokens
                + _RESIDENT_SLOT * len(self.pages))

    # ------------------------------------------------------------------ eviction
    def evict_tokens(self, token_head_set: Set[Tuple[int, int]]) -> int:
        """Evict token-heads page-locally; untouched pages are never re-packed (paged_kv_store.py:560-611).

        A token leaves its page only when all its heads are evicted (the page splits into
        runs of survivors); a partially evicted token keeps its position with the evicted
        heads' rows zeroed.  Returns the number of (token, head) pairs removed; absent or
        already evicted pairs are never counted and never revived.
        """
        if not token_head_set or not self._order:
            return 0
        H = self.num_heads
        want: Dict[int, List[int]] = {}
        for item in token_head_set:
            try:
                t, h = item
            except (TypeError, ValueError):
                continue
            t, h = _as_index(t), _as_index(h)
            if t is None or h is None or not 0 <= h < H or not 0 <= t < self._max_seq:
                continue
            want.setdefault(t, []).append(h)
        if not want:
            return 0
        tokens = sorted(want)
        removed = 0
        runs_by_slot: Dict[int, List[Tuple[_Page, Dict[int, List[int]]]]] = {}
        retired: Set[int] = set()
        for slot in list(self._order):
            page = self.pages[slot]
            if page is None:
                continue
            i0 = bisect.bisect_left(tokens, page.start_token)
            i1 = bisect.bisect_left(tokens, page.end_token)
            if i0 == i1:
                continue
            n_removed, runs = self._plan_eviction(page, tokens[i0:i1], want)
            if n_removed == 0:
                continue
            removed += n_removed
            self._page_evictions += 1
            if runs:
                runs_by_slot[slot] = runs
            else:
                retired.add(slot)
        if removed == 0:
            return 0
        for slot in retired:
            self.pages[slot] = None
            self._free_slots.append(slot)
        new_order: List[int] = []
        clears: List[Tuple[int, int, int]] = []
        for slot in self._order:
            if slot in retired:
                continue
            runs = runs_by_slot.get(slot)
            if runs is None:
                new_order.append(slot)
                continue
            for run_index, (run_page, partial) in enumerate(runs):
                s = slot if run_index == 0 else self._alloc_slot()
                self.pages[s] = run_page
                new_order.append(s)
                pos = len(new_order) - 1
                for row, heads in partial.items():
                    clears.extend((pos, row, h) for h in heads)
        self._order = new_order
        self._recompute_geometry()
        dev = self._cdev
        self._upload_table(dev)
        if clears:
            self._clear_heads(clears, dev)
        return removed

    def _plan_eviction(self, page: _Page, tokens: List[int], want: Dict[int, List[int]]):
        """Survivor runs of one page (paged_kv_store.py:620-692): (run page, {row: heads to zero})."""
        H = self.num_heads
        removed = 0
        full: List[int] = []
        partial: Dict[int, List[int]] = {}
        for t in tokens:
            heads = sorted({h for h in want[t] if (t, h) not in self._evicted_pairs})
            if not heads:
                continue
            removed += len(heads)
            self._evicted_pairs.update((t, h) for h in heads)
            self._evicted_tokens.add(t)
            if len(heads) == H:
                full.append(t - page.start_token)
            else:
                partial[t - page.start_token] = heads
        if removed == 0:
            return 0, []
        runs: List[Tuple[int, int]] = []
        i = 0
        for f in full + [page.num_tokens]:
            if f > i:
                runs.append((i, f))
            i = f + 1
        out = []
        host = self._host_device()
        for run_index, (a, b) in enumerate(runs):
            sealed = page.sealed or run_index < len(runs) - 1 or (b - a) == self.page_size
            run = _Page(page.precision, page._chunk, page._idx, page._row0 + a, page.start_token + a, b - a, sealed,
                        host)
            out.append((run, {row - a: hs for row, hs in partial.items() if a <= row < b}))
        return removed, out

    def _clear_heads(self, clears: List[Tuple[int, int, int]], dev: torch.device) -> None:
        items = torch.tensor(clears, dtype=torch.int32).reshape(-1, 3).to(dev)
        if self._flag is None:
            self._flag = torch.zeros(1, dtype=torch.int32, device=dev)
        lib = _lib.load()
        with device_ctx(dev):
            st = lib.skv_paged_clear_heads(_lib.ptr(self._table), len(self._order), _lib.ptr(items), len(clears),
                                           self.batch_size, self.num_heads, self.head_dim, _lib.ptr(self._flag),
                                           _lib.stream_of(dev))
        _lib.check(st, "PagedKVStore.evict_tokens")
        if int(self._flag.item()):
            raise RuntimeError("PagedKVStore.evict_tokens: a head row to clear lay outside its page")

    # ------------------------------------------------------------------ reset
    def clear(self) -> None:
        """Drop all pages and counters (paged_kv_store.py:694-704)."""
        self._reset()

    def __repr__(self) -> str:
        return (
            f"PagedKVStore(batch={self.batch_size}, heads={self.num_heads}, "
            f"head_dim={self.head_dim}, page_size={self.page_size}, "
            f"max_seq={self._max_seq}, pages={self.page_count})"
        )
