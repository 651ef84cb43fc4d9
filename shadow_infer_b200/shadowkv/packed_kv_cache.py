"""Byte-level packed KV cache (drop-in for ``shadowinfer/shadowkv/packed_kv_cache.py``).

Same class, methods, ``packed_data`` schema and byte accounting as the
reference ``PackedKVCache``; every data-plane operation is one or two sm_100a
kernels behind the C ABI:

============================  ===============================  ======================
reference method              kernel(s)                        reference lines
============================  ===============================  ======================
``pack`` (plan or map)        skv_plan_bucket + skv_pack       packed_kv_cache.py:44-388
``unpack``                    skv_unpack                       :535-577, :636-656
``apply_reuse_mask``          skv_apply_reuse                  :753-854
``evict``                     skv_evict_count + _compact       :666-740
============================  ===============================  ======================

Per bucket the cache also keeps the device ``flat`` index list (``h*S+t`` in
bucket order) and one ``slot`` map (``int32 [S*H]``: ``(pos << 2) | code``, -1
when absent), so no operation rebuilds Python lists.  ``indices`` and
``byte_offsets`` in ``packed_data`` are materialised on first access.
Tensors stay on the device the caller packed from; host tensors are computed
on the current CUDA device and copied back.
"""

from __future__ import annotations

from typing import Any, Callable, Dict, List, Optional, Set, Tuple, Sequence

import torch

from .. import _lib
from .._device import back, compute_device, device_ctx, mask_u8, on, scratch
from .precision_plan import EVICTED, PRECISION_ORDER, PrecisionPlan, _entries, map_to_codes

_LAZY = object()
_CODE = {p: i for i, p in enumerate(PRECISION_ORDER)}


class _Bucket(dict):
    """One ``packed_data`` entry; ``indices`` / ``byte_offsets`` materialise on first read."""

    __slots__ = ("_resolvers",)

    def __init__(self, data: Dict[str, Any], resolvers: Dict[str, Callable[[], Any]]):
        dict.__init__(self, data)
        self._resolvers = dict(resolvers)
        for key in resolvers:
            dict.__setitem__(self, key, _LAZY)

    def set_lazy(self, key: str, fn: Callable[[], Any]) -> None:
        self._resolvers[key] = fn
        dict.__setitem__(self, key, _LAZY)

    def __getitem__(self, key):
        value = dict.__getitem__(self, key)
        if value is _LAZY:
            value = self._resolvers.pop(key)()
            dict.__setitem__(self, key, value)
        return value

    def get(self, key, default=None):
        return self[key] if dict.__contains__(self, key) else default

    def items(self):
        return [(k, self[k]) for k in dict.keys(self)]

    def values(self):
        return [self[k] for k in dict.keys(self)]

    def copy(self):
        return {k: self[k] for k in dict.keys(self)}

    def pop(self, key, *default):
        if dict.__contains__(self, key):
            value = self[key]
            dict.__delitem__(self, key)
            return value
        if default:
            return default[0]
        raise KeyError(key)

    def __eq__(self, other):
        return dict(self.items()) == (dict(other.items()) if isinstance(other, dict) else other)

    def __ne__(self, other):
        return not self.__eq__(other)

    __hash__ = None

    def __repr__(self):
        return repr(dict(self.items()))


def _int4_group(head_dim: int, group_size: int) -> int:
    if group_size < 1:
        raise ValueError(f"int4 group_size must be >= 1, got {group_size}")
    return group_size if head_dim % group_size == 0 else head_dim


_F32, _F16, _I8, _U8 = torch.float32, torch.float16, torch.int8, torch.uint8
_ALIGN = 256


def _bucket_parts(code: int, n: int, B: int, D: int, G: int):
    """(key, dtype, shape, bytes) of a bucket's tensors in the reference layout
    (packed_kv_cache.py:265-363); ``scale_*`` absent (None) for fp32 / fp16."""
    if code == 0:
        return (("k", _F32, (n, B, D), n * B * D * 4), ("v", _F32, (n, B, D), n * B * D * 4))
    if code == 1:
        return (("k", _F16, (n, B, D), n * B * D * 2), ("v", _F16, (n, B, D), n * B * D * 2))
    if code == 2:
        return (("k", _I8, (n, B, D), n * B * D), ("v", _I8, (n, B, D), n * B * D),
                ("scale_k", _F32, (n, B, 1), n * B * 4), ("scale_v", _F32, (n, B, 1), n * B * 4))
    rb = (B * D + 1) // 2
    ng = D // G
    return (("k", _U8, (n * rb,), n * rb), ("v", _U8, (n * rb,), n * rb),
            ("scale_k", _F32, (n * B, ng, 1), n * B * ng * 4), ("scale_v", _F32, (n * B, ng, 1), n * B * ng * 4))


def _nbytes(t: Optional[torch.Tensor]) -> int:
    return 0 if t is None else t.numel() * t.element_size()


# Slab bytes to try for the next pack of a shape, per (device, B, H, S, D, int4 group): the last
# exact layout plus an eighth, so that packing launches before the plan's counts reach the host.
_SLAB_HINT: Dict[Tuple[int, int, int, int, int, int], int] = {}


def _slab_layout(counts: Sequence[int], B: int, D: int, G: int):
    """Per code: None or ((key, dtype, shape, offset, bytes), ...); and the slab bytes.  The
    arithmetic of the library's slab_layout (each tensor at a 256-byte boundary)."""
    layout = []
    total = 0
    for code in range(4):
        n = counts[code]
        if n == 0:
            layout.append(None)
            continue
        parts = []
        for key, dt, shape, nb in _bucket_parts(code, n, B, D, G):
            parts.append((key, dt, shape, total, nb))
            total += (nb + _ALIGN - 1) // _ALIGN * _ALIGN
        layout.append(parts)
    return layout, total


def _slab_views(slab: torch.Tensor, layout, counts: Sequence[int], plan: PrecisionPlan):
    """Bucket dicts of typed views into ``slab`` for ``layout``."""
    typed: Dict[torch.dtype, torch.Tensor] = {}
    buckets: List[Optional[Dict[str, Any]]] = []
    start = 0
    flat_all = plan._flat_all
    for code in range(4):
        parts = layout[code]
        n = counts[code]
        if parts is None:
            buckets.append(None)
            start += n
            continue
        b: Dict[str, Any] = {"scale_k": None, "scale_v": None}
        for key, dt, shape, off, nb in parts:
            t = typed.get(dt)
            if t is None:
                t = typed[dt] = slab.view(dt)
            es = t.element_size()
            stride = (shape[1] * shape[2], shape[2], 1) if len(shape) == 3 else (1,)
            b[key] = t.as_strided(shape, stride, off // es)
        b["flat"] = flat_all[start:start + n]
        b["count"] = n
        start += n
        buckets.append(b)
    return buckets


def _slab_buckets(counts: Sequence[int], B: int, D: int, G: int, dev: torch.device,
                  skip: Sequence[bool] = (False,) * 4) -> List[Optional[Dict[str, Any]]]:
    """Empty buckets of ``counts`` entries (None where a count is 0 or ``skip`` is set), every
    tensor -- payload, scales and the int64 flat indices -- a view into ONE allocation, so that
    sizing new buckets costs one allocator call instead of five per bucket."""
    want = [0 if skip[c] else int(counts[c]) for c in range(4)]
    layout, total = _slab_layout(want, B, D, G)
    flat_off = total
    total += sum(want) * 8
    slab = torch.empty(max(total, 1), dtype=torch.uint8, device=dev)
    typed: Dict[torch.dtype, torch.Tensor] = {}
    flat_all = slab[flat_off:flat_off + sum(want) * 8].view(torch.int64)
    buckets: List[Optional[Dict[str, Any]]] = []
    start = 0
    for code in range(4):
        parts = layout[code]
        if parts is None:
            buckets.append(None)
            continue
        b: Dict[str, Any] = {"scale_k": None, "scale_v": None}
        for key, dt, shape, off, nb in parts:
            t = typed.get(dt)
            if t is None:
                t = typed[dt] = slab.view(dt)
            es = t.element_size()
            stride = (shape[1] * shape[2], shape[2], 1) if len(shape) == 3 else (1,)
            b[key] = t.as_strided(shape, stride, off // es)
        n = want[code]
        b["flat"] = flat_all[start:start + n]
        b["count"] = n
        start += n
        buckets.append(b)
    return buckets


class _SlabFlat:
    """The int64 flat indices of a slab's buckets, in bucket order (what ``_slab_views`` and
    ``_bucket_array`` read from a plan's ``_flat_all``)."""
    __slots__ = ("_flat_all",)

    def __init__(self, flat_all: torch.Tensor):
        self._flat_all = flat_all


def _empty_slab(counts: Sequence[int], B: int, D: int, G: int, dev: torch.device):
    """One allocation for buckets of ``counts`` entries (payload, scales, then the flat indices)
    and its ``skv_bucket[4]`` array, without making any tensor views: (slab, layout, flat
    holder, array).  The views come later from ``_slab_views`` (``_materialise``)."""
    layout, total = _slab_layout(counts, B, D, G)
    n = sum(counts)
    slab = torch.empty(max(total + n * 8, 1), dtype=torch.uint8, device=dev)
    flat = _SlabFlat(slab[total:total + n * 8].view(torch.int64))
    return slab, layout, flat, _bucket_array(slab.data_ptr(), layout, counts, flat)


def _bucket_array(slab_base: int, layout, counts: Sequence[int], plan: PrecisionPlan):
    arr = _lib.Buckets4()
    flat_base = plan._flat_all.data_ptr()
    start = 0
    for code in range(4):
        parts = layout[code]
        n = counts[code]
        if parts is not None:
            a = [slab_base + off for _, _, _, off, _ in parts]
            arr[code] = _lib.SkvBucket(a[0], a[1], a[2] if len(a) > 2 else None, a[3] if len(a) > 2 else None,
                                       flat_base + 8 * start, n)
        start += n
    return arr


def run_pack(k: torch.Tensor, v: torch.Tensor, plan: PrecisionPlan, group_size: int, dense: bool = False,
             k_prev: Optional[torch.Tensor] = None, v_prev: Optional[torch.Tensor] = None,
             events: Optional[Tuple[Any, Any]] = None, want_arr: bool = False,
             ):
    """Launch ``skv_pack`` for ``plan``; returns device buckets (+ dense working copy), and with
    ``want_arr`` also the ``skv_bucket[4]`` array of those buckets (see ``pack_slab``)."""
    slab, layout, counts, arr, dk, dv = pack_slab(k, v, plan, group_size, dense, k_prev, v_prev, events)
    buckets = _slab_views(slab, layout, counts, plan)
    if want_arr:
        return buckets, dk, dv, arr
    return buckets, dk, dv


def pack_slab(k: torch.Tensor, v: torch.Tensor, plan: PrecisionPlan, group_size: int, dense: bool = False,
              k_prev: Optional[torch.Tensor] = None, v_prev: Optional[torch.Tensor] = None,
              events: Optional[Tuple[Any, Any]] = None):
    """Launch ``skv_pack`` for ``plan``; returns ``(slab, layout, counts, skv_bucket[4], dense_k,
    dense_v)`` -- the buckets as one allocation and its layout (``_slab_layout``), no views.

    All buckets live in one allocation (each tensor 256-byte aligned in it).  When the plan's
    counts are still on their way to the host and a slab size is known for this shape, the
    kernel is launched at once on a layout the device computes from the counts
    (``skv_pack_slab``) and the host reads the counts while it runs; a slab that turns out too
    small receives nothing and the buckets are packed again into an exact one.  Otherwise the
    layout is computed here and the kernel gets it directly.  The typed tensor views are made
    by the caller (``_slab_views``) after the launch.  ``events``: optional pair of CUDA events
    recorded around the launch.
    """
    B, H, S, D = k.shape
    dev = plan.compute_device
    G = _int4_group(D, group_size)
    kd = on(k, dev, torch.float32)
    vd = on(v, dev, torch.float32)
    lib = _lib.load()
    key = (dev.index, B, H, S, D, G)
    hint = None
    if plan._counts is None and not dense and D in (64, 128, 256) and G % 16 == 0:
        hint = _SLAB_HINT.get(key)
    if hint is not None:
        slab = torch.empty(hint + _ALIGN, dtype=torch.uint8, device=dev)      # + the descriptors
        base = slab.data_ptr()
        with device_ctx(dev):
            if events is not None:
                events[0].record()
            st = lib.skv_pack_slab(_lib.ptr(kd), _lib.ptr(vd), B, H, S, D, group_size, _lib.ptr(plan.slot),
                                   _lib.ptr(plan.counts_device), _lib.ptr(plan._flat_all), base, hint, base + hint,
                                   _lib.stream_of(dev))
            if events is not None:
                events[1].record()
        _lib.check(st, "PackedKVCache.pack")
        counts = plan._host_counts()
        layout, total = _slab_layout(counts, B, D, G)
        _SLAB_HINT[key] = (total + total // 8 + _ALIGN - 1) // _ALIGN * _ALIGN or _ALIGN
        if total <= hint:
            return slab, layout, counts, _bucket_array(base, layout, counts, plan), None, None
        # the layout did not fit: the device wrote nothing; pack into an exact slab below
    counts = plan._host_counts()
    layout, total = _slab_layout(counts, B, D, G)
    _SLAB_HINT[key] = (total + total // 8 + _ALIGN - 1) // _ALIGN * _ALIGN or _ALIGN
    slab = torch.empty(max(total, _ALIGN), dtype=torch.uint8, device=dev)
    base = slab.data_ptr()
    arr = _bucket_array(base, layout, counts, plan)
    dk = dv = None
    kp = vp = None
    if dense:
        dk = torch.empty(B, H, S, D, dtype=torch.float32, device=dev)
        dv = torch.empty(B, H, S, D, dtype=torch.float32, device=dev)
        if k_prev is not None and plan.reuse_mask_device is not None:
            kp = on(k_prev, dev, torch.float32)
            vp = on(v_prev, dev, torch.float32)
    with device_ctx(dev):
        if events is not None:
            events[0].record()
        st = lib.skv_pack(_lib.ptr(kd), _lib.ptr(vd), B, H, S, D, group_size, _lib.ptr(plan.slot), arr,
                          _lib.ptr(dk), _lib.ptr(dv), _lib.ptr(kp), _lib.ptr(vp),
                          _lib.ptr(plan.reuse_mask_device) if kp is not None else None, _lib.stream_of(dev))
        if events is not None:
            events[1].record()
    _lib.check(st, "PackedKVCache.pack")
    return slab, layout, counts, arr, dk, dv


class PackedKVCache:
    """Byte-level packed KV cache storage with per-token-head precision."""

    PRECISION_BITS = {"fp32": 32, "fp16": 16, "int8": 8, "int4": 4}
    # optional (start, end) CUDA events recorded around every pack kernel launch (profiling hook)
    _pack_events: Optional[Tuple[Any, Any]] = None

    def __init__(self, batch_size: int, num_heads: int, seq_len: int, head_dim: int, device: Any = "cpu"):
        self.batch_size = batch_size
        self.num_heads = num_heads
        self.seq_len = seq_len
        self.head_dim = head_dim
        self.device = device
        self._packed_data: Dict[str, Dict[str, Any]] = {}
        # (slab, layout, counts, plan, group_size) of a pack whose packed_data views are not made yet
        self._pending = None
        self._memory_bytes = 0
        self._slot: Optional[torch.Tensor] = None       # device int32 [S*H]
        self._slot_owned = False
        self._flat: Dict[str, torch.Tensor] = {}         # device int64 per bucket
        self._count: Dict[str, int] = {}
        self._dev: Optional[torch.device] = None
        self._hidx: Optional[Tuple[torch.Tensor, torch.Tensor]] = None   # per-head row lists (attention)
        self._arr_cache = None     # (packed_data, dev, skv_bucket[4], device buckets, direct, snapshot)

    @property
    def packed_data(self) -> Dict[str, Dict[str, Any]]:
        """Per-precision bucket dicts (reference schema); after ``pack`` the tensor views into the
        bucket allocation are made on first access."""
        if self._pending is not None:
            self._materialise()
        return self._packed_data

    @packed_data.setter
    def packed_data(self, value: Dict[str, Dict[str, Any]]) -> None:
        self._pending = None
        self._packed_data = value
        self._arr_cache = None

    # ------------------------------------------------------------------------------ pack
    @classmethod
    def pack(
        cls,
        k_tensor: torch.Tensor,
        v_tensor: torch.Tensor,
        precision_map: Optional[Dict[int, Dict[int, str]]],
        group_size: int = 16,
        plan: Any = None,
        precomputed: Optional[Dict[str, Any]] = None,
    ) -> Dict[str, Any]:
        """Pack K/V ``[B, H, S, D]`` into byte-level buckets (packed_kv_cache.py:44-82).

        Returns ``{"packed_kv", "memory_bytes", "memory_mb"}``.  ``precomputed``
        is accepted for API compatibility; the fused kernel always quantises
        (the reference's precomputed payloads are bit-identical to it).
        """
        batch_size, num_heads, seq_len, head_dim = k_tensor.shape
        cache = cls(batch_size, num_heads, seq_len, head_dim, device=k_tensor.device)
        cache._do_pack(k_tensor, v_tensor, precision_map, group_size=group_size, plan=plan, precomputed=precomputed)
        return {"packed_kv": cache, "memory_bytes": cache.memory_bytes(), "memory_mb": cache.memory_mb()}

    def _do_pack(self, k_tensor, v_tensor, precision_map, group_size: int = 16, plan: Any = None,
                 precomputed: Optional[Dict[str, Any]] = None) -> None:
        """Map path: unknown precisions -> fp16, ``evicted`` skipped (packed_kv_cache.py:84-220)."""
        if plan is None:
            codes = map_to_codes(precision_map or {}, self.seq_len, self.num_heads, strict=False)
            plan = PrecisionPlan.from_codes(codes, device=k_tensor.device)
        self._do_pack_with_plan(k_tensor, v_tensor, plan, group_size, precomputed=precomputed)

    def _do_pack_with_plan(self, k_tensor, v_tensor, plan: Any, group_size: int,
                           precomputed: Optional[Dict[str, Any]] = None) -> None:
        """Plan-driven packing with the reference's validation (packed_kv_cache.py:222-365)."""
        batch_size, num_heads, seq_len, head_dim = k_tensor.shape
        if plan.seq_len != seq_len or plan.num_heads != num_heads:
            raise ValueError(
                "PrecisionPlan shape mismatch: plan "
                f"(seq_len={plan.seq_len}, num_heads={plan.num_heads}) vs "
                f"tensor (seq_len={seq_len}, num_heads={num_heads})"
            )
        if v_tensor.shape != k_tensor.shape:
            raise ValueError("k_tensor and v_tensor must have identical shapes")
        if plan.codes.device.type != k_tensor.device.type:
            raise ValueError(
                f"PrecisionPlan device ({plan.codes.device}) does not match KV device ({k_tensor.device})"
            )
        if not isinstance(plan, PrecisionPlan):
            plan = PrecisionPlan.from_codes(plan.codes, device=plan.codes.device)
        slab, layout, counts, arr, _, _ = pack_slab(k_tensor, v_tensor, plan, group_size, events=self._pack_events)
        self._adopt_pending(slab, layout, counts, plan, group_size, arr)

    def _adopt_pending(self, slab: torch.Tensor, layout, counts: Sequence[int], plan: PrecisionPlan,
                       group_size: int, arr) -> None:
        """Install a freshly packed slab: counts, bytes and the kernels' bucket array now, the
        ``packed_data`` views on first access (``_materialise``)."""
        self._dev = plan.slot.device
        self._slot = plan.slot
        self._slot_owned = False
        self._hidx = None
        self._packed_data = {}
        self._flat = {}
        self._count = {PRECISION_ORDER[c]: counts[c] for c in range(4) if counts[c]}
        self._memory_bytes = sum(nb for parts in layout if parts for _, _, _, _, nb in parts)
        self._pending = (slab, layout, counts, plan, group_size)
        self._arr_cache = (None, self._dev, arr, None, True, None)

    def _materialise(self) -> None:
        """Make the ``packed_data`` views of a pending slab (keeps the kernels' bucket array)."""
        slab, layout, counts, plan, group_size = self._pending
        self._pending = None
        arr = self._arr_cache[2]
        hidx = self._hidx
        self._adopt(_slab_views(slab, layout, counts, plan), self._slot, shared_slot=not self._slot_owned,
                    group_size=group_size, arr=arr)
        self._hidx = hidx

    def _adopt(self, buckets, slot: torch.Tensor, shared_slot: bool, group_size: int, arr=None) -> None:
        """Install device buckets as ``packed_data`` (on the cache's device); ``arr``: their
        ``skv_bucket[4]``, kept as the kernels' view when the payload stays on that device."""
        self._dev = slot.device
        self._slot = slot
        self._slot_owned = not shared_slot
        self._hidx = None
        self._arr_cache = None
        self._pending = None
        self._packed_data = {}
        self._flat = {}
        self._count = {}
        total = 0
        G = _int4_group(self.head_dim, group_size)
        for code, p in enumerate(PRECISION_ORDER):
            b = buckets[code]
            if b is None:
                continue
            self._flat[p] = b["flat"]
            self._count[p] = int(b["count"])
            data = {key: (None if b[key] is None else back(b[key], self.device))
                    for key in ("k", "v", "scale_k", "scale_v")}
            if code == 3:
                data["group_size"] = G
                data["num_groups"] = self.head_dim // G
            bucket = _Bucket(data, {"indices": self._indices_fn(p)})
            if code == 3:
                bucket.set_lazy("byte_offsets", self._offsets_fn(p))
            self.packed_data[p] = bucket
            for key in ("k", "v", "scale_k", "scale_v"):
                total += _nbytes(data[key])
        self._memory_bytes = total
        if arr is not None and all(b is None or all(b[x] is dict.__getitem__(self._packed_data[p], x)
                                                    for x in ("k", "v", "scale_k", "scale_v"))
                                   for p, b in zip(PRECISION_ORDER, buckets)):
            self._arr_cache = (self._packed_data, self._dev, arr, buckets, True, self._arr_snapshot())

    def _indices_fn(self, p: str) -> Callable[[], List[Tuple[int, int]]]:
        flat, S = self._flat[p], self.seq_len
        return lambda: _entries(flat, S)

    def _offsets_fn(self, p: str) -> Callable[[], List[Tuple[int, int, int, int]]]:
        n = self._count[p]
        rb = (self.batch_size * self.head_dim + 1) // 2
        return lambda: [(i * rb, (i + 1) * rb, i * rb, (i + 1) * rb) for i in range(n)]

    @staticmethod
    def _pack_int4_rows(quantized: torch.Tensor) -> Tuple[torch.Tensor, int]:
        """Row-wise int4 nibble packing of ``[n, ...]`` int8 codes (packed_kv_cache.py:367-388)."""
        if quantized.shape[0] == 0:
            return torch.empty(0, 0, dtype=torch.uint8, device=quantized.device), 0
        rows = quantized.reshape(quantized.shape[0], -1)
        off = (rows + 8).to(torch.uint8)
        if off.shape[1] % 2:
            off = torch.cat([off, torch.zeros(off.shape[0], 1, dtype=torch.uint8, device=off.device)], dim=1)
        packed = (off[:, 0::2] << 4) | (off[:, 1::2] & 0x0F)
        return packed, packed.shape[1]

    # ----------------------------------------------------------------------- device state
    def _ensure_state(self) -> torch.device:
        """Device slot/flat state, rebuilt from ``indices`` if the cache was filled by hand."""
        if self._slot is not None:
            return self._dev
        dev = compute_device(*[d.get("k") for d in self.packed_data.values()])
        slot = torch.full((self.seq_len * self.num_heads,), -1, dtype=torch.int32)
        for p, data in self.packed_data.items():
            idx = torch.tensor(list(data["indices"]), dtype=torch.int64).reshape(-1, 2)
            n = idx.shape[0]
            if n:
                slot[idx[:, 0] * self.num_heads + idx[:, 1]] = (torch.arange(n, dtype=torch.int32) << 2) | _CODE[p]
            self._flat[p] = (idx[:, 1] * self.seq_len + idx[:, 0]).to(dev)
            self._count[p] = n
        self._slot = slot.to(dev)
        self._slot_owned = True
        self._dev = dev
        return dev

    def _arr_snapshot(self):
        """(precision, bucket dict, ((key, tensor, address), ...)) of the current payload."""
        snap = []
        for p, d in self.packed_data.items():
            ts = []
            for x in ("k", "v", "scale_k", "scale_v"):
                t = dict.get(d, x)
                ts.append((x, t, None if t is None else t.data_ptr()))
            snap.append((p, d, tuple(ts)))
        return tuple(snap)

    def _arr_valid(self, snap) -> bool:
        """The payload is still the snapshot's: same buckets, tensor objects and addresses."""
        pd = self.packed_data
        if len(pd) != len(snap):
            return False
        for p, d, ts in snap:
            if pd.get(p) is not d:
                return False
            for x, t, a in ts:
                if dict.get(d, x) is not t or (t is not None and t.data_ptr() != a):
                    return False
        return True

    def _device_arr(self, dev: torch.device):
        """``skv_bucket[4]`` of this cache for ``dev`` plus a flag: True when the kernels work on
        the ``packed_data`` tensors themselves (no copy-back needed).  Cached while the payload
        (bucket dicts, tensor objects and their addresses) stays the same."""
        cached = self._arr_cache
        if self._pending is not None and cached is not None and cached[1] == dev:
            return cached[2], None, True                   # views not made yet: the pack's own array
        if cached is not None and cached[0] is self.packed_data and cached[1] == dev and self._arr_valid(cached[5]):
            return cached[2], cached[3], cached[4]
        bk = self._device_buckets(dev)
        direct = True
        for p, b in zip(PRECISION_ORDER, bk):
            if b is None:
                continue
            data = self.packed_data[p]
            direct &= all(b[x] is data[x] for x in ("k", "v", "scale_k", "scale_v"))
        arr = _lib.buckets(bk)
        self._arr_cache = (self.packed_data, dev, arr, bk, direct, self._arr_snapshot())
        return arr, bk, direct

    def _device_buckets(self, dev: torch.device) -> List[Optional[Dict[str, Any]]]:
        out: List[Optional[Dict[str, Any]]] = []
        for p in PRECISION_ORDER:
            data = self.packed_data.get(p)
            if data is None or self._count.get(p, 0) == 0:
                out.append(None)
                continue
            out.append({"k": on(data["k"], dev), "v": on(data["v"], dev),
                        "scale_k": on(data["scale_k"], dev), "scale_v": on(data["scale_v"], dev),
                        "flat": self._flat[p].to(dev), "count": self._count[p]})
        return out

    def _head_index(self, dev: torch.device) -> Tuple[torch.Tensor, torch.Tensor]:
        """Per-head stored-entry lists grouped by precision (built once per layout, ``skv_head_index``)."""
        if self._hidx is None:
            S, H = self.seq_len, self.num_heads
            rows = torch.empty(H * S, dtype=torch.int32, device=dev)
            counts = torch.empty(H * 5, dtype=torch.int32, device=dev)
            lib = _lib.load()
            with device_ctx(dev):
                st = lib.skv_head_index(_lib.ptr(self._slot.to(dev)), S, H, _lib.ptr(rows), _lib.ptr(counts),
                                        _lib.stream_of(dev))
            _lib.check(st, "PackedKVCache head index")
            self._hidx = (rows, counts)
        return self._hidx

    def _has_int4(self) -> bool:
        return "int4" in self._count if self._pending is not None else "int4" in self.packed_data

    def _has_buckets(self) -> bool:
        return bool(self._count) if self._pending is not None else bool(self.packed_data)

    def _int4_group_of(self) -> int:
        if self._pending is not None:
            return _int4_group(self.head_dim, self._pending[4]) if "int4" in self._count else self.head_dim
        d = self.packed_data.get("int4")
        return int(d["group_size"]) if d is not None else self.head_dim

    # ---------------------------------------------------------------------------- unpack
    def unpack(self) -> Tuple[torch.Tensor, torch.Tensor]:
        """Zero-filled float32 ``[B,H,S,D]`` K and V from all buckets (packed_kv_cache.py:535-577)."""
        shape = (self.batch_size, self.num_heads, self.seq_len, self.head_dim)
        if not (self._count if self._pending is not None else self.packed_data):
            k_out = torch.zeros(shape, dtype=torch.float32, device=self.device)
            return k_out, torch.zeros_like(k_out)
        dev = self._ensure_state()
        k_out = torch.empty(shape, dtype=torch.float32, device=dev)
        v_out = torch.empty(shape, dtype=torch.float32, device=dev)
        arr, _, _ = self._device_arr(dev)
        lib = _lib.load()
        with device_ctx(dev):
            st = lib.skv_unpack(arr, _lib.ptr(self._slot.to(dev)), self.batch_size, self.num_heads, self.seq_len,
                                self.head_dim, self._int4_group_of(), _lib.ptr(k_out), _lib.ptr(v_out),
                                _lib.stream_of(dev))
        _lib.check(st, "PackedKVCache.unpack")
        return back(k_out, torch.device(self.device)), back(v_out, torch.device(self.device))

    def unpack_reference(self) -> Tuple[torch.Tensor, torch.Tensor]:
        """Independent torch restatement of the per-entry golden unpack (packed_kv_cache.py:579-634).

        Kept for cross-checking ``unpack``; it uses plain torch indexing, not the kernels.
        """
        B, H, S, D = self.batch_size, self.num_heads, self.seq_len, self.head_dim
        k_out = torch.zeros(B, H, S, D, dtype=torch.float32, device=self.device)
        v_out = torch.zeros_like(k_out)
        for p, data in self.packed_data.items():
            idx = torch.tensor(list(data["indices"]), dtype=torch.int64, device=self.device).reshape(-1, 2)
            n = idx.shape[0]
            if n == 0:
                continue
            vals = []
            for key in ("k", "v"):
                x = data[key]
                if p in ("fp32", "fp16"):
                    y = x.float()
                elif p == "int8":
                    y = x.float() * data["scale_" + key]
                else:
                    rows = x.reshape(n, -1)
                    nib = torch.stack([(rows >> 4) & 0x0F, rows & 0x0F], dim=-1).reshape(n, -1)[:, : B * D]
                    g, ng = data["group_size"], data["num_groups"]
                    y = ((nib.to(torch.int16) - 8).float().reshape(n, B, ng, g)
                         * data["scale_" + key].reshape(n, B, ng, 1)).reshape(n, B, D)
                vals.append(y.permute(1, 0, 2))
            k_out[:, idx[:, 1], idx[:, 0], :] = vals[0]
            v_out[:, idx[:, 1], idx[:, 0], :] = vals[1]
        return k_out, v_out

    # ------------------------------------------------------------------------ accounting
    def memory_bytes(self) -> int:
        """Actual byte-level memory usage."""
        return self._memory_bytes

    def memory_mb(self) -> float:
        return self._memory_bytes / (1024.0 * 1024.0)

    def _compute_data_bytes(self) -> int:
        total = 0
        for data in self.packed_data.values():
            for key in ("k", "v", "scale_k", "scale_v"):
                total += _nbytes(data.get(key))
        return total

    def data_plane_bytes(self) -> int:
        """Tensor storage bytes only (packed_kv_cache.py:865-867)."""
        return self._compute_data_bytes()

    def resident_bytes(self) -> int:
        """Data bytes + 48 bytes of metadata per token-head (packed_kv_cache.py:869-878)."""
        if not self.packed_data:
            return 0
        n = 0
        for p, data in self.packed_data.items():
            n += self._count[p] if p in self._count else len(data["indices"])
        return self._compute_data_bytes() + 48 * n

    # ----------------------------------------------------------------------------- evict
    def evict(self, token_head_set: Any) -> int:
        """Remove token-heads from their buckets, keeping order (packed_kv_cache.py:666-740).

        ``token_head_set``: set of ``(t, h)`` or a bool ``[S, H]`` mask.  Returns
        the number of entries removed; buckets that become empty are deleted.
        """
        if token_head_set is None:
            return 0
        if not torch.is_tensor(token_head_set) and not token_head_set:
            return 0
        if self._pending is not None:
            if not self._count:
                return 0
            removed = self._evict_pending(token_head_set)
            if removed is not None:
                return removed
        if not self.packed_data:
            return 0
        dev = self._ensure_state()
        mask = self._entry_mask(token_head_set, dev)
        src = self._device_buckets(dev)
        lib = _lib.load()
        max_n = max([b["count"] for b in src if b is not None] + [0])
        scr = scratch(lib.skv_evict_scratch_bytes(max_n), dev)
        kept_d = torch.empty(5, dtype=torch.int64, device=dev)
        src_arr = _lib.buckets(src)
        stream = _lib.stream_of(dev)
        with device_ctx(dev):
            st = lib.skv_evict_count(src_arr, _lib.ptr(mask), self.seq_len, self.num_heads, _lib.ptr(kept_d),
                                     _lib.ptr(scr), scr.numel(), stream)
        _lib.check(st, "PackedKVCache.evict")
        kept = [int(x) for x in kept_d.tolist()]
        removed = kept[4]
        if removed == 0:
            return 0
        if not self._slot_owned:
            self._slot = self._slot.clone()
            self._slot_owned = True
        self._hidx = None
        self._arr_cache = None
        G = self._int4_group_of()
        # untouched buckets (dst.count == src.count) stay as they are; the others get new
        # buckets, all in one allocation
        same = [src[c] is None or kept[c] == src[c]["count"] for c in range(4)]
        fresh = _slab_buckets(kept[:4], self.batch_size, self.head_dim, G, dev, skip=same)
        dst: List[Optional[Dict[str, Any]]] = [src[c] if same[c] else fresh[c] for c in range(4)]
        work: List[Optional[Dict[str, Any]]] = [None if same[c] else src[c] for c in range(4)]
        with device_ctx(dev):
            st = lib.skv_evict_compact(src_arr, _lib.buckets(dst), _lib.ptr(mask), _lib.ptr(self._slot),
                                       self.batch_size, self.seq_len, self.num_heads, self.head_dim, G,
                                       _lib.ptr(scr), scr.numel(), stream)
        _lib.check(st, "PackedKVCache.evict")
        for code, p in enumerate(PRECISION_ORDER):
            if work[code] is None:
                continue
            if dst[code] is None:
                del self.packed_data[p]
                del self._flat[p]
                del self._count[p]
                continue
            nb = dst[code]
            data = self.packed_data[p]
            for key in ("k", "v", "scale_k", "scale_v"):
                dict.__setitem__(data, key, None if nb[key] is None else back(nb[key], torch.device(self.device)))
            self._flat[p] = nb["flat"]
            self._count[p] = nb["count"]
            data.set_lazy("indices", self._indices_fn(p)) if isinstance(data, _Bucket) else None
            if isinstance(data, _Bucket) and p == "int4":
                data.set_lazy("byte_offsets", self._offsets_fn(p))
        self._memory_bytes = self._compute_data_bytes()
        return removed

    def _evict_pending(self, token_head_set: Any) -> Optional[int]:
        """``evict`` of a cache whose ``packed_data`` views are not made yet: the pack's own bucket
        array is the source and the survivors are installed directly, so the views of the buckets
        being replaced are never built.  Returns None (nothing changed) when a stored bucket loses
        no entry -- the general path then keeps that bucket as it is."""
        dev = self._dev
        slab, layout, counts, plan, group_size = self._pending
        src_arr = self._arr_cache[2]
        mask = self._entry_mask(token_head_set, dev)
        lib = _lib.load()
        scr = scratch(lib.skv_evict_scratch_bytes(max(counts[:4])), dev)
        kept_d = torch.empty(5, dtype=torch.int64, device=dev)
        stream = _lib.stream_of(dev)
        with device_ctx(dev):
            st = lib.skv_evict_count(src_arr, _lib.ptr(mask), self.seq_len, self.num_heads, _lib.ptr(kept_d),
                                     _lib.ptr(scr), scr.numel(), stream)
        _lib.check(st, "PackedKVCache.evict")
        kept = kept_d.tolist()
        if kept[4] == 0:
            return 0
        if any(0 < kept[c] == counts[c] for c in range(4)):
            return None
        if not self._slot_owned:
            self._slot = self._slot.clone()
            self._slot_owned = True
        G = _int4_group(self.head_dim, group_size)
        want = [kept[c] if counts[c] else 0 for c in range(4)]
        new_slab, new_layout, flat, dst_arr = _empty_slab(want, self.batch_size, self.head_dim, G, dev)
        with device_ctx(dev):
            st = lib.skv_evict_compact(src_arr, dst_arr, _lib.ptr(mask), _lib.ptr(self._slot),
                                       self.batch_size, self.seq_len, self.num_heads, self.head_dim, G,
                                       _lib.ptr(scr), scr.numel(), stream)
        _lib.check(st, "PackedKVCache.evict")
        # the survivors' slab replaces the pack's, its views again made on first access
        self._hidx = None
        self._packed_data = {}
        self._flat = {}
        self._count = {PRECISION_ORDER[c]: want[c] for c in range(4) if want[c]}
        self._memory_bytes = sum(nb for parts in new_layout if parts for _, _, _, _, nb in parts)
        self._pending = (new_slab, new_layout, want, flat, group_size)
        self._arr_cache = (None, self._dev, dst_arr, None, True, None)
        return kept[4]

    def _entry_mask(self, entries: Any, dev: torch.device) -> torch.Tensor:
        S, H = self.seq_len, self.num_heads
        if torch.is_tensor(entries):
            fast = mask_u8(entries.detach(), S, H, dev)
            if fast is not None:
                return fast
            m = torch.zeros(S, H, dtype=torch.uint8, device=dev)
            s, h = min(S, entries.shape[0]), min(H, entries.shape[1])
            m[:s, :h] = on(entries[:s, :h], dev).to(torch.uint8)
            return m
        keys = [(int(t), int(h)) for (t, h) in entries if 0 <= t < S and 0 <= h < H]
        m = torch.zeros(S * H, dtype=torch.uint8)
        if keys:
            idx = torch.tensor(keys, dtype=torch.int64)
            m[idx[:, 0] * H + idx[:, 1]] = 1
        return m.view(S, H).to(dev, non_blocking=True)

    def _precision_for(self, token_idx: int, head_idx: int) -> str:
        """Bucket holding ``(t, h)``; missing entries are evicted (packed_kv_cache.py:742-751)."""
        if not self.packed_data or not (0 <= token_idx < self.seq_len and 0 <= head_idx < self.num_heads):
            return EVICTED
        self._ensure_state()
        s = int(self._slot[token_idx * self.num_heads + head_idx].item())
        return EVICTED if s < 0 else PRECISION_ORDER[s & 3]

    # ----------------------------------------------------------------------------- reuse
    def apply_reuse_mask(
        self,
        kv_previous_packed: "PackedKVCache",
        reuse_mask: Any,
        return_stats: bool = False,
    ) -> Optional[Dict[str, int]]:
        """Copy same-precision reused rows from the previous cache (packed_kv_cache.py:753-854).

        ``reuse_mask``: ``{(t, h): bool}`` or a bool ``[S, H]`` tensor.
        Cross-precision entries keep their values and count as ``skipped_precision``.
        """
        prev = kv_previous_packed
        if (self.batch_size != prev.batch_size or self.num_heads != prev.num_heads
                or self.head_dim != prev.head_dim):
            raise ValueError(
                "packed cache shape mismatch for reuse: "
                f"current=({self.batch_size},{self.num_heads},{self.head_dim}) "
                f"previous=({prev.batch_size},{prev.num_heads},{prev.head_dim})"
            )
        if self._has_int4() and prev._has_int4() and self._int4_group_of() != prev._int4_group_of():
            raise ValueError(
                "INT4 group_size mismatch for reuse: "
                f"current={self._int4_group_of()} previous={prev._int4_group_of()}"
            )
        stats = {"applied": 0, "skipped_precision": 0}
        empty_mask = reuse_mask is None or (not torch.is_tensor(reuse_mask) and not reuse_mask)
        if empty_mask or not prev._has_buckets() or not self._has_buckets():
            return stats if return_stats else None
        dev = self._ensure_state()
        prev._ensure_state()
        mask = self._entry_mask_from_reuse(reuse_mask, dev)
        cur_arr, cur_b, direct = self._device_arr(dev)
        prev_arr, _, _ = prev._device_arr(dev)
        stats_d = torch.empty(2, dtype=torch.int64, device=dev) if return_stats else None
        lib = _lib.load()
        with device_ctx(dev):
            st = lib.skv_apply_reuse(cur_arr, _lib.ptr(self._slot), self.seq_len, prev_arr,
                                     _lib.ptr(prev._slot.to(dev)), prev.seq_len, _lib.ptr(mask), self.batch_size,
                                     self.num_heads, self.head_dim, self._int4_group_of(), _lib.ptr(stats_d),
                                     _lib.stream_of(dev))
        _lib.check(st, "PackedKVCache.apply_reuse_mask")
        # write back when the payload lives elsewhere (host caches, non-contiguous views)
        for code, p in enumerate(PRECISION_ORDER if not direct else ()):
            b = cur_b[code]
            if b is None:
                continue
            data = self.packed_data[p]
            for key in ("k", "v", "scale_k", "scale_v"):
                orig = data[key]
                if orig is not None and b[key] is not orig:
                    orig.copy_(b[key].view(orig.shape))
        if not return_stats:
            return None
        a, s = stats_d.tolist()
        return {"applied": int(a), "skipped_precision": int(s)}

    def _entry_mask_from_reuse(self, reuse_mask: Any, dev: torch.device) -> torch.Tensor:
        if torch.is_tensor(reuse_mask):
            return self._entry_mask(reuse_mask, dev)
        return self._entry_mask([key for key, flag in reuse_mask.items() if flag], dev)

    def _invalidate_device_views(self) -> None:
        self._arr_cache = None

    def __repr__(self) -> str:
        return (
            f"PackedKVCache(batch={self.batch_size}, heads={self.num_heads}, "
            f"seq_len={self.seq_len}, head_dim={self.head_dim}, "
            f"memory_mb={self.memory_mb():.2f})"
        )
