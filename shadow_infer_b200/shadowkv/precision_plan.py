"""Precision/reuse plan (drop-in for ``shadowinfer/shadowkv/precision_plan.py``).

``PrecisionPlan.from_codes`` buckets the ``int8 [seq, heads]`` precision codes
on the GPU (``skv_plan_bucket``: a tile-count pass and a scan + scatter pass,
no sort) into token-major buckets with head-major flat gather indices
``h*S + t``, exactly as the reference does with ``nonzero`` per code
(precision_plan.py:113-177).  The Python-object views of the plan (``groups``,
``evicted_entries``, ``reuse_entries``) and the SHA-256 ``fingerprint``
(precision_plan.py:179-190) are materialised on first access, so building a
plan costs one small device-to-host copy (the six bucket counts).
"""

from __future__ import annotations

import dataclasses
import hashlib
import struct
from typing import Any, Dict, List, Optional, Tuple

import torch

from .. import _lib
from .._device import as_device, compute_device, device_ctx, mask_u8, on

PRECISION_ORDER: Tuple[str, ...] = ("fp32", "fp16", "int8", "int4")
EVICTED = "evicted"
PRECISION_CODES: Dict[str, int] = {"fp32": 0, "fp16": 1, "int8": 2, "int4": 3, EVICTED: 4}
CODE_PRECISIONS: Dict[int, str] = {code: name for name, code in PRECISION_CODES.items()}


def map_to_codes(
    precision_map: Dict[int, Dict[int, str]],
    seq_len: int,
    num_heads: int,
    strict: bool = True,
    device: Any = "cpu",
) -> torch.Tensor:
    """``token -> head -> precision`` map to ``int8 [seq, heads]`` (precision_plan.py:30-55).

    Missing entries are ``fp16``; unsupported names raise ``ValueError`` when
    ``strict``, else become ``fp16``.
    """
    out = torch.full((seq_len, num_heads), PRECISION_CODES["fp16"], dtype=torch.int8)
    if seq_len > 0 and num_heads > 0:
        view = out.numpy()
        for t in range(seq_len):
            tmap = precision_map.get(t)
            if not tmap:
                continue
            for h in range(num_heads):
                if h not in tmap:
                    continue
                raw = tmap[h]
                p = raw.lower() if isinstance(raw, str) else raw
                code = PRECISION_CODES.get(p) if isinstance(p, str) else None
                if code is None:
                    if strict:
                        raise ValueError(f"Unsupported precision: {raw}")
                    code = PRECISION_CODES["fp16"]
                view[t, h] = code
    return out.to(device)


def codes_to_map(codes: torch.Tensor) -> Dict[int, Dict[int, str]]:
    """``int8 [seq, heads]`` codes back to a precision map (precision_plan.py:58-69)."""
    rows = codes.detach().to("cpu").to(torch.int64).tolist()
    out: Dict[int, Dict[int, str]] = {}
    for t, row in enumerate(rows):
        tmap: Dict[int, str] = {}
        for h, c in enumerate(row):
            if c not in CODE_PRECISIONS:
                raise ValueError(f"Unsupported precision code: {c}")
            tmap[h] = CODE_PRECISIONS[c]
        out[t] = tmap
    return out


def reuse_mask_tensor(reuse_mask: Any, seq_len: int, num_heads: int, dev: torch.device) -> Optional[torch.Tensor]:
    """Reuse flags as ``uint8 [seq, heads]`` on ``dev``; ``None`` when nothing is flagged.

    Accepts the reference's ``{(t, h): bool}`` dict (out-of-range keys are
    dropped, precision_plan.py:153-159) or a bool/uint8 ``[seq, heads]`` tensor.
    """
    if reuse_mask is None:
        return None
    if torch.is_tensor(reuse_mask):
        m = reuse_mask.detach()
        fast = mask_u8(m, seq_len, num_heads, dev)
        if fast is not None:
            return fast
        if m.dim() != 2:
            raise ValueError(f"reuse mask tensor must be 2-D [seq, heads], got {tuple(m.shape)}")
        full = torch.zeros(seq_len, num_heads, dtype=torch.uint8, device=dev)
        s, h = min(seq_len, m.shape[0]), min(num_heads, m.shape[1])
        full[:s, :h] = on(m[:s, :h], dev).to(torch.uint8)
        return full
    if not reuse_mask:
        return None
    keys = [(int(t), int(h)) for (t, h), flag in reuse_mask.items()
            if flag and 0 <= t < seq_len and 0 <= h < num_heads]
    full = torch.zeros(seq_len * num_heads, dtype=torch.uint8)
    if keys:
        idx = torch.tensor(keys, dtype=torch.int64)
        full[idx[:, 0] * num_heads + idx[:, 1]] = 1
    return full.view(seq_len, num_heads).to(dev, non_blocking=True)


# (pinned int64[6] host buffer, event) pairs for plan counts, returned here once read
_PINNED: List[Tuple[torch.Tensor, Any]] = []


def _entries(flat: torch.Tensor, seq_len: int) -> List[Tuple[int, int]]:
    f = flat.detach().to("cpu")
    return list(zip((f % seq_len).tolist(), torch.div(f, seq_len, rounding_mode="floor").tolist()))


class PrecisionPlan:
    """Immutable grouping/index plan shared by compress and pack (precision_plan.py:72-194).

    Public fields match the reference dataclass: ``seq_len``, ``num_heads``,
    ``codes``, ``groups``, ``flat_indices``, ``reuse_entries``, ``reuse_flat``,
    ``fingerprint``, ``evicted_entries``.  Tensors live on the plan's device;
    the bucketing itself always runs on the GPU.
    """

    __slots__ = ("_seq_len", "_num_heads", "_codes", "_device", "_dev", "_flat_all", "_counts", "_slot",
                 "_reuse_flat_dev", "_reuse_mask_dev", "_lazy", "_frozen", "_counts_dev", "_pending")

    def __init__(self, *args, **kwargs):
        raise TypeError("use PrecisionPlan.build(...) or PrecisionPlan.from_codes(...)")

    def __setattr__(self, name, value):
        if getattr(self, "_frozen", False):
            raise dataclasses.FrozenInstanceError(f"cannot assign to field '{name}'")
        object.__setattr__(self, name, value)

    # -- construction ------------------------------------------------------------------
    @classmethod
    def build(
        cls,
        precision_map: Dict[int, Dict[int, str]],
        seq_len: int,
        num_heads: int,
        reuse_mask: Optional[Dict[Tuple[int, int], bool]] = None,
        device: Any = "cpu",
        strict: bool = True,
    ) -> "PrecisionPlan":
        """Plan from a precision map (precision_plan.py:84-111)."""
        codes = map_to_codes(precision_map, seq_len, num_heads, strict=strict, device="cpu")
        return cls.from_codes(codes, reuse_mask=reuse_mask, device=device)

    @classmethod
    def from_codes(
        cls,
        codes: torch.Tensor,
        reuse_mask: Any = None,
        device: Any = None,
    ) -> "PrecisionPlan":
        """Plan from dense ``int8 [seq, heads]`` codes (precision_plan.py:113-177)."""
        if codes.dim() != 2:
            raise ValueError(f"codes must be 2-D [seq, heads], got shape {tuple(codes.shape)}")
        seq_len, num_heads = int(codes.shape[0]), int(codes.shape[1])
        if seq_len <= 0 or num_heads <= 0:
            raise ValueError(f"seq_len and num_heads must be positive, got {seq_len}, {num_heads}")
        device = codes.device if device is None else as_device(device)
        if codes.dtype is torch.int8 and codes.is_cuda and codes.device == device and codes.is_contiguous():
            codes_nom = codes_d = codes                  # already what the kernel reads
            dev = codes.device
        else:
            codes_nom = codes.detach().to(device=device, dtype=torch.int8).contiguous()
            dev = compute_device(codes_nom)
            codes_d = on(codes_nom, dev)
        mask_d = reuse_mask_tensor(reuse_mask, seq_len, num_heads, dev)
        n = seq_len * num_heads
        lib = _lib.load()
        nbytes = lib.skv_plan_scratch_bytes(seq_len, num_heads)
        flat_all = torch.empty(n, dtype=torch.int64, device=dev)
        slot = torch.empty(n, dtype=torch.int32, device=dev)
        reuse_all = torch.empty(n if mask_d is not None else 0, dtype=torch.int64, device=dev)
        counts_d = torch.empty(6, dtype=torch.int64, device=dev)
        scr = torch.empty(max(int(nbytes), 256), dtype=torch.uint8, device=dev)
        with device_ctx(dev):
            st = lib.skv_plan_bucket(_lib.ptr(codes_d), _lib.ptr(mask_d), seq_len, num_heads, flat_all.data_ptr(),
                                     slot.data_ptr(), reuse_all.data_ptr() if mask_d is not None else None,
                                     counts_d.data_ptr(), scr.data_ptr(), scr.numel(), _lib.stream_of(dev))
        _lib.check(st, "PrecisionPlan.from_codes")
        # the counts travel to a pinned host buffer behind an event: nothing waits for them
        # until a host-side field needs them (packing launches on the device counts)
        counts_h, ev = _PINNED.pop() if _PINNED else (torch.empty(6, dtype=torch.int64, pin_memory=True),
                                                      torch.cuda.Event())
        with device_ctx(dev):
            counts_h.copy_(counts_d, non_blocking=True)
            ev.record()
        plan = object.__new__(cls)
        st = object.__setattr__
        st(plan, "_seq_len", seq_len)
        st(plan, "_num_heads", num_heads)
        st(plan, "_codes", codes_nom)
        st(plan, "_device", device)
        st(plan, "_dev", dev)
        st(plan, "_flat_all", flat_all)
        st(plan, "_counts", None)
        st(plan, "_counts_dev", counts_d)
        st(plan, "_pending", (ev, counts_h, reuse_all, mask_d))
        st(plan, "_slot", slot)
        st(plan, "_reuse_flat_dev", None)
        st(plan, "_reuse_mask_dev", None)
        st(plan, "_lazy", {})
        st(plan, "_frozen", True)
        return plan

    def _host_counts(self) -> List[int]:
        """Counts per code 0..4 and the reuse count, waiting for the plan kernel if needed."""
        c = self._counts
        if c is None:
            ev, counts_h, reuse_all, mask_d = self._pending
            ev.synchronize()
            c = counts_h.tolist()
            if len(_PINNED) < 64:
                _PINNED.append((counts_h, ev))
            st = object.__setattr__
            st(self, "_counts", c)
            st(self, "_reuse_flat_dev", reuse_all[: c[5]] if mask_d is not None else reuse_all)
            st(self, "_reuse_mask_dev", mask_d if (mask_d is not None and c[5] > 0) else None)
            st(self, "_pending", None)
        return c

    @property
    def counts_device(self) -> torch.Tensor:
        """Device int64 ``[6]``: entries per code 0..4, then reuse entries (no host sync)."""
        return self._counts_dev

    # -- device-side state used by PackedKVCache / compress ------------------------------
    def bucket_flat(self, code: int) -> torch.Tensor:
        """Device int64 ``h*S+t`` of the entries with ``code`` (bucket order)."""
        c = self._host_counts()
        start = sum(c[:code])
        return self._flat_all[start:start + c[code]]

    @property
    def counts(self) -> List[int]:
        """Entries per code 0..4 (fp32, fp16, int8, int4, evicted)."""
        return self._host_counts()[:5]

    @property
    def slot(self) -> torch.Tensor:
        """Device int32 ``[S*H]``: ``(pos << 2) | code`` of stored entries, -1 for evicted."""
        return self._slot

    @property
    def compute_device(self) -> torch.device:
        return self._dev

    @property
    def reuse_mask_device(self) -> Optional[torch.Tensor]:
        self._host_counts()
        return self._reuse_mask_dev

    # -- reference fields ----------------------------------------------------------------
    @property
    def seq_len(self) -> int:
        return self._seq_len

    @property
    def num_heads(self) -> int:
        return self._num_heads

    @property
    def codes(self) -> torch.Tensor:
        return self._codes

    @property
    def flat_indices(self) -> Dict[str, torch.Tensor]:
        if "flat_indices" not in self._lazy:
            d = {}
            for code, p in enumerate(PRECISION_ORDER):
                t = self.bucket_flat(code)
                d[p] = t if t.device == self._device else t.to(self._device)
            self._lazy["flat_indices"] = d
        return self._lazy["flat_indices"]

    @property
    def groups(self) -> Dict[str, List[Tuple[int, int]]]:
        if "groups" not in self._lazy:
            self._lazy["groups"] = {p: _entries(self.bucket_flat(c), self._seq_len) if self._host_counts()[c] else []
                                    for c, p in enumerate(PRECISION_ORDER)}
        return self._lazy["groups"]

    @property
    def evicted_entries(self) -> List[Tuple[int, int]]:
        if "evicted" not in self._lazy:
            self._lazy["evicted"] = _entries(self.bucket_flat(4), self._seq_len) if self._host_counts()[4] else []
        return self._lazy["evicted"]

    @property
    def reuse_flat(self) -> torch.Tensor:
        if "reuse_flat" not in self._lazy:
            self._host_counts()
            t = self._reuse_flat_dev
            self._lazy["reuse_flat"] = t if t.device == self._device else t.to(self._device)
        return self._lazy["reuse_flat"]

    @property
    def reuse_entries(self) -> List[Tuple[int, int]]:
        if "reuse_entries" not in self._lazy:
            c = self._host_counts()
            self._lazy["reuse_entries"] = _entries(self._reuse_flat_dev, self._seq_len) if c[5] else []
        return self._lazy["reuse_entries"]

    @property
    def fingerprint(self) -> str:
        """SHA-256 of ``<QQ`` (S, H), the codes bytes and the reuse_flat bytes (precision_plan.py:179-190)."""
        if "fingerprint" not in self._lazy:
            digest = hashlib.sha256()
            digest.update(struct.pack("<QQ", self._seq_len, self._num_heads))
            digest.update(self._codes.detach().to("cpu").contiguous().numpy().tobytes())
            self._host_counts()
            digest.update(self._reuse_flat_dev.detach().to("cpu").contiguous().numpy().tobytes())
            self._lazy["fingerprint"] = digest.hexdigest()
        return self._lazy["fingerprint"]

    def reuse_set(self) -> set:
        """Reuse entries as a set for O(1) membership checks."""
        return set(self.reuse_entries)

    def __repr__(self) -> str:
        return (f"PrecisionPlan(seq_len={self._seq_len}, num_heads={self._num_heads}, "
                f"counts={dict(zip(PRECISION_ORDER + (EVICTED,), self._host_counts()[:5]))}, "
                f"reuse={self._host_counts()[5]})")
