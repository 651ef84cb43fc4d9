"""Rate-distortion KV admission (drop-in for ``shadowinfer/shadowkv/rd_allocator.py``).

``kv_sensitivity``, ``predict_codes_bytes`` and ``admit_codes`` run as sm_100a
kernels (``skv_kv_sensitivity``, ``skv_predict_codes_bytes``,
``skv_admit_codes``).  ``admit_codes`` replaces the reference's stable argsort
+ prefix sums (rd_allocator.py:245-316) with a weighted radix select over a
unique 64-bit (score, index) key, which finds the same boundary entry and so
yields identical codes, predicted bytes and eviction count.
``entry_bytes`` is the reference's cost model, evaluated on the host.
"""

from __future__ import annotations

from typing import Dict, Optional, Set, Tuple

import torch

from .. import _lib
from .._device import back, compute_device, on, scratch, device_ctx
from .precision_plan import codes_to_map, map_to_codes

EVICTED = "evicted"
DOWNGRADE_LADDER = {"fp32": "fp16", "fp16": "int8", "int8": "int4"}
CODE_PRECISIONS = {0: "fp32", 1: "fp16", 2: "int8", 3: "int4", 4: EVICTED}
PRECISION_CODE_DOWNGRADE = {0: 1, 1: 2, 2: 3}
EVICTED_CODE = 4


def entry_bytes(precision: str, batch: int, head_dim: int, group_size: int = 16) -> float:
    """Stored K+V bytes of one token-head incl. scales (rd_allocator.py:26-44)."""
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


def kv_sensitivity(k: torch.Tensor, v: torch.Tensor) -> torch.Tensor:
    """Per-token-head ``(|k|max^2 + |v|max^2)/2`` over batch and head_dim, ``[seq, heads]`` (rd_allocator.py:47-61)."""
    if k.shape != v.shape:
        raise ValueError("k and v must have identical shapes")
    B, H, S, D = k.shape
    dev = compute_device(k, v)
    kd = on(k, dev, torch.float32)
    vd = on(v, dev, torch.float32)
    out = torch.empty(S, H, dtype=torch.float32, device=dev)
    lib = _lib.load()
    with device_ctx(dev):
        st = lib.skv_kv_sensitivity(_lib.ptr(kd), _lib.ptr(vd), B, H, S, D, _lib.ptr(out), _lib.stream_of(dev))
    _lib.check(st, "kv_sensitivity")
    return back(out, k.device)


def predict_codes_bytes(codes: torch.Tensor, batch: int, head_dim: int, group_size: int = 16) -> int:
    """Byte prediction of dense codes (rd_allocator.py:170-187)."""
    dev = compute_device(codes)
    cd = on(codes, dev, torch.int8)
    out = torch.empty(1, dtype=torch.int64, device=dev)
    lib = _lib.load()
    with device_ctx(dev):
        st = lib.skv_predict_codes_bytes(_lib.ptr(cd), cd.numel(), batch, head_dim, group_size, _lib.ptr(out),
                                         _lib.stream_of(dev))
    _lib.check(st, "predict_codes_bytes")
    return int(out.item())


def admit_codes_device(
    codes: torch.Tensor,
    importance: torch.Tensor,
    sensitivity: Optional[torch.Tensor],
    budget_bytes: Optional[int],
    batch: int,
    head_dim: int,
    sink_tokens: int = 0,
    rd_allocation: bool = True,
    allow_eviction: bool = False,
    protected_mask: Optional[torch.Tensor] = None,
    group_size: int = 16,
) -> Tuple[torch.Tensor, torch.Tensor]:
    """``admit_codes`` without a host sync: returns device codes and ``int64[2]`` (predicted, evicted)."""
    if codes.dim() != 2:
        raise ValueError(f"codes must be 2-D [seq, heads], got shape {tuple(codes.shape)}")
    S, H = int(codes.shape[0]), int(codes.shape[1])
    dev = compute_device(codes, importance, sensitivity)
    cd = on(codes, dev, torch.int8)
    imp = importance.detach()
    if tuple(imp.shape) != (S, H):
        imp = imp[:S, :H]
        if tuple(imp.shape) != (S, H):
            raise ValueError(f"importance must cover codes {(S, H)}, got {tuple(importance.shape)}")
    imp = on(imp, dev, torch.float32)
    sens = None
    if sensitivity is not None:
        s = sensitivity.detach()
        if tuple(s.shape) != (S, H):
            s = s[:S, :H]
        if tuple(s.shape) == (S, H):
            sens = on(s, dev, torch.float32)
    prot = None
    if protected_mask is not None:
        pm = protected_mask.detach()[:S, :H]
        prot = torch.zeros(S, H, dtype=torch.uint8, device=dev)
        prot[: pm.shape[0], : pm.shape[1]] = on(pm, dev).to(torch.uint8)
    out = torch.empty(S, H, dtype=torch.int8, device=dev)
    res = torch.empty(2, dtype=torch.int64, device=dev)
    lib = _lib.load()
    scr = scratch(lib.skv_admit_scratch_bytes(S, H), dev)
    budget = -1 if budget_bytes is None or budget_bytes < 0 else int(budget_bytes)
    with device_ctx(dev):
        st = lib.skv_admit_codes(_lib.ptr(cd), _lib.ptr(out), _lib.ptr(imp), _lib.ptr(sens), _lib.ptr(prot), S, H,
                                 budget, batch, head_dim, group_size, int(sink_tokens), int(bool(rd_allocation)),
                                 int(bool(allow_eviction)), _lib.ptr(scr), scr.numel(), _lib.ptr(res),
                                 _lib.stream_of(dev))
    _lib.check(st, "admit_codes")
    return out, res


def admit_codes(
    codes: torch.Tensor,
    importance: torch.Tensor,
    sensitivity: Optional[torch.Tensor],
    budget_bytes: Optional[int],
    batch: int,
    head_dim: int,
    sink_tokens: int = 0,
    rd_allocation: bool = True,
    allow_eviction: bool = False,
    protected_mask: Optional[torch.Tensor] = None,
    group_size: int = 16,
) -> Tuple[torch.Tensor, int, int]:
    """Fit dense ``int8 [seq, heads]`` codes into ``budget_bytes`` (rd_allocator.py:190-318).

    Returns ``(codes_out, predicted_bytes, evicted_count)``; the input is not
    mutated.  Candidates (non-sink, unprotected) are ranked by ascending
    ``importance * sensitivity`` (or importance only), stable on ``(token,
    head)``; a sensitivity whose shape differs from the importance counts as ones.
    """
    out, res = admit_codes_device(codes, importance, sensitivity, budget_bytes, batch, head_dim, sink_tokens,
                                  rd_allocation, allow_eviction, protected_mask, group_size)
    predicted, evicted = (int(x) for x in res.tolist())
    if predicted < 0:
        raise RuntimeError("admit_codes: the admission kernel's grid barrier timed out")
    return back(out, codes.device), predicted, evicted


def admit_budget(
    importance: torch.Tensor,
    sensitivity: torch.Tensor,
    precision_map: Dict[int, Dict[int, str]],
    budget_bytes: int,
    batch: int,
    head_dim: int,
    sink_tokens: int = 0,
    rd_allocation: bool = True,
    allow_eviction: bool = False,
    protected: Optional[Set[Tuple[int, int]]] = None,
    group_size: int = 16,
) -> Tuple[Dict[int, Dict[int, str]], int, int]:
    """Dict form of the admission (rd_allocator.py:64-167), evaluated through ``admit_codes``.

    The reference asserts ``admit_codes`` == ``admit_budget`` on codes built
    from the map; this form converts the map, runs the kernel and converts back.
    """
    seq_len = int(importance.shape[0])
    num_heads = int(importance.shape[1]) if importance.dim() > 1 else 1
    codes = map_to_codes(precision_map, seq_len, num_heads, strict=False)
    prot = None
    if protected:
        prot = torch.zeros(seq_len, num_heads, dtype=torch.bool)
        for t, h in protected:
            if 0 <= t < seq_len and 0 <= h < num_heads:
                prot[t, h] = True
    imp = importance if importance.dim() > 1 else importance.reshape(-1, 1)
    out, predicted, evicted = admit_codes(codes, imp, sensitivity, budget_bytes, batch, head_dim, sink_tokens,
                                          rd_allocation, allow_eviction, prot, group_size)
    return codes_to_map(out), predicted, evicted
