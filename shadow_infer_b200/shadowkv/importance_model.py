"""IRAP importance (drop-in for ``compute_irap_importance`` of ``shadowinfer/shadowkv/importance_model.py``).

``compute_irap_importance`` (importance_model.py:37-134) turns one layer's attention
weights ``[batch, heads, seq_q, seq_k]`` into per-(token, head) importance ``[seq_k, heads]``:
the received attention (column mean over batch and queries) is blended into an EMA across
steps, ranked per head (rank / seq_k), mixed with the normalised entropy of each query row
and scaled by a depth factor; the first ``sink_tokens`` tokens get 1.0.  Here one pass over
the weights on the GPU produces both reductions (``skv_irap_importance``); the rank, EMA and
blend are small kernels.  Same arguments, results, ``ValueError`` messages and return tuple
``(importance, new_ema, delta_a)``.

Numerics: the reductions are float64 sums (the reference's float32 torch reductions differ by
their own rounding, ~1e-7 relative); the importance agrees with the reference within the
reference's own 1e-6 tolerance.  Tokens whose EMA values tie exactly are ranked by index (the
reference's unstable argsort leaves their order to its sort implementation).
"""

from __future__ import annotations

import math
from typing import Optional, Tuple

import torch

from .. import _lib
from .._device import back, compute_device, device_ctx, on, scratch
from .kv_cache_manager import TokenHeadScore

__all__ = ["compute_irap_importance", "irap_importance", "TokenHeadScore"]

INPUT_PROBABILITIES = 0      # weights used as given
INPUT_LOGITS = 1             # softmax of the NaN-cleaned logits
INPUT_UNNORMALISED = 2       # probabilities divided by their row sum (clamped to 1e-10)


def _validate(weights: torch.Tensor, irap_decay: float, entropy_weight: float, sink_tokens: int) -> None:
    """importance_model.py:66-74."""
    if weights.dim() != 4:
        raise ValueError(f"weights must be 4-D (batch, heads, seq_q, seq_k), got {weights.dim()}-D")
    if not 0.0 < irap_decay < 1.0:
        raise ValueError(f"irap_decay must be in (0, 1), got {irap_decay}")
    if not 0.0 <= entropy_weight <= 1.0:
        raise ValueError(f"entropy_weight must be in [0, 1], got {entropy_weight}")
    if sink_tokens < 0:
        raise ValueError(f"sink_tokens must be >= 0, got {sink_tokens}")


def irap_importance(
    scores: torch.Tensor,
    input_mode: int,
    received_ema_prev: Optional[torch.Tensor] = None,
    irap_decay: float = 0.9,
    entropy_weight: float = 0.3,
    sink_tokens: int = 4,
    layer_index: int = 0,
    num_layers: int = 1,
) -> Tuple[torch.Tensor, torch.Tensor, Optional[float]]:
    """``compute_irap_importance`` with the attention-input contract fused in: ``input_mode``
    selects probabilities as given, logits (softmax) or unnormalised rows (row-sum correction)."""
    _validate(scores, irap_decay, entropy_weight, sink_tokens)
    B, H, Sq, Sk = (int(x) for x in scores.shape)
    dev = compute_device(scores, received_ema_prev)
    if Sk == 0 or H == 0:
        empty = torch.zeros(Sk, H, dtype=torch.float32, device=scores.device)
        return empty, empty.clone(), (None if received_ema_prev is None else 0.0)
    if B == 0 or Sq == 0:
        raise ValueError("weights must have at least one batch row and one query row")
    x = on(scores, dev, torch.float32)
    prev = None
    s_prev = 0
    if received_ema_prev is not None:
        prev = on(received_ema_prev, dev, torch.float32)
        if prev.dim() != 2:
            raise ValueError(f"received_ema_prev must be 2-D [seq, heads], got {prev.dim()}-D")
        if prev.shape[1] != H:
            if prev.shape[1] != 1:
                raise RuntimeError(
                    f"received_ema_prev has {prev.shape[1]} heads, the weights have {H}"
                )
            prev = prev.expand(-1, H).contiguous()
        s_prev = int(prev.shape[0])
    layer_factor = 1.0 + 0.1 * (layer_index / max(num_layers, 1))
    lib = _lib.load()
    imp = torch.empty(Sk, H, dtype=torch.float32, device=dev)
    ema = torch.empty(Sk, H, dtype=torch.float32, device=dev)
    parts = torch.empty(2, dtype=torch.float64, device=dev)
    scr = scratch(lib.skv_irap_scratch_bytes(B, H, Sq, Sk), dev)
    with device_ctx(dev):
        st = lib.skv_irap_importance(_lib.ptr(x), B, H, Sq, Sk, int(input_mode), _lib.ptr(prev), s_prev,
                                     float(irap_decay), float(entropy_weight), int(sink_tokens), layer_factor,
                                     _lib.ptr(scr), scr.numel(), _lib.ptr(imp), _lib.ptr(ema), _lib.ptr(parts),
                                     _lib.stream_of(dev))
    _lib.check(st, "compute_irap_importance")
    delta_a: Optional[float] = None
    if prev is not None:
        a, b = parts.tolist()
        delta_a = math.sqrt(a) / (math.sqrt(b) + 1e-12)
    return back(imp, scores.device), back(ema, scores.device), delta_a


def compute_irap_importance(
    weights: torch.Tensor,
    received_ema_prev: Optional[torch.Tensor] = None,
    irap_decay: float = 0.9,
    entropy_weight: float = 0.3,
    sink_tokens: int = 4,
    layer_index: int = 0,
    num_layers: int = 1,
) -> Tuple[torch.Tensor, torch.Tensor, Optional[float]]:
    """(importance ``[seq_k, heads]``, new EMA ``[seq_k, heads]``, delta_a | None)
    (importance_model.py:37-134); ``weights`` are normalised attention probabilities."""
    return irap_importance(weights, INPUT_PROBABILITIES, received_ema_prev, irap_decay, entropy_weight,
                           sink_tokens, layer_index, num_layers)
