"""CPU oracle for the ShadowKV decision inputs -- TEST INFRASTRUCTURE ONLY.

numpy restatement of
  * ``compute_irap_importance`` (reference ``shadowinfer/shadowkv/importance_model.py:37-134``):
    received attention (column mean over batch and queries), its EMA across steps, the per-head
    rank of the EMA, the row entropy of the attention weights, the blend and the sink guard;
  * the attention-input contract of ``ShadowKVAgent._compute_importance_with_state``
    (``shadowinfer/shadowkv/shadowkv_agent.py:899-965``): softmax of NaN-free logits, or the
    row-sum correction of probabilities;
  * ``ShadowKVAgent.decide_reuse_per_token`` (``shadowkv_agent.py:1165-1256``): relative L2
    drift per (token, head) against an importance-scaled threshold.
Imported only by ``tests/`` and ``bench.py``'s CPU legs.

Arithmetic: reductions are float64 sums of the float32 inputs (the reference's torch CPU
float32 reductions differ from them by ~1e-7 relative, its own rounding); every elementwise
step the reference does in float32 (the EMA, ``+ 1e-8``, the drift ratios) is done in
float32 here, the float64 steps (thresholds, rank blend) in float64.  Ties in the EMA are
ranked by token index (a stable sort; the reference's unstable ``argsort`` leaves their order
to its sort implementation).  Parity with the reference is pinned by
``tests/golden/make_golden.py`` (fixtures recorded from the reference) within the reference's
own 1e-6 tolerance (``tests/test_irap_contract.py`` of the reference).
"""

from __future__ import annotations

import math
from typing import Dict, Optional, Tuple

import numpy as np

F32 = np.float32


def _f32(x) -> np.ndarray:
    return np.asarray(x, dtype=np.float32)


def irap_inputs(scores: np.ndarray, attn_is_probabilities: bool) -> np.ndarray:
    """Contract normalisation (shadowkv_agent.py:894-897, :955-960): probabilities are
    divided by their row sum clamped to 1e-10; logits are NaN/inf-cleaned then softmaxed."""
    x = scores.astype(np.float64)
    if attn_is_probabilities:
        s = x.sum(axis=-1, keepdims=True)
        return (x / np.maximum(s, 1e-10)).astype(np.float32)
    x = np.nan_to_num(x, nan=0.0, posinf=float(np.finfo(np.float32).max), neginf=float(np.finfo(np.float32).min))
    m = x.max(axis=-1, keepdims=True)
    e = np.exp(x - m)
    return (e / e.sum(axis=-1, keepdims=True)).astype(np.float32)


def compute_irap_importance(weights: np.ndarray, received_ema_prev: Optional[np.ndarray] = None,
                            irap_decay: float = 0.9, entropy_weight: float = 0.3, sink_tokens: int = 4,
                            layer_index: int = 0, num_layers: int = 1
                            ) -> Tuple[np.ndarray, np.ndarray, Optional[float]]:
    """(importance f32 [Sk,H], new EMA f32 [Sk,H], delta_a or None) (importance_model.py:37-134)."""
    if weights.ndim != 4:
        raise ValueError(f"weights must be 4-D (batch, heads, seq_q, seq_k), got {weights.ndim}-D")
    if not 0.0 < irap_decay < 1.0:
        raise ValueError(f"irap_decay must be in (0, 1), got {irap_decay}")
    if not 0.0 <= entropy_weight <= 1.0:
        raise ValueError(f"entropy_weight must be in [0, 1], got {entropy_weight}")
    if sink_tokens < 0:
        raise ValueError(f"sink_tokens must be >= 0, got {sink_tokens}")
    B, H, Sq, Sk = weights.shape
    log_seq = math.log(max(Sk, 2))
    w = np.nan_to_num(weights.astype(np.float32), nan=0.0, posinf=0.0, neginf=0.0)
    w64 = w.astype(np.float64)
    received = (w64.sum(axis=(0, 2)) / (B * Sq)).astype(np.float32)            # [H, Sk]
    if received_ema_prev is None:
        ema = received
        delta_a = None
    else:
        prev = _f32(received_ema_prev)
        if prev.shape[0] < Sk:
            prev = np.concatenate([prev, np.zeros((Sk - prev.shape[0], prev.shape[1]), np.float32)], axis=0)
        else:
            prev = prev[:Sk]
        prev_t = prev.T                                                         # [H, Sk]
        d = np.float32(irap_decay)
        e = np.float32(1.0 - irap_decay)
        ema = (d * prev_t).astype(np.float32) + (e * received).astype(np.float32)
        ema = ema.astype(np.float32)
        diff = (ema.astype(np.float64) - prev_t.astype(np.float64))
        delta_a = float(math.sqrt(float((diff * diff).sum())) /
                        (math.sqrt(float((prev_t.astype(np.float64) ** 2).sum())) + 1e-12))
    order = np.argsort(ema, axis=-1, kind="stable")
    ranks = np.empty_like(order)
    np.put_along_axis(ranks, order, np.arange(Sk)[None, :].repeat(H, axis=0), axis=-1)
    rank_norm = (ranks.astype(np.float64) + 1.0) / Sk                           # [H, Sk]
    c = np.maximum(w64, 1e-10)
    denom = c.sum(axis=(0, 3))                                                  # [H, Sq]
    s1 = (c * np.log(c)).sum(axis=(0, 3))
    entropy = np.log(denom) - s1 / denom
    nent = (entropy / log_seq).astype(np.float32).T                             # [Sq, H]
    if nent.shape[0] != Sk:
        padded = np.zeros((Sk, H), np.float32)
        keep = min(Sk, nent.shape[0])
        padded[:keep] = nent[:keep]
        nent = padded
    layer_factor = 1.0 + 0.1 * (layer_index / max(num_layers, 1))
    blended = (1.0 - entropy_weight) * rank_norm.T
    blended = blended + (np.float32(entropy_weight) * nent).astype(np.float32).astype(np.float64)
    importance = np.minimum(blended * layer_factor, 1.0).astype(np.float32)
    if sink_tokens > 0:
        importance[:min(sink_tokens, Sk)] = 1.0
    return importance, ema.T.copy(), delta_a


def effective_threshold(step_id: int, total_steps: int, qdrift_drift_score: float, mode: str) -> float:
    """shadowkv_agent.py:1222-1231 (Python float arithmetic)."""
    progress = step_id / max(total_steps, 1)
    base = {"aggressive": 0.20, "balanced": 0.15, "conservative": 0.10}.get(mode, 0.15)
    adaptive = base * (1.0 - 0.5 * progress)
    return adaptive * (1.0 - qdrift_drift_score * 0.3)


def reuse_drift(k_cur: np.ndarray, v_cur: np.ndarray, k_prev: np.ndarray, v_prev: np.ndarray) -> np.ndarray:
    """float32 drift ``(|dk|/(|k|+1e-8) + |dv|/(|v|+1e-8)) / 2`` per (head, token), norms over
    (batch, head_dim) (shadowkv_agent.py:1207-1216)."""
    def norm(x):
        x64 = x.astype(np.float64)
        return np.sqrt((x64 * x64).sum(axis=(0, 3))).astype(np.float32)

    eps = np.float32(1e-8)
    dk = (norm(k_cur - k_prev) / (norm(k_cur) + eps)).astype(np.float32)
    dv = (norm(v_cur - v_prev) / (norm(v_cur) + eps)).astype(np.float32)
    return ((dk + dv) / np.float32(2.0)).astype(np.float32)                   # [H, S]


def decide_reuse_per_token(k_cur, v_cur, k_prev, v_prev, step_id: int, total_steps: int,
                           qdrift_drift_score: float, mode: str, importance_map: np.ndarray
                           ) -> Tuple[np.ndarray, Dict[str, float], np.ndarray]:
    """(mask bool [S,H], stats, drift f32 [H,S]) (shadowkv_agent.py:1165-1256)."""
    B, H, S, D = k_cur.shape
    delta = reuse_drift(k_cur, v_cur, k_prev, v_prev)
    eff = effective_threshold(step_id, total_steps, qdrift_drift_score, mode)
    imp = np.clip(importance_map.astype(np.float64), 0.0, 1.0)
    thr = np.maximum(eff * (1.0 - 0.3 * imp), 1e-5)
    mask = delta.astype(np.float64).T < thr
    per_token = mask.sum(axis=1)
    full = int((per_token == H).sum())
    none = int((per_token == 0).sum())
    stats = {"full_reuse_count": float(full), "partial_reuse_count": float(S - full - none),
             "no_reuse_count": float(none), "reuse_ratio": float(int(mask.sum()) / max(S * H, 1))}
    return mask, stats, delta
