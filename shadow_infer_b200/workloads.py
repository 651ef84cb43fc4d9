"""Seeded synthetic workloads for the ShadowKV packed-KV data plane.

The reference quotes its numbers on synthetic tensors only (no dataset), so
every workload here is generated from a seeded ``torch.Generator`` on the CPU,
in a fixed order, so that the CUDA path, the CPU oracle and the reference see
identical bits.

Shapes follow the five benchmark configurations of the data plane:

  cfg1  B1 H32 S512  D128, codes fp16/int8/int4 = 25/50/25 %, group 16
  cfg2  B1 H32 S8192 D128, budget = 30 % of the fp16 size, hard eviction,
        50 % random reuse mask against a previous cache perturbed by N(0, 0.01)
  cfg3  32 layers of packed K/V B1 H32 S4096 D128 (codes 20/50/30 %),
        fp16 queries ~N(0,1), non-causal attention, scale 1/sqrt(128)
  cfg4  B8 S2048 H32 D128, 32 layers, 16 denoising steps (drift/reuse/evict)
  cfg5  B1 S32768 H32 D128, codes 10/30/60 %, 4 outlier channels per head x10
"""

from __future__ import annotations

import math
from typing import Dict, Optional, Tuple

import torch

CONFIGS: Dict[str, Dict] = {
    "cfg1": dict(B=1, H=32, S=512, D=128, fractions=(0.25, 0.50, 0.25), group=16, seed=0),
    "cfg2": dict(B=1, H=32, S=8192, D=128, fractions=(0.25, 0.50, 0.25), group=16, seed=0,
                 budget_frac_of_fp16=0.3, sink_tokens=4, reuse_p=0.5, prev_noise=0.01),
    "cfg3": dict(B=1, H=32, S=4096, D=128, fractions=(0.20, 0.50, 0.30), group=16, layers=32),
    "cfg4": dict(B=8, H=32, S=2048, D=128, fractions=(0.25, 0.50, 0.25), group=16, layers=32,
                 steps=16, evict_frac=0.25),
    "cfg5": dict(B=1, H=32, S=32768, D=128, fractions=(0.10, 0.30, 0.60), group=16, layers=32,
                 outlier_channels=4, outlier_channel_scale=10.0),
}


def kv_tensors(
    B: int, H: int, S: int, D: int, seed: int,
    outlier_frac: float = 0.01, outlier_scale: float = 8.0,
    outlier_channels: int = 0, outlier_channel_scale: float = 10.0,
) -> Tuple[torch.Tensor, torch.Tensor]:
    """K, V ~ N(0,1) fp32 [B,H,S,D]; independent 1 % Bernoulli masks scale entries x8.

    With ``outlier_channels`` > 0, K additionally gets that many seeded channels
    per head multiplied by ``outlier_channel_scale``.
    """
    g = torch.Generator().manual_seed(int(seed))
    k = torch.randn(B, H, S, D, generator=g)
    v = torch.randn(B, H, S, D, generator=g)
    if outlier_frac > 0:
        mk = torch.rand(B, H, S, D, generator=g) < outlier_frac
        k = torch.where(mk, k * outlier_scale, k)
        del mk
        mv = torch.rand(B, H, S, D, generator=g) < outlier_frac
        v = torch.where(mv, v * outlier_scale, v)
        del mv
    if outlier_channels > 0:
        for h in range(H):
            ch = torch.randperm(D, generator=g)[:outlier_channels]
            k[:, h, :, ch] *= outlier_channel_scale
    return k.contiguous(), v.contiguous()


def _head_seed(seed: int, h: int, salt: int = 0) -> int:
    return int(seed) * 1_000_003 + int(salt) * 7_919 + int(h)


def kv_heads(
    B: int, S: int, D: int, seed: int, h0: int, h1: int,
    outlier_frac: float = 0.01, outlier_scale: float = 8.0,
    outlier_channels: int = 0, outlier_channel_scale: float = 10.0,
) -> Tuple[torch.Tensor, torch.Tensor]:
    """K, V ~ N(0,1) fp32 [B, h1-h0, S, D] for heads [h0, h1) of a layer, each head drawn from
    its own generator, so that any head slice is generated alone with the same bits as in the
    whole layer (the long-context and batched workloads, whose layers are 1 GB / 537 MB of
    fp32 K/V).  Per head, in order: K, V, the 1 % Bernoulli x8 outlier masks of K and V, and
    ``outlier_channels`` channels of K scaled by ``outlier_channel_scale``."""
    ks, vs = [], []
    for h in range(h0, h1):
        g = torch.Generator().manual_seed(_head_seed(seed, h))
        k = torch.randn(B, S, D, generator=g)
        v = torch.randn(B, S, D, generator=g)
        if outlier_frac > 0:
            k = torch.where(torch.rand(B, S, D, generator=g) < outlier_frac, k * outlier_scale, k)
            v = torch.where(torch.rand(B, S, D, generator=g) < outlier_frac, v * outlier_scale, v)
        if outlier_channels > 0:
            ch = torch.randperm(D, generator=g)[:outlier_channels]
            k[:, :, ch] *= outlier_channel_scale
        ks.append(k)
        vs.append(v)
    return torch.stack(ks, dim=1).contiguous(), torch.stack(vs, dim=1).contiguous()


def queries_heads(B: int, S: int, D: int, seed: int, h0: int, h1: int) -> torch.Tensor:
    """fp16 queries ~N(0,1) [B, h1-h0, S, D] for heads [h0, h1), one generator per head."""
    qs = []
    for h in range(h0, h1):
        g = torch.Generator().manual_seed(_head_seed(seed, h, salt=31337))
        qs.append(torch.randn(B, S, D, generator=g).to(torch.float16))
    return torch.stack(qs, dim=1).contiguous()


def drift_noise(B: int, S: int, D: int, seed: int, step: int, h0: int, h1: int,
                sigma: float = 0.074, eps: float = 1.0) -> Tuple[torch.Tensor, torch.Tensor]:
    """Per-step drift of the batched denoising loop: for each (token, head) a relative drift
    r ~ |N(0, sigma)| shared by its K and V rows, applied as ``x + r * eps * ||x_row|| / sqrt(D) *
    n`` with n ~ N(0, 1) per element; returns the unit-row noise ``n`` scaled by ``r * eps /
    sqrt(D)`` (multiply by the row norm to apply).  [B, h1-h0, S, D] fp32 for K and for V."""
    nk, nv = [], []
    for h in range(h0, h1):
        g = torch.Generator().manual_seed(_head_seed(seed, h, salt=1000 + step))
        r = torch.randn(S, generator=g).abs() * sigma * eps / math.sqrt(D)
        nk.append(torch.randn(B, S, D, generator=g) * r[None, :, None])
        nv.append(torch.randn(B, S, D, generator=g) * r[None, :, None])
    return torch.stack(nk, dim=1).contiguous(), torch.stack(nv, dim=1).contiguous()


def cfg5_layer(h0: int = 0, h1: Optional[int] = None, layer: int = 0) -> Dict[str, torch.Tensor]:
    """Heads [h0, h1) of one long-context layer (cfg5, seed = layer): K, V fp32 [1, h, 32768, 128]
    with 1 % x8 outliers and 4 outlier channels x10 per head in K, the layer's importance
    [S, H] (all heads; codes 10/30/60 % fp16/int8/int4, 4 fp16 sinks) and fp16 queries."""
    c = CONFIGS["cfg5"]
    h1 = c["H"] if h1 is None else h1
    k, v = kv_heads(c["B"], c["S"], c["D"], layer, h0, h1, outlier_channels=c["outlier_channels"],
                    outlier_channel_scale=c["outlier_channel_scale"])
    return {"k": k, "v": v, "importance": importance_map(c["S"], c["H"], layer, c["fractions"]),
            "q": queries_heads(c["B"], c["S"], c["D"], layer, h0, h1), "group": c["group"]}


def cfg4_layer(h0: int = 0, h1: Optional[int] = None, layer: int = 0) -> Dict[str, torch.Tensor]:
    """Heads [h0, h1) of one batched-denoising layer (cfg4, seed = layer) at step 0: K, V fp32
    [8, h, 2048, 128], the layer's importance [S, H] (codes 25/50/25 %) and fp16 queries."""
    c = CONFIGS["cfg4"]
    h1 = c["H"] if h1 is None else h1
    k, v = kv_heads(c["B"], c["S"], c["D"], 10_000 + layer, h0, h1)
    return {"k": k, "v": v, "importance": importance_map(c["S"], c["H"], 10_000 + layer, c["fractions"]),
            "q": queries_heads(c["B"], c["S"], c["D"], 10_000 + layer, h0, h1), "group": c["group"]}


def apply_drift(x: torch.Tensor, noise: torch.Tensor) -> torch.Tensor:
    """``x + noise * ||x_row||`` (row = the head_dim vector of one (batch, head, token))."""
    return x + noise * torch.linalg.vector_norm(x, dim=-1, keepdim=True)


def lowest_importance_mask(importance: torch.Tensor, frac: float, sink_tokens: int = 4) -> torch.Tensor:
    """bool [S, H]: the ``floor(frac * n)`` entries of lowest importance among the n non-sink
    (t >= sink_tokens) entries, ties in row-major (token, head) order -- the eviction set of
    the batched denoising loop."""
    S, H = importance.shape
    flat = importance.reshape(-1).to(torch.float64).clone()
    flat[: min(sink_tokens, S) * H] = float("inf")
    n = int(math.floor(frac * (S - min(sink_tokens, S)) * H))
    order = torch.argsort(flat, stable=True)
    mask = torch.zeros(S * H, dtype=torch.bool, device=importance.device)
    mask[order[:n]] = True
    return mask.reshape(S, H)


def sample_rows(S: int, n: int, seed: int) -> torch.Tensor:
    """int64 [n]: sorted distinct query rows of a sequence of S, always holding the first and the
    last row (sampled rows of a non-causal attention are checked against the oracle)."""
    g = torch.Generator().manual_seed(int(seed) + 4242)
    mid = torch.randperm(max(S - 2, 0), generator=g)[: max(n - 2, 0)] + 1
    return torch.unique(torch.cat([torch.tensor([0, S - 1]), mid])).to(torch.int64)


def importance_map(
    S: int, H: int, seed: int, fractions=(0.25, 0.50, 0.25), sink_tokens: int = 4
) -> torch.Tensor:
    """fp32 [S,H] importance whose ``balanced`` threshold codes hit ``fractions`` exactly.

    ``softmax`` of N(0,1) logits over the sequence gives the raw ranking per
    head; the top ``f16`` share maps into [0.5, 0.79), the next ``f8`` share
    into [0.2, 0.5) and the rest into [0, 0.2), ordered by rank.  Sink tokens
    (t < ``sink_tokens``) get 0.65 (fp16).
    """
    g = torch.Generator().manual_seed(int(seed) + 7919)
    raw = torch.softmax(torch.randn(S, H, generator=g), dim=0)
    f16, f8, _ = fractions
    n16 = int(math.floor(f16 * S))
    n8 = int(math.floor(f8 * S))
    out = torch.empty(S, H, dtype=torch.float32)
    for h in range(H):
        order = torch.argsort(raw[:, h], descending=True, stable=True)
        rank = torch.empty(S, dtype=torch.long)
        rank[order] = torch.arange(S)
        val = torch.empty(S, dtype=torch.float32)
        in16 = rank < n16
        in8 = (rank >= n16) & (rank < n16 + n8)
        in4 = rank >= n16 + n8
        # u in [0,1): 0 = least important member of the band
        u16 = (n16 - 1 - rank).clamp(min=0).float() / max(n16, 1)
        u8 = (n16 + n8 - 1 - rank).clamp(min=0).float() / max(n8, 1)
        n4 = S - n16 - n8
        u4 = (S - 1 - rank).clamp(min=0).float() / max(n4, 1)
        val[in16] = 0.5 + 0.29 * u16[in16]
        val[in8] = 0.2 + 0.3 * u8[in8]
        val[in4] = 0.2 * u4[in4]
        out[:, h] = val
    if sink_tokens > 0:
        out[: min(sink_tokens, S)] = 0.65
    return out


def reuse_mask(S: int, H: int, seed: int, p: float = 0.5) -> torch.Tensor:
    """Bernoulli(p) bool [S,H] reuse mask."""
    g = torch.Generator().manual_seed(int(seed) + 104729)
    return torch.rand(S, H, generator=g) < p


def perturbed(x: torch.Tensor, seed: int, sigma: float) -> torch.Tensor:
    """``x + N(0, sigma)`` with a seeded generator (the previous step's K or V)."""
    g = torch.Generator().manual_seed(int(seed) + 15485863)
    return x + sigma * torch.randn(x.shape, generator=g)


def fp16_budget(B: int, H: int, S: int, D: int, frac: float) -> int:
    """``floor(frac * fp16 K+V bytes)``."""
    return int(math.floor(frac * 2 * B * H * S * D * 2))


def queries(B: int, H: int, S: int, D: int, seed: int) -> torch.Tensor:
    """fp16 queries ~N(0,1) [B,H,S,D]."""
    g = torch.Generator().manual_seed(int(seed) + 31337)
    return torch.randn(B, H, S, D, generator=g).to(torch.float16)


def cfg2_inputs(S: Optional[int] = None, seed: Optional[int] = None) -> Dict[str, torch.Tensor]:
    """K, V, importance, reuse mask, previous K/V and the budget of cfg2 (``S``/``seed`` override)."""
    c = dict(CONFIGS["cfg2"])
    if S is not None:
        c["S"] = S
    if seed is not None:
        c["seed"] = seed
    B, H, S, D = c["B"], c["H"], c["S"], c["D"]
    k, v = kv_tensors(B, H, S, D, c["seed"])
    imp = importance_map(S, H, c["seed"], c["fractions"], c["sink_tokens"])
    return {
        "k": k, "v": v, "importance": imp,
        "reuse": reuse_mask(S, H, c["seed"], c["reuse_p"]),
        "k_prev": perturbed(k, c["seed"], c["prev_noise"]),
        "v_prev": perturbed(v, c["seed"] + 1, c["prev_noise"]),
        "budget": fp16_budget(B, H, S, D, c["budget_frac_of_fp16"]),
        "sink_tokens": c["sink_tokens"], "group": c["group"],
    }
