"""Shared helpers for the golden fixtures: canonical digests of packed caches.

A packed cache (the reference's ``PackedKVCache.packed_data`` schema) is
summarised bucket by bucket as dtype/shape/SHA-256 of every tensor plus the
entry list, byte offsets and int4 group fields.  The same summary is computed
from the reference (when the fixtures are generated), from the CPU oracle and
from the CUDA path, so equality of summaries is bit-exact equality of the
packed bytes, scales and index lists.
"""

from __future__ import annotations

import hashlib
import json
import os
from typing import Any, Dict

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
SMALL_NPZ = os.path.join(HERE, "small_cases.npz")
PINS_JSON = os.path.join(HERE, "pins.json")

_DTYPE_NAMES = {
    "float32": "float32", "float16": "float16", "int8": "int8", "uint8": "uint8",
    "int64": "int64", "int32": "int32", "bool": "bool",
}


def to_numpy(x: Any) -> np.ndarray:
    """torch tensor (any device, any strides) or array -> contiguous numpy array."""
    if hasattr(x, "detach"):
        x = x.detach().to("cpu").contiguous().numpy()
    return np.ascontiguousarray(np.asarray(x))


def array_digest(x: Any) -> str:
    a = to_numpy(x)
    h = hashlib.sha256()
    h.update(str(a.dtype).encode())
    h.update(str(tuple(a.shape)).encode())
    h.update(a.tobytes())
    return h.hexdigest()


def packed_summary(packed_data: Dict[str, Dict[str, Any]], memory_bytes: int) -> Dict[str, Any]:
    """Canonical summary of a ``packed_data`` dict (reference schema)."""
    out: Dict[str, Any] = {"memory_bytes": int(memory_bytes), "buckets": {}}
    for name in sorted(packed_data.keys()):
        d = packed_data[name]
        b: Dict[str, Any] = {}
        for key in ("k", "v", "scale_k", "scale_v"):
            t = d.get(key)
            b[key] = None if t is None else array_digest(t)
        idx = np.array(list(d["indices"]), dtype=np.int64).reshape(-1, 2)
        b["indices"] = array_digest(idx)
        b["n"] = int(idx.shape[0])
        if "byte_offsets" in d:
            b["byte_offsets"] = array_digest(np.array(list(d["byte_offsets"]), dtype=np.int64).reshape(-1, 4))
            b["group_size"] = int(d["group_size"])
            b["num_groups"] = int(d["num_groups"])
        out["buckets"][name] = b
    return out


def load_pins() -> Dict[str, Any]:
    with open(PINS_JSON) as f:
        return json.load(f)


def load_small() -> Dict[str, np.ndarray]:
    with np.load(SMALL_NPZ, allow_pickle=False) as z:
        return {k: z[k] for k in z.files}


def case_arrays(small: Dict[str, np.ndarray], case: str) -> Dict[str, np.ndarray]:
    pre = case + "/"
    return {k[len(pre):]: v for k, v in small.items() if k.startswith(pre)}


# ------------------------------------------------------------------------------ paged store
def paged_inputs(seed: int, B: int, H: int, T: int, D: int):
    """Seeded K/V ``[B,H,T,D]`` fp32 for the paged-store scripts: N(0, 2^2) values, about 3% of
    the (b, h, t) rows exactly zero (scale 0 -> 1) and a few values large enough to overflow fp16."""
    rng = np.random.default_rng(seed)
    out = []
    for _ in range(2):
        x = (rng.standard_normal((B, H, T, D)) * 2.0).astype(np.float32)
        x[rng.random((B, H, T)) < 0.03] = 0.0
        x[rng.random((B, H, T, D)) < 0.002] *= np.float32(4.0e4)
        out.append(x)
    return out[0], out[1]


def paged_bad_inputs(kind: str, seed: int, B: int, H: int, D: int):
    """Inputs that every append/rewrite must refuse with ValueError (paged_kv_store.py:149-183)."""
    k, v = paged_inputs(seed, B, H, 3, D)
    if kind == "heads":
        k, v = paged_inputs(seed, B, H + 1, 3, D)
    elif kind == "dim":
        k, v = paged_inputs(seed, B, H, 3, D + 1)
    elif kind == "batch":
        k, v = paged_inputs(seed, B + 1, H, 3, D)
    elif kind == "ndim":
        k = k[..., 0]
    elif kind == "kv_mismatch":
        v = v[:, :, :2]
    return k, v


def state_digest(page_digests) -> str:
    """One SHA-256 over the per-page tensor digests of a store state."""
    return hashlib.sha256(json.dumps(page_digests).encode()).hexdigest()


def paged_apply(store, op, B: int, H: int, D: int, conv):
    """Apply one scripted operation (as recorded in the fixtures) to a paged store; ``conv``
    turns the numpy inputs into what the store takes.  Returns the operation's return value."""
    name = op[0]
    if name == "append":
        _, T, prec, seed = op
        k, v = paged_inputs(seed, B, H, T, D)
        return store.append(conv(k), conv(v), prec)
    if name == "append_bad":
        _, kind, prec, seed = op
        k, v = paged_bad_inputs(kind, seed, B, H, D)
        return store.append(conv(k), conv(v), prec)
    if name == "rewrite":
        _, start, T, prec, seed = op
        k, v = paged_inputs(seed, B, H, T, D)
        return store.rewrite_tokens(start, conv(k), conv(v), prec)
    if name == "rewrite_bad":
        _, start, kind, prec, seed = op
        k, v = paged_bad_inputs(kind, seed, B, H, D)
        return store.rewrite_tokens(start, conv(k), conv(v), prec)
    if name == "evict":
        return store.evict_tokens({(int(t), int(h)) for t, h in op[1]})
    if name == "clear":
        return store.clear()
    if name == "validate":
        return store.validate_against(*op[1:])
    raise ValueError(f"unknown scripted operation {name}")


# ---------------------------------------------------------------------- decision inputs
def irap_scores(seed: int, B: int, H: int, Sq: int, Sk: int, kind: str = "probs", sharpen: float = 6.0,
                bad: bool = False) -> np.ndarray:
    """Seeded attention input ``[B,H,Sq,Sk]`` fp32: ``logits`` = N(0,1) with 3/4 of the query
    rows sharpened; ``probs`` = their row softmax; ``raw`` = unnormalised non-negative rows
    (some all-zero).  ``bad`` plants NaN / +-inf entries."""
    rng = np.random.default_rng(seed)
    x = rng.standard_normal((B, H, Sq, Sk)).astype(np.float64)
    x[:, :, : (3 * Sq) // 4] *= sharpen
    if kind == "probs":
        e = np.exp(x - x.max(axis=-1, keepdims=True))
        x = e / e.sum(axis=-1, keepdims=True)
    elif kind == "raw":
        x = np.abs(x) * rng.random((B, H, Sq, 1))
        x[:, :, rng.random(Sq) < 0.05] = 0.0
    x = x.astype(np.float32)
    if bad:
        flat = x.reshape(-1)
        idx = rng.choice(flat.size, size=max(3, flat.size // 2000), replace=False)
        flat[idx[0::3]] = np.nan
        flat[idx[1::3]] = np.inf
        flat[idx[2::3]] = -np.inf
    return x


def reuse_inputs(seed: int, B: int, H: int, S: int, D: int):
    """Seeded (k_cur, v_cur, k_prev, v_prev, importance): the previous step's K/V drift by a
    per-(token, head) relative amount spread around the reuse thresholds; a few rows exactly
    zero; importance in [-0.1, 1.1] (clamped by the reference)."""
    rng = np.random.default_rng(seed)
    k = rng.standard_normal((B, H, S, D)).astype(np.float32)
    v = rng.standard_normal((B, H, S, D)).astype(np.float32)
    rk = np.abs(rng.normal(0.0, 0.12, (1, H, S, 1))).astype(np.float32)
    rv = np.abs(rng.normal(0.0, 0.12, (1, H, S, 1))).astype(np.float32)
    kp = (k + rk * rng.standard_normal((B, H, S, D)).astype(np.float32)).astype(np.float32)
    vp = (v + rv * rng.standard_normal((B, H, S, D)).astype(np.float32)).astype(np.float32)
    zero = rng.random((H, S)) < 0.01
    k[:, zero] = 0.0
    kp[:, zero] = 0.0
    imp = (rng.random((S, H)) * 1.2 - 0.1).astype(np.float32)
    return k, v, kp, vp, imp


BLOCK_PARAM_ORDER = ("ln1.weight", "ln1.bias", "q_proj.weight", "q_proj.bias", "k_proj.weight", "k_proj.bias",
                     "v_proj.weight", "v_proj.bias", "o_proj.weight", "o_proj.bias", "ln2.weight", "ln2.bias",
                     "up_proj.weight", "up_proj.bias", "down_proj.weight", "down_proj.bias")


def block_params(seed: int, hidden: int, inter: int) -> Dict[str, Any]:
    """Seeded parameters of one diffusion transformer block (the attribute names and shapes of
    shadowinfer/models/simple_diffusion_llm.py:26-52), drawn in BLOCK_PARAM_ORDER so that the
    fixture generator and the GPU test build the same block without storing weights."""
    import torch
    g = torch.Generator().manual_seed(int(seed))
    shapes = {"ln1": (hidden,), "ln2": (hidden,), "q_proj": (hidden, hidden), "k_proj": (hidden, hidden),
              "v_proj": (hidden, hidden), "o_proj": (hidden, hidden), "up_proj": (inter, hidden),
              "down_proj": (hidden, inter)}
    out = {}
    for name in BLOCK_PARAM_ORDER:
        mod, kind = name.split(".")
        shp = shapes[mod]
        if mod.startswith("ln"):
            base = 1.0 if kind == "weight" else 0.0
            out[name] = base + 0.1 * torch.randn(shp, generator=g)
        elif kind == "weight":
            out[name] = torch.randn(shp, generator=g) / (shp[1] ** 0.5)
        else:
            out[name] = 0.02 * torch.randn(shp[0], generator=g)
    return out
