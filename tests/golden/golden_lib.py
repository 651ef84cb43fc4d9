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
