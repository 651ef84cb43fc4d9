"""ctypes binding of ``libshadowkv_b200.so`` (the C ABI declared in ``include/shadowkv_b200.h``).

The library is loaded from the package's ``_lib/`` directory.  There is no
fallback: if the library is missing or no CUDA device is present, every data
plane call raises.
"""

from __future__ import annotations

import ctypes
import os
import threading
from typing import Optional, Sequence

import torch

_LIB_PATH = os.path.join(os.path.dirname(os.path.abspath(__file__)), "_lib", "libshadowkv_b200.so")
_LOCK = threading.Lock()
_LIB: Optional[ctypes.CDLL] = None

SKV_OK = 0
SKV_ERR_INVALID_ARGUMENT = 1
SKV_ERR_SHAPE = 2
SKV_ERR_GROUP_SIZE = 3
SKV_ERR_SCRATCH = 4
SKV_ERR_TOO_LARGE = 5
SKV_ERR_CUDA = 6
SKV_ERR_UNSUPPORTED = 7

SKV_ATTN_FAST_K = 1   # attention flag: K in fp16 only (include/shadowkv_b200.h)
SKV_ATTN_ONE_TILE = 2  # attention flag: the single-query-tile pipeline
SKV_ATTN_FMA_EXP = 4   # attention flag: a quarter of the softmax exponentials on the FMA pipe
SKV_ATTN_PAIR = 8      # attention flag: the CTA-pair pipeline (head_dim 128)
SKV_ATTN_OUT_F16 = 16  # attention flag: fp16 output (and fp16 peer buffers)

c_void_p = ctypes.c_void_p
c_int = ctypes.c_int
c_int64 = ctypes.c_int64
c_size_t = ctypes.c_size_t


class SkvBucket(ctypes.Structure):
    """``skv_bucket`` of the C ABI."""

    _fields_ = [
        ("k", c_void_p),
        ("v", c_void_p),
        ("scale_k", c_void_p),
        ("scale_v", c_void_p),
        ("flat", c_void_p),
        ("count", c_int64),
    ]


Buckets4 = SkvBucket * 4

# name -> (restype, argtypes); mirrors include/shadowkv_b200.h
_SIGNATURES = {
    "skv_version": (ctypes.c_char_p, []),
    "skv_status_string": (ctypes.c_char_p, [c_int]),
    "skv_last_error": (ctypes.c_char_p, []),
    "skv_launch_count": (c_int64, []),
    "skv_allocate_codes": (c_int, [c_void_p, c_int64, c_int, c_void_p, c_void_p]),
    "skv_kv_sensitivity": (c_int, [c_void_p, c_void_p, c_int, c_int, c_int, c_int, c_void_p, c_void_p]),
    "skv_predict_codes_bytes": (c_int, [c_void_p, c_int64, c_int, c_int, c_int, c_void_p, c_void_p]),
    "skv_admit_scratch_bytes": (c_size_t, [c_int, c_int]),
    "skv_admit_codes": (c_int, [c_void_p, c_void_p, c_void_p, c_void_p, c_void_p, c_int, c_int, c_int64,
                                c_int, c_int, c_int, c_int, c_int, c_int, c_void_p, c_size_t, c_void_p,
                                c_void_p]),
    "skv_plan_scratch_bytes": (c_size_t, [c_int, c_int]),
    "skv_plan_bucket": (c_int, [c_void_p, c_void_p, c_int, c_int, c_void_p, c_void_p, c_void_p, c_void_p,
                                c_void_p, c_size_t, c_void_p]),
    "skv_plan_static_max_entries": (c_int64, []),
    "skv_plan_bucket_static": (c_int, [c_void_p, c_void_p, c_int, c_int, c_void_p, c_void_p, c_void_p, c_void_p,
                                       c_void_p]),
    "skv_pack": (c_int, [c_void_p, c_void_p, c_int, c_int, c_int, c_int, c_int, c_void_p, ctypes.POINTER(SkvBucket),
                         c_void_p, c_void_p, c_void_p, c_void_p, c_void_p, c_void_p]),
    "skv_unpack": (c_int, [ctypes.POINTER(SkvBucket), c_void_p, c_int, c_int, c_int, c_int, c_int, c_void_p,
                           c_void_p, c_void_p]),
    "skv_apply_reuse": (c_int, [ctypes.POINTER(SkvBucket), c_void_p, c_int, ctypes.POINTER(SkvBucket), c_void_p,
                                c_int, c_void_p, c_int, c_int, c_int, c_int, c_void_p, c_void_p]),
    "skv_head_index": (c_int, [c_void_p, c_int, c_int, c_void_p, c_void_p, c_void_p]),
    "skv_packed_attention_scratch_bytes": (c_size_t, [c_int, c_int, c_int, c_int]),
    "skv_packed_attention": (c_int, [c_void_p, c_int, c_int, c_int, c_int, ctypes.POINTER(SkvBucket), c_int, c_int,
                                     c_void_p, c_void_p, ctypes.c_float, c_void_p, c_size_t, c_void_p, c_void_p,
                                     c_void_p]),
    "skv_stage_kv_tiles": (c_int, [ctypes.POINTER(SkvBucket), c_int, c_int, c_int, c_int, c_int, c_void_p, c_void_p,
                                   c_void_p, c_size_t, c_void_p]),
    "skv_attend_kv_tiles": (c_int, [c_void_p, c_int, c_int, c_int, c_int, c_int, c_void_p, c_void_p, ctypes.c_float,
                                    c_void_p, c_size_t, c_void_p, c_void_p, c_void_p]),
    "skv_stage_kv_tiles_gqa": (c_int, [ctypes.POINTER(SkvBucket), c_int, c_int, c_int, c_int, c_int, c_void_p,
                                       c_void_p, c_void_p, c_void_p, c_int, c_void_p, c_size_t, c_int, c_void_p]),
    "skv_attend_kv_tiles_gqa": (c_int, [c_void_p, c_int, c_int, c_int, c_int, c_int, c_int, c_void_p, c_void_p, c_int,
                                        ctypes.c_float, c_void_p, c_size_t, c_void_p, c_void_p, c_int, c_int,
                                        c_void_p]),
    "skv_attend_kv_tiles_peers": (c_int, [c_void_p, c_int, c_int, c_int, c_int, c_int, c_int, c_void_p, c_void_p,
                                          c_int, ctypes.c_float, c_void_p, c_size_t, c_void_p, c_int, c_int, c_int,
                                          c_void_p, c_int, c_int, c_void_p]),
    "skv_pack_slab_bytes": (c_int64, [ctypes.POINTER(c_int64), c_int, c_int, c_int]),
    "skv_pack_slab": (c_int, [c_void_p, c_void_p, c_int, c_int, c_int, c_int, c_int, c_void_p, c_void_p, c_void_p,
                              c_void_p, c_int64, c_void_p, c_void_p]),
    "skv_ipc_handle_bytes": (c_int, []),
    "skv_ipc_export": (c_int, [c_void_p, c_void_p, ctypes.POINTER(c_int64)]),
    "skv_ipc_open": (c_int, [c_void_p, c_int64, ctypes.POINTER(c_void_p), ctypes.POINTER(c_void_p)]),
    "skv_ipc_close": (c_int, [c_void_p]),
    "skv_peer_store": (c_int, [c_void_p, c_int64, c_void_p, c_int, c_int64, c_void_p]),
    "skv_packed_attention_gqa": (c_int, [c_void_p, c_int, c_int, c_int, c_int, ctypes.POINTER(SkvBucket), c_int, c_int,
                                         c_int, c_void_p, c_void_p, c_void_p, c_void_p, c_int, ctypes.c_float,
                                         c_void_p, c_size_t, c_void_p, c_void_p, c_int, c_int, c_void_p]),
    "skv_budget_candidates": (c_int, [c_void_p, c_int, c_int, c_void_p, c_int, c_int, c_int, c_void_p, c_void_p,
                                      c_void_p, c_void_p]),
    "skv_rank_select_scratch_bytes": (c_size_t, [c_int64]),
    "skv_rank_select": (c_int, [c_void_p, c_void_p, c_int64, c_int64, c_void_p, c_size_t, c_void_p, c_void_p]),
    "skv_mark_smallest": (c_int, [c_void_p, c_int64, c_void_p, c_void_p, c_void_p]),
    "skv_evict_scratch_bytes": (c_size_t, [c_int64]),
    "skv_evict_count": (c_int, [ctypes.POINTER(SkvBucket), c_void_p, c_int, c_int, c_void_p, c_void_p, c_size_t,
                                c_void_p]),
    "skv_evict_compact": (c_int, [ctypes.POINTER(SkvBucket), ctypes.POINTER(SkvBucket), c_void_p, c_void_p, c_int,
                                  c_int, c_int, c_int, c_int, c_void_p, c_size_t, c_void_p]),
    "skv_paged_write": (c_int, [c_void_p, c_void_p, c_int, c_int, c_int64, c_int, c_int, c_void_p, c_int, c_void_p,
                                c_void_p]),
    "skv_paged_gather": (c_int, [c_void_p, c_int, c_int, c_int, c_int, c_int, c_int64, c_int64, c_void_p, c_void_p,
                                 c_void_p]),
    "skv_paged_clear_heads": (c_int, [c_void_p, c_int, c_void_p, c_int64, c_int, c_int, c_int, c_void_p, c_void_p]),
    "skv_reuse_decide": (c_int, [c_void_p, c_void_p, c_void_p, c_void_p, c_int, c_int, c_int, c_int, c_void_p,
                                 ctypes.c_double, c_void_p, c_void_p, c_void_p, c_void_p]),
    "skv_irap_scratch_bytes": (c_size_t, [c_int, c_int, c_int, c_int]),
    "skv_irap_importance": (c_int, [c_void_p, c_int, c_int, c_int, c_int, c_int, c_void_p, c_int, ctypes.c_double,
                                    ctypes.c_double, c_int, ctypes.c_double, c_void_p, c_size_t, c_void_p, c_void_p,
                                    c_void_p, c_void_p]),
}

EXPORTED_SYMBOLS = tuple(_SIGNATURES.keys())


def library_path() -> str:
    return _LIB_PATH


def load() -> ctypes.CDLL:
    """Load the native library once (thread-safe); raises if it is missing."""
    global _LIB
    if _LIB is not None:
        return _LIB
    with _LOCK:
        if _LIB is None:
            if not os.path.exists(_LIB_PATH):
                raise RuntimeError(
                    f"shadow_infer_b200 native library not found at {_LIB_PATH}; "
                    "build it with `python -m shadow_infer_b200.build`"
                )
            lib = ctypes.CDLL(_LIB_PATH)
            for name, (res, args) in _SIGNATURES.items():
                fn = getattr(lib, name)
                fn.restype = res
                fn.argtypes = args
            _LIB = lib
    return _LIB


def last_error() -> str:
    return load().skv_last_error().decode(errors="replace")


def check(status: int, what: str) -> None:
    """Map a C-ABI status to the reference's exception types."""
    if status == SKV_OK:
        return
    msg = last_error() or load().skv_status_string(status).decode()
    if status in (SKV_ERR_INVALID_ARGUMENT, SKV_ERR_SHAPE, SKV_ERR_GROUP_SIZE):
        raise ValueError(f"{what}: {msg}")
    raise RuntimeError(f"{what} failed ({load().skv_status_string(status).decode()}): {msg}")


def ptr(t: Optional[torch.Tensor]) -> Optional[int]:
    """Device address of a CUDA tensor (None passes NULL)."""
    if t is None:
        return None
    if not t.is_cuda:
        raise RuntimeError("internal error: host tensor passed to a device entry point")
    return t.data_ptr()


_raw_stream = getattr(torch._C, "_cuda_getCurrentRawStream", None)


def stream_of(device: torch.device) -> int:
    """The ``cudaStream_t`` of the current stream of ``device`` (without building a Stream object)."""
    if _raw_stream is not None:
        return _raw_stream(device.index if device.index is not None else torch.cuda.current_device())
    return torch.cuda.current_stream(device).cuda_stream


def buckets(entries: Sequence[Optional[dict]]) -> "ctypes.Array":
    """Build ``skv_bucket[4]`` from per-precision dicts of device tensors (None = empty)."""
    arr = Buckets4()
    for i, e in enumerate(entries):
        if e is None:
            arr[i] = SkvBucket(None, None, None, None, None, 0)
        else:
            arr[i] = SkvBucket(ptr(e.get("k")), ptr(e.get("v")), ptr(e.get("scale_k")), ptr(e.get("scale_v")),
                               ptr(e.get("flat")), int(e.get("count", 0)))
    return arr
