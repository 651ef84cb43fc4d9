"""Device placement for the data plane: all compute runs on a CUDA device.

Tensors keep the device the caller gave them (the reference's semantics):
host tensors are copied to the current CUDA device for the kernels and the
results are copied back.  There is no CPU compute path -- without a CUDA device
every data-plane call raises ``RuntimeError``.
"""

from __future__ import annotations

import contextlib
from typing import Any, Optional

import torch

_NULL_CTX = contextlib.nullcontext()


_get_device = getattr(torch._C, "_cuda_getDevice", None)


def device_ctx(dev: torch.device):
    """``torch.cuda.device(dev)`` only when ``dev`` is not already the current device."""
    cur = _get_device() if _get_device is not None and torch.cuda.is_initialized() else torch.cuda.current_device()
    return _NULL_CTX if cur == dev.index else torch.cuda.device(dev)


def mask_u8(mask: torch.Tensor, rows: int, cols: int, dev: torch.device) -> Optional[torch.Tensor]:
    """A bool/uint8 ``[rows, cols]`` mask already on ``dev`` as a zero-copy uint8 view, else None."""
    if (mask.dim() == 2 and tuple(mask.shape) == (rows, cols) and mask.device == dev
            and mask.dtype in (torch.bool, torch.uint8) and mask.is_contiguous()):
        return mask if mask.dtype == torch.uint8 else mask.view(torch.uint8)
    return None


def compute_device(*tensors: Optional[torch.Tensor]) -> torch.device:
    """The CUDA device to compute on: that of the first CUDA tensor, else the current one."""
    for t in tensors:
        if t is not None and t.is_cuda:
            return t.device
    if not torch.cuda.is_available():
        raise RuntimeError(
            "shadow_infer_b200 runs the ShadowKV data plane on a CUDA (sm_100a) device only; "
            "no CUDA device is available"
        )
    return torch.device("cuda", torch.cuda.current_device())


def as_device(device: Any) -> torch.device:
    return device if isinstance(device, torch.device) else torch.device(device)


def on(t: Optional[torch.Tensor], dev: torch.device, dtype: Optional[torch.dtype] = None) -> Optional[torch.Tensor]:
    """``t`` contiguous on ``dev`` (and ``dtype``), copying only when needed; detached from autograd
    (the kernels read the storage only)."""
    if t is None:
        return None
    if (dtype is None or t.dtype is dtype) and t.is_cuda and t.get_device() == dev.index and t.is_contiguous():
        return t.detach() if t.requires_grad else t  # already what the kernel reads
    t = t.detach()
    if dtype is not None and t.dtype != dtype:
        t = t.to(dtype)
    if t.device != dev:
        t = t.to(dev, non_blocking=True)
    return t.contiguous()


def back(t: torch.Tensor, device: torch.device) -> torch.Tensor:
    """Move a result to the caller's device."""
    if isinstance(device, torch.device) and device.type == "cuda" and device.index == t.get_device():
        return t
    return t if t.device == device else t.to(device)


def scratch(nbytes: int, dev: torch.device) -> torch.Tensor:
    """Scratch buffer from the caching allocator (at least 256 bytes, 256-byte aligned)."""
    return torch.empty(max(int(nbytes), 256), dtype=torch.uint8, device=dev)
