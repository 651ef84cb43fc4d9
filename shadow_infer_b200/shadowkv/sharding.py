"""Head sharding of the data plane over the GPUs of one node (torch.distributed, NCCL).

Every operation on the path is independent per attention head except budget
admission, which ranks all (token, head) entries of a layer together.  A layer can
therefore be split by heads: rank ``r`` of ``n`` owns heads ``[r*H/n, (r+1)*H/n)``
and packs, unpacks, reuses, evicts and attends over them locally.  Two exchange
steps remain:

* ``admit_codes_sharded`` -- all-gather of the ``[S, H/n]`` codes, importance and
  sensitivity slices; every rank then runs the same deterministic admission on the
  full ``[S, H]`` problem and keeps its own columns, so the result equals the
  single-GPU admission exactly.
* ``all_gather_heads`` -- the attention outputs ``[B, H/n, S, D]`` of all ranks
  assembled into ``[B, H, S, D]`` (one NCCL all-gather).
* ``PeerOutputs`` -- the fused alternative: every rank's ``[B, H, S, D]`` output buffer is
  mapped into all ranks (CUDA IPC), and the attention kernel's epilogue stores each finished
  row straight into every rank's buffer over NVLink (``packed_attention(...,
  peer_outputs=...)``), so the exchange overlaps the attention itself and no NCCL kernel
  competes with it for SMs.

The collectives go through ``torch.distributed``, so the same code runs on a gloo
(CPU) group in tests.
"""

from __future__ import annotations

import ctypes

from typing import Optional, Tuple

import torch
import torch.distributed as dist


def head_range(num_heads: int, world_size: int, rank: int) -> Tuple[int, int]:
    """Heads ``[h0, h1)`` owned by ``rank``; heads must divide evenly."""
    if world_size <= 0 or not 0 <= rank < world_size:
        raise ValueError(f"bad rank {rank} for world size {world_size}")
    if num_heads % world_size:
        raise ValueError(f"{num_heads} heads do not shard evenly over {world_size} ranks")
    per = num_heads // world_size
    return rank * per, (rank + 1) * per


def _world(group) -> Tuple[int, int]:
    return dist.get_world_size(group), dist.get_rank(group)


def all_gather_heads(local: torch.Tensor, group=None, out: Optional[torch.Tensor] = None) -> torch.Tensor:
    """``[B, h, ...]`` per rank -> ``[B, world*h, ...]`` in rank order (heads are dim 1)."""
    n, _ = _world(group)
    local = local.contiguous()
    buf = torch.empty((n * local.shape[0],) + tuple(local.shape[1:]), dtype=local.dtype, device=local.device)
    dist.all_gather_into_tensor(buf, local, group=group)
    buf = buf.view((n,) + tuple(local.shape))
    full = buf.movedim(0, 1).reshape((local.shape[0], n * local.shape[1]) + tuple(local.shape[2:]))
    if out is not None:
        out.copy_(full)
        return out
    return full


def all_gather_columns(local: torch.Tensor, group=None) -> torch.Tensor:
    """``[S, h]`` per rank -> ``[S, world*h]`` (token-major maps of one layer)."""
    n, _ = _world(group)
    local = local.contiguous()
    buf = torch.empty((n * local.shape[0],) + tuple(local.shape[1:]), dtype=local.dtype, device=local.device)
    dist.all_gather_into_tensor(buf, local, group=group)
    return buf.view((n,) + tuple(local.shape)).permute(1, 0, 2).reshape(local.shape[0], n * local.shape[1])


def admit_codes_sharded(
    codes_local: torch.Tensor,
    importance_local: torch.Tensor,
    sensitivity_local: Optional[torch.Tensor],
    budget_bytes: Optional[int],
    batch: int,
    head_dim: int,
    sink_tokens: int = 0,
    rd_allocation: bool = True,
    allow_eviction: bool = False,
    protected_local: Optional[torch.Tensor] = None,
    group=None,
    group_size: int = 16,
    admit=None,
) -> Tuple[torch.Tensor, int, int]:
    """Budget admission of a head-sharded layer; identical to the unsharded ``admit_codes``.

    ``budget_bytes`` is the budget of the WHOLE layer.  Returns this rank's columns of
    the admitted codes and the layer-wide predicted bytes and eviction count.
    ``admit`` defaults to ``rd_allocator.admit_codes`` (the GPU kernel).
    """
    if admit is None:
        from .rd_allocator import admit_codes as admit
    n, r = _world(group)
    h = codes_local.shape[1]
    codes = all_gather_columns(codes_local.to(torch.int8), group)
    imp = all_gather_columns(importance_local.float(), group)
    sens = all_gather_columns(sensitivity_local.float(), group) if sensitivity_local is not None else None
    prot = all_gather_columns(protected_local.to(torch.uint8), group).bool() if protected_local is not None else None
    out, predicted, evicted = admit(codes, imp, sens, budget_bytes, batch, head_dim, sink_tokens, rd_allocation,
                                    allow_eviction, prot, group_size)
    return out[:, r * h:(r + 1) * h].contiguous(), predicted, evicted


class PeerOutputs:
    """One output buffer ``shape`` = [B, H, S_q, D] per rank (``dtype`` float32, or float16 for
    ``packed_attention(..., out_dtype=torch.float16)``), each mapped into every rank
    of ``group`` through CUDA IPC.  ``ptrs`` is a device int64 array of the ranks' buffer
    addresses as seen from this process, in rank order; ``local`` is this rank's buffer.  A
    kernel that stores into all of them leaves every rank with the full result once all ranks'
    kernels have finished (the caller synchronises the ranks, e.g. with
    ``torch.distributed.barrier``, before reading ``local``).
    Collective: every rank of ``group`` constructs it with the same shape, each on its own GPU.

    The peer buffers are opened by the library (``skv_ipc_open``) on THIS rank's device, which
    enables peer access from it to the owner's GPU; only the handle bytes travel through the
    process group.
    """

    def __init__(self, shape, group=None, device=None, dtype: torch.dtype = torch.float32) -> None:
        from .. import _lib
        from .._device import device_ctx

        if dtype not in (torch.float32, torch.float16):
            raise ValueError(f"PeerOutputs: dtype must be float32 or float16, got {dtype}")
        n, r = _world(group)
        dev = torch.device("cuda", torch.cuda.current_device()) if device is None else torch.device(device)
        self.world, self.rank = n, r
        self.dtype = dtype
        self.local = torch.zeros(tuple(shape), dtype=dtype, device=dev)
        lib = _lib.load()
        hb = lib.skv_ipc_handle_bytes()
        handle = ctypes.create_string_buffer(hb)
        offset = ctypes.c_int64(0)
        with device_ctx(dev):
            st = lib.skv_ipc_export(_lib.ptr(self.local), handle, ctypes.byref(offset))
        # every rank takes part in the exchange, also after a failed export (it sends None), so
        # that a failure raises on all ranks instead of leaving the others in the collective
        mine = (bytes(handle.raw), int(offset.value), int(self.local.numel())) if st == 0 else None
        export_error = None if st == 0 else _lib.last_error()
        entries = [None] * n
        dist.all_gather_object(entries, mine, group=group)
        self._lib = lib
        self._bases = []
        failed = [i for i, e in enumerate(entries) if e is None]
        if failed:
            raise RuntimeError(f"PeerOutputs: ranks {failed} could not export their buffer"
                               + (f" ({export_error})" if export_error else ""))
        ptrs = []
        error = None
        with device_ctx(dev):
            for i, (h, off, numel) in enumerate(entries):
                if numel != self.local.numel():
                    error = ValueError(f"PeerOutputs: rank {i} has {numel} elements, this rank {self.local.numel()}")
                    break
                if i == r:
                    ptrs.append(self.local.data_ptr())
                    continue
                base = ctypes.c_void_p()
                p = ctypes.c_void_p()
                st = lib.skv_ipc_open(ctypes.create_string_buffer(h, hb), off, ctypes.byref(base), ctypes.byref(p))
                if st != 0:
                    error = RuntimeError(f"PeerOutputs: opening rank {i}'s buffer failed: {_lib.last_error()}")
                    break
                self._bases.append(base.value)
                ptrs.append(int(p.value))
        # every rank learns whether every rank mapped all its peers, so that a failure on one rank
        # raises on all of them together instead of leaving the others blocked in a later collective
        opened = [None] * n
        dist.all_gather_object(opened, None if error is None else str(error), group=group)
        failed = [i for i, e in enumerate(opened) if e is not None]
        if failed:
            self.close()
            if error is not None:
                raise error
            raise RuntimeError(f"PeerOutputs: ranks {failed} could not map their peers' buffers ({opened[failed[0]]})")
        self.ptrs = torch.tensor(ptrs, dtype=torch.int64, device=dev)

    @property
    def shape(self):
        return tuple(self.local.shape)

    def close(self) -> None:
        """Unmap the peer buffers (call on every rank after a barrier: no kernel may still be
        storing into them, and no rank may still be reading its own)."""
        from .. import _lib
        from .._device import device_ctx

        bases, self._bases = self._bases, []
        with device_ctx(self.local.device):
            for b in bases:
                _lib.check(self._lib.skv_ipc_close(b), "PeerOutputs.close")
