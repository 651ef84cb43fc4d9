"""Attention over the packed cache, without unpacking it.

In the reference the ``kv_execution="packed"`` path unpacks every layer to
dense fp32 K/V (``PackedKVCache.unpack``, shadowinfer/shadowkv/packed_kv_cache.py:535-577,
called from ``PyTorchModelBackend.forward_step``, core/backends/pytorch_backend.py:302-304)
and then runs ``softmax(q @ k^T / sqrt(D)) @ v`` (shadowinfer/models/simple_diffusion_llm.py:165-169).
``packed_attention`` computes the same result from the packed buckets without the dense
fp32 unpack: one kernel dequantises each head's stored rows once into fp16 tensor-core
tiles (evicted rows are skipped), and a tcgen05 kernel runs the attention over those tiles.
Evicted token-heads behave exactly as the zero rows that ``unpack`` would have produced
(logit 0, value 0).
"""

from __future__ import annotations

import math
from typing import Optional

import torch

from .. import _lib
from .._device import back, device_ctx, on, scratch
from .packed_kv_cache import PackedKVCache


def packed_attention(
    q: torch.Tensor,
    kv_cache: PackedKVCache,
    scale: Optional[float] = None,
    check: bool = True,
    events: Optional[tuple] = None,
    k_new: Optional[torch.Tensor] = None,
    v_new: Optional[torch.Tensor] = None,
    max_ctas: int = 0,
    peer_outputs=None,
    head_offset: int = 0,
    attention_mask: Optional[torch.Tensor] = None,
    fast_k: bool = False,
    one_tile: bool = False,
    fma_exp: bool = False,
    pair: bool = False,
    out_dtype: torch.dtype = torch.float32,
) -> torch.Tensor:
    """Non-causal attention of ``q`` [B, H_q, S_q, D] over a packed cache; returns fp32 [B, H_q, S_q, D].

    ``scale`` defaults to ``1/sqrt(D)``.  ``q`` is used in fp16 (the tensor-core operand type).
    With ``check`` the call synchronises and raises ``RuntimeError`` if the kernel
    reported a pipeline timeout.  ``events``: three CUDA events recorded before the staging
    kernel, between the two kernels and after the attention kernel (timing hook).

    Grouped-query attention: the cache holds H_kv heads and query head h reads KV head
    ``h // (H_q / H_kv)`` (the reference's ``_repeat_kv`` order, diffusion_llama.py:300-308).
    ``k_new`` / ``v_new`` [B, H_kv, S_new, D]: this step's own K/V, attended together with the
    cached rows -- the reference's ``cat((past_k, k), dim=2)`` before the attention
    (simple_diffusion_llm.py:160-169, diffusion_llama.py:376-390) -- staged straight from the
    dense tensors.  ``max_ctas`` caps the persistent attention kernel's CTAs (0: one per SM), to
    leave SMs to work that should run beside it, such as an NCCL all-gather on another stream.

    ``peer_outputs`` (a ``sharding.PeerOutputs`` of shape [B, H_total, S_q, D]): the kernel stores
    each finished output row into every rank's buffer, at heads ``[head_offset, head_offset +
    H_q)``, over NVLink -- the all-gather of head-sharded outputs fused into the attention
    epilogue.  Returns the local buffer, complete only once EVERY rank's call has finished: the
    caller synchronises all ranks (a stream-ordered collective such as a one-element NCCL
    all-reduce after the call, or a stream synchronize plus ``torch.distributed.barrier``)
    before reading it, and again before the next call that writes the same buffers, so that
    no rank overwrites a buffer another rank is still reading.

    ``out_dtype=torch.float16``: the output is written in fp16, each value the fp32 result rounded
    to nearest even (the same bits as ``.half()`` of the fp32 output) -- half the bytes to store
    and, with ``peer_outputs`` (which must then be float16 buffers), half the bytes sent over
    NVLink; it adds about 2.8e-4 of relative L2 error.

    Precision: Q, K, V and the softmax weights P are fp16 tensor-core operands with fp32
    accumulation and softmax; the 16 channels of largest max |K| in each KV head also contribute
    the lo part of K (k - fp16(k)) through one extra K = 16 MMA, so channel outliers of K (a few
    channels ten times larger than the rest) do not turn fp16's 2^-11 rounding into the dominant
    error: relative L2 <= 1e-3 against the reference's fp32 attention.  ``fast_k=True`` skips the
    channel selection and the lo part (K in fp16 only; ~2e-3 with outlier channels).

    ``one_tile=True`` runs the single-query-tile pipeline (units of 128 queries whose next KV
    step's scores are computed while this step's softmax runs) instead of the default two-tile
    one (units of 256 queries, one score buffer per tile); both compute the same result.

    ``fma_exp=True`` (two-tile pipeline) computes a quarter of the softmax exponentials with a
    polynomial on the FMA pipe instead of the MUFU.

    ``attention_mask``: accepted for the reference's signature; like
    ``SimpleDiffusionLLM._compute_block`` (simple_diffusion_llm.py:140-142), which raises when an
    additive mask meets a KV cache, a mask together with a packed past raises ``ValueError``
    (the packed path always attends over a past).
    """
    if q.dim() != 4:
        raise ValueError(f"q must be 4-D [batch, heads, seq, head_dim], got shape {tuple(q.shape)}")
    B, H, S_q, D = (int(x) for x in q.shape)
    c = kv_cache
    H_kv = int(c.num_heads)
    if B != c.batch_size or D != c.head_dim or H_kv <= 0 or H % H_kv:
        raise ValueError(
            "q shape mismatch for packed attention: "
            f"q=(batch={B}, heads={H}, head_dim={D}) cache=({c.batch_size},{c.num_heads},{c.head_dim})"
        )
    if (k_new is None) != (v_new is None):
        raise ValueError("k_new and v_new must be given together")
    if attention_mask is not None:
        raise ValueError("attention_mask is not supported together with kv_cache")
    S_new = 0
    if k_new is not None:
        if k_new.dim() != 4 or tuple(k_new.shape) != tuple(v_new.shape) or \
                (int(k_new.shape[0]), int(k_new.shape[1]), int(k_new.shape[3])) != (B, H_kv, D):
            raise ValueError(
                f"k_new/v_new must be [batch, kv_heads, tokens, head_dim] = [{B}, {H_kv}, T, {D}], "
                f"got {tuple(k_new.shape)} and {tuple(v_new.shape)}"
            )
        S_new = int(k_new.shape[2])
    if scale is None:
        scale = 1.0 / math.sqrt(D)
    if not c.packed_data and S_new == 0:
        # every token-head evicted: unpack() would give zero K/V, so the output is zero
        return torch.zeros(B, H, S_q, D, dtype=out_dtype if out_dtype == torch.float16 else torch.float32,
                           device=q.device)
    dev = c._ensure_state()
    qd = on(q, dev, torch.float16)
    kn = on(k_new, dev, torch.float32) if S_new else None
    vn = on(v_new, dev, torch.float32) if S_new else None
    rows, counts = c._head_index(dev)
    if out_dtype not in (torch.float32, torch.float16):
        raise ValueError(f"out_dtype must be torch.float32 or torch.float16, got {out_dtype}")
    out = torch.empty(B, H, S_q, D, dtype=out_dtype, device=dev)
    err = torch.empty(1, dtype=torch.int32, device=dev)
    arr, _, _ = c._device_arr(dev)
    lib = _lib.load()
    tiles = scratch(lib.skv_packed_attention_scratch_bytes(B, H_kv, c.seq_len + S_new, D), dev)
    stream = _lib.stream_of(dev)
    g = c._int4_group_of()
    flags = ((_lib.SKV_ATTN_FAST_K if fast_k else 0) | (_lib.SKV_ATTN_ONE_TILE if one_tile else 0) |
             (_lib.SKV_ATTN_FMA_EXP if fma_exp else 0) | (_lib.SKV_ATTN_PAIR if pair else 0) |
             (_lib.SKV_ATTN_OUT_F16 if out_dtype == torch.float16 else 0))
    if peer_outputs is not None:
        Bp, Hp, Sp, Dp = peer_outputs.shape
        if getattr(peer_outputs, "dtype", torch.float32) != out_dtype:
            raise ValueError(f"peer output buffers hold {getattr(peer_outputs, 'dtype', torch.float32)}, "
                             f"out_dtype is {out_dtype}")
        if (Bp, Sp, Dp) != (B, S_q, D) or not 0 <= head_offset <= Hp - H:
            raise ValueError(f"peer output buffers {peer_outputs.shape} cannot take heads "
                             f"[{head_offset}, {head_offset + H}) of q {tuple(q.shape)}")
        with device_ctx(dev):
            if events is not None:
                events[0].record()
            st = lib.skv_stage_kv_tiles_gqa(arr, B, H_kv, c.seq_len, D, g, _lib.ptr(rows), _lib.ptr(counts),
                                            _lib.ptr(kn), _lib.ptr(vn), S_new, _lib.ptr(tiles), tiles.numel(), flags,
                                            stream)
            _lib.check(st, "packed_attention")
            if events is not None:
                events[1].record()
            st = lib.skv_attend_kv_tiles_peers(_lib.ptr(qd), B, H, S_q, D, H_kv, c.seq_len, _lib.ptr(rows),
                                               _lib.ptr(counts), S_new, float(scale), _lib.ptr(tiles), tiles.numel(),
                                               _lib.ptr(peer_outputs.ptrs), peer_outputs.world, int(head_offset), Hp,
                                               _lib.ptr(err), int(max_ctas), flags, stream)
            if events is not None:
                events[2].record()
        _lib.check(st, "packed_attention")
        if check:
            code = int(err.item())
            if code:
                raise RuntimeError(f"packed_attention: a pipeline wait timed out inside the kernel (code {code})")
        return peer_outputs.local
    with device_ctx(dev):
        if events is None:
            st = lib.skv_packed_attention_gqa(_lib.ptr(qd), B, H, S_q, D, arr, H_kv, c.seq_len, g, _lib.ptr(rows),
                                              _lib.ptr(counts), _lib.ptr(kn), _lib.ptr(vn), S_new, float(scale),
                                              _lib.ptr(tiles), tiles.numel(), _lib.ptr(out), _lib.ptr(err),
                                              int(max_ctas), flags, stream)
        else:
            events[0].record()
            st = lib.skv_stage_kv_tiles_gqa(arr, B, H_kv, c.seq_len, D, g, _lib.ptr(rows), _lib.ptr(counts),
                                            _lib.ptr(kn), _lib.ptr(vn), S_new, _lib.ptr(tiles), tiles.numel(), flags,
                                            stream)
            _lib.check(st, "packed_attention")
            events[1].record()
            st = lib.skv_attend_kv_tiles_gqa(_lib.ptr(qd), B, H, S_q, D, H_kv, c.seq_len, _lib.ptr(rows),
                                             _lib.ptr(counts), S_new, float(scale), _lib.ptr(tiles), tiles.numel(),
                                             _lib.ptr(out), _lib.ptr(err), int(max_ctas), flags, stream)
            events[2].record()
    _lib.check(st, "packed_attention")
    if check:
        code = int(err.item())
        if code:
            raise RuntimeError(f"packed_attention: a pipeline wait timed out inside the kernel (code {code})")
    return back(out, q.device)


def packed_block_forward(block, hidden: torch.Tensor, kv_cache: PackedKVCache, fast_k: bool = False):
    """``DiffusionTransformerBlock._compute_block`` (shadowinfer/models/simple_diffusion_llm.py:
    122-180) for ``kv_execution="packed"``: the block's own modules (``ln1``, ``q_proj`` /
    ``k_proj`` / ``v_proj`` / ``o_proj``, ``ln2``, ``up_proj`` / ``down_proj``; ``num_heads``,
    ``head_dim``, ``hidden_dim``) run as in the reference, and the attention over
    ``cat((past, new), dim=2)`` reads the past from the packed cache through ``packed_attention``
    (the past is never unpacked, pytorch_backend.py:302-304).

    ``hidden`` [B, S, hidden_dim].  Returns ``(hidden_out, k_new, v_new)``: the reference's
    first three results (its ``k_full`` / ``v_full`` / attention weights are not formed).
    """
    import torch.nn.functional as F

    batch, seq_len, _ = hidden.shape
    nh, hd = int(block.num_heads), int(block.head_dim)
    normed = block.ln1(hidden)
    q = block.q_proj(normed).view(batch, seq_len, nh, hd).transpose(1, 2)
    k = block.k_proj(normed).view(batch, seq_len, nh, hd).transpose(1, 2)
    v = block.v_proj(normed).view(batch, seq_len, nh, hd).transpose(1, 2)
    attn = packed_attention(q, kv_cache, k_new=k, v_new=v, fast_k=fast_k)
    attn_out = attn.transpose(1, 2).contiguous().view(batch, seq_len, int(block.hidden_dim))
    hidden = hidden + block.o_proj(attn_out)
    hidden = hidden + block.down_proj(F.gelu(block.up_proj(block.ln2(hidden))))
    return hidden, k, v
