"""Head sharding host logic on a world-size-2 gloo group (CPU, no GPU).

The admission itself is replaced by the CPU oracle here (the kernel needs a GPU);
what is checked is the exchange: every rank assembles the same full [S, H]
problem, keeps its own columns, and the result equals the unsharded admission.
"""

import os
import socket

import numpy as np
import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    port = s.getsockname()[1]
    s.close()
    return port


def _oracle_admit(codes, imp, sens, budget, batch, head_dim, sink, rd, evict, prot, group):
    from oracle import shadowkv_oracle as O
    out, pred, ev = O.admit_codes(codes.numpy(), imp.numpy(), None if sens is None else sens.numpy(), budget,
                                  batch, head_dim, sink_tokens=sink, rd_allocation=rd, allow_eviction=evict,
                                  protected_mask=None if prot is None else prot.numpy(), group_size=group)
    return torch.from_numpy(out), pred, ev


def _worker(rank, world, port, ret):
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        import sys
        repo = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
        sys.path.insert(0, repo)
        from shadow_infer_b200.shadowkv.sharding import (admit_codes_sharded, all_gather_columns,
                                                         all_gather_heads, head_range)
        g = torch.Generator().manual_seed(11)
        S, H, B, D = 64, 8, 2, 16
        full = torch.randn(B, H, S, D, generator=g)
        codes = torch.randint(0, 5, (S, H), generator=g, dtype=torch.int8)
        imp = torch.rand(S, H, generator=g)
        sens = torch.rand(S, H, generator=g)
        prot = torch.rand(S, H, generator=g) < 0.1
        h0, h1 = head_range(H, world, rank)
        ok = torch.equal(all_gather_heads(full[:, h0:h1].clone()), full)
        ok &= torch.equal(all_gather_columns(imp[:, h0:h1].clone()), imp)
        budget = 5000
        local, pred, ev = admit_codes_sharded(codes[:, h0:h1], imp[:, h0:h1], sens[:, h0:h1], budget, B, D,
                                              sink_tokens=3, allow_eviction=True, protected_local=prot[:, h0:h1],
                                              admit=_oracle_admit)
        want, wpred, wev = _oracle_admit(codes, imp, sens, budget, B, D, 3, True, True, prot, 16)
        ok &= torch.equal(local, want[:, h0:h1]) and (pred, ev) == (wpred, wev)
        ret[rank] = bool(ok)
    finally:
        dist.destroy_process_group()


def test_head_sharding_gloo_world2():
    world = 2
    ctx = mp.get_context("spawn")
    manager = ctx.Manager()
    ret = manager.dict()
    procs = [ctx.Process(target=_worker, args=(r, world, PORT, ret)) for r in range(world)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(timeout=120)
        assert p.exitcode == 0
    assert ret.get(0) and ret.get(1)


PORT = _free_port()


def test_head_range_validation():
    from shadow_infer_b200.shadowkv.sharding import head_range
    assert head_range(32, 4, 3) == (24, 32)
    with pytest.raises(ValueError):
        head_range(30, 4, 0)
    with pytest.raises(ValueError):
        head_range(32, 4, 4)


def test_peer_outputs_rejects_other_dtypes_before_any_collective():
    """PeerOutputs takes float32 or float16 buffers; another dtype raises at once, on every rank
    alike, before any handle exchange (so no rank is left waiting in a collective)."""
    from shadow_infer_b200.shadowkv.sharding import PeerOutputs
    with pytest.raises(ValueError, match="float32 or float16"):
        PeerOutputs((1, 2, 8, 64), dtype=torch.bfloat16)
