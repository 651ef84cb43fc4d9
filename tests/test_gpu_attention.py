"""Attention read from the packed cache vs the oracle (unpack + dense float64 attention).

Tolerance: relative L2 error <= 1e-3 over the whole output, the bound the data plane is
held to for attention (fp16 tensor-core operands, fp32 accumulation and softmax).
"""

import numpy as np
import pytest
import torch

from golden_lib import case_arrays, load_pins
from oracle import shadowkv_oracle as O

pytestmark = pytest.mark.gpu

REL_L2_TOL = 1e-3


def rel_l2(a, b):
    a = np.asarray(a, dtype=np.float64)
    b = np.asarray(b, dtype=np.float64)
    return float(np.linalg.norm(a - b) / max(np.linalg.norm(b), 1e-30))


@pytest.fixture(scope="module")
def skv():
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    import shadow_infer_b200.shadowkv as m
    return m


def _pack(skv, k, v, codes, group=16):
    plan = skv.PrecisionPlan.from_codes(torch.from_numpy(codes).cuda())
    return skv.PackedKVCache.pack(torch.from_numpy(k).cuda(), torch.from_numpy(v).cuda(), None, group, plan=plan)["packed_kv"]


@pytest.mark.parametrize("case", sorted(c for c, v in load_pins()["cases"].items() if v["kind"] == "attention"))
def test_attention_matches_reference_fixture(case, skv, golden_small):
    """The reference's own unpack + fp32 attention output, recorded by make_golden.py."""
    a = case_arrays(golden_small, case)
    cache = _pack(skv, a["k"], a["v"], a["codes"])
    out = skv.packed_attention(torch.from_numpy(a["q"]).cuda(), cache)
    assert rel_l2(out.cpu().numpy(), a["out"]) < REL_L2_TOL


CASES = [
    # B, H, S_kv, S_q, D, code probabilities (fp32, fp16, int8, int4, evicted), q scale
    (1, 4, 300, 200, 128, (0.1, 0.2, 0.3, 0.3, 0.1), 1.0),
    (2, 2, 129, 64, 64, (0.0, 0.3, 0.4, 0.2, 0.1), 1.0),
    (1, 2, 1000, 257, 128, (0.05, 0.2, 0.5, 0.2, 0.05), 4.0),     # wide logits: running-max rescales
    (1, 3, 512, 128, 128, (0.0, 0.0, 1.0, 0.0, 0.0), 1.0),       # int8 only
    (1, 3, 512, 128, 128, (0.0, 0.0, 0.0, 1.0, 0.0), 1.0),       # int4 only
    (1, 2, 384, 130, 128, (1.0, 0.0, 0.0, 0.0, 0.0), 1.0),       # fp32 only, ragged query tile
    (3, 1, 77, 33, 64, (0.2, 0.2, 0.2, 0.2, 0.2), 2.0),
]


@pytest.mark.parametrize("B,H,S,SQ,D,probs,qs", CASES)
def test_attention_matches_oracle(skv, B, H, S, SQ, D, probs, qs):
    rng = np.random.default_rng(S * 31 + D)
    k = rng.standard_normal((B, H, S, D)).astype(np.float32)
    v = rng.standard_normal((B, H, S, D)).astype(np.float32)
    k[rng.random(k.shape) < 0.01] *= 8
    codes = rng.choice(5, size=(S, H), p=probs).astype(np.int8)
    q = (rng.standard_normal((B, H, SQ, D)) * qs).astype(np.float16)
    cache = _pack(skv, k, v, codes)
    out = skv.packed_attention(torch.from_numpy(q).cuda(), cache)
    ref = O.packed_attention(q.astype(np.float32), O.pack(k, v, O.plan_from_codes(codes), 16))
    assert rel_l2(out.cpu().numpy(), ref) < REL_L2_TOL


def _check(skv, k, v, codes, q):
    cache = _pack(skv, k, v, codes)
    out = skv.packed_attention(torch.from_numpy(q).cuda(), cache).cpu().numpy()
    ref = O.packed_attention(q.astype(np.float32), O.pack(k, v, O.plan_from_codes(codes), 16))
    assert rel_l2(out, ref) < REL_L2_TOL
    # row by row too: a unit merged from two CTAs' partial results must be right everywhere
    err = np.linalg.norm(out - ref, axis=-1) / np.maximum(np.linalg.norm(ref, axis=-1), 1e-30)
    assert float(err.max()) < 1e-2


@pytest.mark.parametrize("B,D", [(1, 64), (2, 128)])
def test_attention_units_cut_between_ctas(skv, B, D):
    """Heads with 1, 2, 3 and 4 KV tiles: the even split of the steps over the working CTAs
    cuts units in two, whose partial (O, max, sum) are merged; evicted entries in a cut unit
    are counted once."""
    rng = np.random.default_rng(11 + D)
    H, S, SQ = 4, 512, 256
    k = rng.standard_normal((B, H, S, D)).astype(np.float32)
    v = rng.standard_normal((B, H, S, D)).astype(np.float32)
    codes = rng.integers(1, 4, size=(S, H)).astype(np.int8)
    for h in range(H):
        codes[(h + 1) * 128 - 7:, h] = 4               # head h keeps (h+1)*128-7 rows
    q = rng.standard_normal((B, H, SQ, D)).astype(np.float16)
    _check(skv, k, v, codes, q)


def test_attention_more_units_than_sms(skv):
    """160 units of 256 queries (more than one per SM): every CTA's range is cut somewhere."""
    rng = np.random.default_rng(23)
    B, H, S, SQ, D = 1, 8, 384, 5000, 128
    k = rng.standard_normal((B, H, S, D)).astype(np.float32)
    v = rng.standard_normal((B, H, S, D)).astype(np.float32)
    codes = rng.choice(5, size=(S, H), p=(0.0, 0.3, 0.4, 0.25, 0.05)).astype(np.int8)
    q = rng.standard_normal((B, H, SQ, D)).astype(np.float16)
    _check(skv, k, v, codes, q)


@pytest.mark.parametrize("B,H,S,SQ,D,evict", [
    (1, 1, 4096, 256, 128, 0.0),    # one unit of 32 tiles over 8 CTAs: 7 later parts merged
    (1, 2, 2000, 100, 64, 0.2),     # two units, ragged queries, evicted rows in multi-part units
    (2, 3, 1100, 300, 128, 0.05),   # 12 units of 9 tiles: parts of 2-3 CTAs
])
def test_attention_units_spread_over_many_ctas(skv, B, H, S, SQ, D, evict):
    """Few units with many KV tiles: the steps are spread over more CTAs than units, so a
    unit's first part merges the partial results of several later parts."""
    rng = np.random.default_rng(S + H)
    k = rng.standard_normal((B, H, S, D)).astype(np.float32)
    v = rng.standard_normal((B, H, S, D)).astype(np.float32)
    p_keep = (1.0 - evict) / 3
    codes = rng.choice(5, size=(S, H), p=(0.0, p_keep, p_keep, p_keep, evict)).astype(np.int8)
    q = (rng.standard_normal((B, H, SQ, D)) * 2.0).astype(np.float16)
    _check(skv, k, v, codes, q)


def test_attention_all_evicted_head_and_after_evict(skv):
    rng = np.random.default_rng(5)
    B, H, S, D = 1, 3, 200, 128
    k = rng.standard_normal((B, H, S, D)).astype(np.float32)
    v = rng.standard_normal((B, H, S, D)).astype(np.float32)
    codes = rng.integers(1, 4, size=(S, H)).astype(np.int8)
    codes[:, 1] = 4                       # head 1 fully evicted -> uniform weights over zero V
    q = rng.standard_normal((B, H, 150, D)).astype(np.float16)
    cache = _pack(skv, k, v, codes)
    ref_cache = O.pack(k, v, O.plan_from_codes(codes), 16)
    out = skv.packed_attention(torch.from_numpy(q).cuda(), cache).cpu().numpy()
    assert rel_l2(out, O.packed_attention(q.astype(np.float32), ref_cache)) < REL_L2_TOL
    assert np.abs(out[:, 1]).max() == 0.0
    # evict a quarter of the entries: attention follows the compacted buckets
    emask = rng.random((S, H)) < 0.25
    assert cache.evict(torch.from_numpy(emask).cuda()) == O.evict(ref_cache, emask)
    out = skv.packed_attention(torch.from_numpy(q).cuda(), cache).cpu().numpy()
    assert rel_l2(out, O.packed_attention(q.astype(np.float32), ref_cache)) < REL_L2_TOL


def test_attention_shape_errors(skv):
    rng = np.random.default_rng(1)
    k = rng.standard_normal((1, 2, 16, 128)).astype(np.float32)
    cache = _pack(skv, k, k, np.full((16, 2), 2, dtype=np.int8))
    with pytest.raises(ValueError, match="shape mismatch"):
        skv.packed_attention(torch.zeros(1, 3, 8, 128, dtype=torch.float16, device="cuda"), cache)
    with pytest.raises(ValueError, match="4-D"):
        skv.packed_attention(torch.zeros(2, 8, 128, dtype=torch.float16, device="cuda"), cache)


# ---------------------------------------------------------------- grouped-query + this step's K/V
@pytest.mark.parametrize("case", sorted(c for c, v in load_pins()["cases"].items() if v["kind"] == "attention_gqa"))
def test_gqa_attention_matches_reference_fixture(case, skv, golden_small):
    """DiffusionLlamaAttention over cat(packed past, new K/V) with repeated KV heads, as the
    reference computes it (recorded by make_golden.py)."""
    a = case_arrays(golden_small, case)
    cache = _pack(skv, a["k"], a["v"], a["codes"])
    out = skv.packed_attention(torch.from_numpy(a["q"]).cuda(), cache, k_new=torch.from_numpy(a["k_new"]).cuda(),
                               v_new=torch.from_numpy(a["v_new"]).cuda())
    assert out.shape == a["out"].shape
    assert rel_l2(out.cpu().numpy(), a["out"]) < REL_L2_TOL


GQA_CASES = [
    # B, H_kv, n_rep, S_past, S_new, S_q, D, code probabilities
    (1, 4, 4, 500, 128, 128, 128, (0.1, 0.3, 0.3, 0.2, 0.1)),     # new rows fill a whole tile
    (2, 2, 2, 257, 100, 100, 64, (0.0, 0.3, 0.4, 0.3, 0.0)),      # packed rows end mid-tile
    (1, 8, 1, 300, 1, 64, 128, (0.2, 0.2, 0.2, 0.2, 0.2)),        # one new row
    (1, 2, 8, 64, 300, 300, 128, (0.0, 1.0, 0.0, 0.0, 0.0)),      # more new rows than cached
    (1, 4, 2, 200, 0, 150, 64, (0.1, 0.2, 0.3, 0.3, 0.1)),        # GQA without new rows
    (1, 3, 2, 50, 64, 77, 64, (0.0, 0.0, 0.0, 0.0, 1.0)),         # every cached entry evicted
]


@pytest.mark.parametrize("B,H_kv,rep,S,SN,SQ,D,probs", GQA_CASES)
def test_gqa_attention_matches_oracle(skv, B, H_kv, rep, S, SN, SQ, D, probs):
    rng = np.random.default_rng(S * 7 + SN * 3 + rep)
    k = rng.standard_normal((B, H_kv, S, D)).astype(np.float32)
    v = rng.standard_normal((B, H_kv, S, D)).astype(np.float32)
    codes = rng.choice(5, size=(S, H_kv), p=probs).astype(np.int8)
    kn = rng.standard_normal((B, H_kv, SN, D)).astype(np.float32)
    vn = rng.standard_normal((B, H_kv, SN, D)).astype(np.float32)
    q = rng.standard_normal((B, H_kv * rep, SQ, D)).astype(np.float16)
    cache = _pack(skv, k, v, codes)
    out = skv.packed_attention(torch.from_numpy(q).cuda(), cache,
                               k_new=torch.from_numpy(kn).cuda() if SN else None,
                               v_new=torch.from_numpy(vn).cuda() if SN else None).cpu().numpy()
    ref = O.packed_attention(q.astype(np.float32), O.pack(k, v, O.plan_from_codes(codes), 16),
                             k_new=kn if SN else None, v_new=vn if SN else None)
    assert rel_l2(out, ref) < REL_L2_TOL
    err = np.linalg.norm(out - ref, axis=-1) / np.maximum(np.linalg.norm(ref, axis=-1), 1e-30)
    assert float(err.max()) < 1e-2


def test_gqa_argument_checks(skv):
    k = torch.randn(1, 2, 40, 64, device="cuda")
    cache = skv.PackedKVCache.pack(k, k, None, 16, plan=skv.PrecisionPlan.from_codes(
        torch.ones(40, 2, dtype=torch.int8, device="cuda")))["packed_kv"]
    with pytest.raises(ValueError, match="mismatch"):
        skv.packed_attention(torch.randn(1, 3, 8, 64, device="cuda"), cache)          # 3 heads over 2
    with pytest.raises(ValueError, match="k_new"):
        skv.packed_attention(torch.randn(1, 4, 8, 64, device="cuda"), cache, k_new=torch.randn(1, 2, 5, 64))
    with pytest.raises(ValueError, match="k_new/v_new"):
        skv.packed_attention(torch.randn(1, 4, 8, 64, device="cuda"), cache, k_new=torch.randn(1, 4, 5, 64),
                             v_new=torch.randn(1, 4, 5, 64))


def test_attention_with_fewer_ctas(skv):
    """A capped persistent grid (SMs left to other work) gives the same result."""
    rng = np.random.default_rng(77)
    B, H, S, SQ, D = 1, 4, 700, 300, 128
    k = rng.standard_normal((B, H, S, D)).astype(np.float32)
    v = rng.standard_normal((B, H, S, D)).astype(np.float32)
    codes = rng.choice(5, size=(S, H), p=(0.0, 0.3, 0.4, 0.25, 0.05)).astype(np.int8)
    q = torch.from_numpy(rng.standard_normal((B, H, SQ, D)).astype(np.float16)).cuda()
    cache = _pack(skv, k, v, codes)
    ref = O.packed_attention(q.cpu().numpy().astype(np.float32), O.pack(k, v, O.plan_from_codes(codes), 16))
    for ctas in (1, 7, 37, 132):
        out = skv.packed_attention(q, cache, max_ctas=ctas).cpu().numpy()
        assert rel_l2(out, ref) < REL_L2_TOL, ctas


class _TwoBuffers:
    """Two output buffers on one GPU standing in for two ranks' IPC-mapped buffers."""

    def __init__(self, shape, local, dtype=torch.float32):
        self.bufs = [torch.zeros(shape, dtype=dtype, device="cuda") for _ in range(2)]
        self.dtype = dtype
        self.local = self.bufs[local]
        self.shape = tuple(shape)
        self.world = 2
        self.ptrs = torch.tensor([b.data_ptr() for b in self.bufs], dtype=torch.int64, device="cuda")


def _sharded_problem(seed, B, H, S, SQ, D):
    rng = np.random.default_rng(seed)
    k = rng.standard_normal((B, H, S, D)).astype(np.float32)
    v = rng.standard_normal((B, H, S, D)).astype(np.float32)
    codes = rng.choice(5, size=(S, H), p=(0.05, 0.25, 0.4, 0.25, 0.05)).astype(np.int8)
    q = rng.standard_normal((B, H, SQ, D)).astype(np.float16)
    return k, v, codes, q


def test_attention_stores_into_peer_buffers(skv):
    """The fused all-gather epilogue: each head shard's call stores its rows into every buffer,
    so after both shards both buffers hold all heads (identical bits) and match the oracle."""
    B, H, S, SQ, D = 2, 6, 500, 260, 128
    k, v, codes, q = _sharded_problem(5, B, H, S, SQ, D)
    ref = O.packed_attention(q.astype(np.float32), O.pack(k, v, O.plan_from_codes(codes), 16))
    peers = _TwoBuffers((B, H, SQ, D), 0)
    for h0, h1 in ((0, 4), (4, 6)):
        cache = _pack(skv, np.ascontiguousarray(k[:, h0:h1]), np.ascontiguousarray(v[:, h0:h1]),
                      np.ascontiguousarray(codes[:, h0:h1]))
        got = skv.packed_attention(torch.from_numpy(np.ascontiguousarray(q[:, h0:h1])).cuda(), cache,
                                   peer_outputs=peers, head_offset=h0)
        assert got.data_ptr() == peers.local.data_ptr()
    torch.cuda.synchronize()
    assert torch.equal(peers.bufs[0], peers.bufs[1])
    assert rel_l2(peers.bufs[0].cpu().numpy(), ref) < REL_L2_TOL
    with pytest.raises(ValueError, match="peer output buffers"):
        skv.packed_attention(torch.from_numpy(np.ascontiguousarray(q[:, :4])).cuda(), cache, peer_outputs=peers,
                             head_offset=3)


def _peer_worker(rank, world, port, ret):
    import os
    import sys
    import torch.distributed as dist
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    torch.cuda.set_device(rank)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        repo = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
        sys.path.insert(0, repo)
        import shadow_infer_b200.shadowkv as skv
        from shadow_infer_b200.shadowkv.sharding import PeerOutputs, head_range
        B, H, S, SQ, D = 1, 8, 700, 300, 128
        k, v, codes, q = _sharded_problem(9, B, H, S, SQ, D)
        h0, h1 = head_range(H, world, rank)
        peers = PeerOutputs((B, H, SQ, D), device=f"cuda:{rank}")
        cache = _pack(skv, np.ascontiguousarray(k[:, h0:h1]), np.ascontiguousarray(v[:, h0:h1]),
                      np.ascontiguousarray(codes[:, h0:h1]))
        out = skv.packed_attention(torch.from_numpy(np.ascontiguousarray(q[:, h0:h1])).cuda(), cache,
                                   peer_outputs=peers, head_offset=h0)
        torch.cuda.synchronize()
        dist.barrier()                          # every rank's stores have landed
        full = out.cpu()
        dist.barrier()                          # nobody rewrites a buffer another rank still reads
        # the plain exchange: this rank's heads of the output copied into every rank's buffer
        from shadow_infer_b200 import _lib
        mine = out[:, h0:h1].clone()            # a copy: the buffer is cleared below
        peers.local.zero_()
        torch.cuda.synchronize()
        dist.barrier()
        st = _lib.load().skv_peer_store(_lib.ptr(mine), mine.numel() * 4, _lib.ptr(peers.ptrs), world,
                                        h0 * SQ * D * 4, _lib.stream_of(torch.device("cuda", rank)))
        torch.cuda.synchronize()
        dist.barrier()
        plain_ok = st == 0 and torch.equal(peers.local.cpu(), full)
        dist.barrier()                          # nobody unmaps a buffer another rank still reads
        peers.close()
        allf = [torch.empty_like(full) for _ in range(world)]
        dist.all_gather(allf, full)
        ref = O.packed_attention(q.astype(np.float32), O.pack(k, v, O.plan_from_codes(codes), 16))
        ret[rank] = (bool(all(torch.equal(f, full) for f in allf)) and rel_l2(full.numpy(), ref) < REL_L2_TOL
                     and plain_ok)
    finally:
        dist.destroy_process_group()


def test_peer_store_local_destinations(skv):
    """skv_peer_store into two buffers of this GPU at a byte offset: both hold the source there
    and nothing else changes."""
    from shadow_infer_b200 import _lib
    src = torch.randn(3, 1000, 4, device="cuda")
    dst = [torch.full((5000 * 4,), -1.0, device="cuda") for _ in range(2)]
    ptrs = torch.tensor([d.data_ptr() for d in dst], dtype=torch.int64, device="cuda")
    st = _lib.load().skv_peer_store(_lib.ptr(src), src.numel() * 4, _lib.ptr(ptrs), 2, 1000 * 16,
                                    _lib.stream_of(torch.device("cuda", 0)))
    assert st == 0
    torch.cuda.synchronize()
    for d in dst:
        assert torch.equal(d[4000:4000 + src.numel()], src.reshape(-1))
        assert bool((d[:4000] == -1).all()) and bool((d[4000 + src.numel():] == -1).all())
    assert _lib.load().skv_peer_store(_lib.ptr(src), 8, _lib.ptr(ptrs), 2, 0, None) != 0   # not 16-byte sized


def test_attention_peer_outputs_two_gpus(skv):
    """Two ranks (one process per GPU), heads sharded, outputs exchanged by the kernel's own
    stores into the CUDA IPC mappings of each other's buffers (and by the plain copy kernel)."""
    if torch.cuda.device_count() < 2:
        pytest.skip("needs two GPUs")
    import socket
    import torch.multiprocessing as mp
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    port = s.getsockname()[1]
    s.close()
    ctx = mp.get_context("spawn")
    ret = ctx.Manager().dict()
    mp.start_processes(_peer_worker, args=(2, port, ret), nprocs=2, join=True, start_method="spawn")
    assert ret.get(0) and ret.get(1)


@pytest.mark.parametrize("B,H,S,SQ,D,probs,qs", CASES[:4])
def test_attention_fast_k_matches_oracle(skv, B, H, S, SQ, D, probs, qs):
    """K in fp16 only (one MMA chain, two K stages): within 1e-3 on N(0,1) data, and never
    closer to the oracle than the default hi + lo K."""
    rng = np.random.default_rng(S * 31 + D)
    k = rng.standard_normal((B, H, S, D)).astype(np.float32)
    v = rng.standard_normal((B, H, S, D)).astype(np.float32)
    k[rng.random(k.shape) < 0.01] *= 8
    codes = rng.choice(5, size=(S, H), p=probs).astype(np.int8)
    q = (rng.standard_normal((B, H, SQ, D)) * qs).astype(np.float16)
    cache = _pack(skv, k, v, codes)
    ref = O.packed_attention(q.astype(np.float32), O.pack(k, v, O.plan_from_codes(codes), 16))
    fast = skv.packed_attention(torch.from_numpy(q).cuda(), cache, fast_k=True).cpu().numpy()
    exact = skv.packed_attention(torch.from_numpy(q).cuda(), cache).cpu().numpy()
    assert rel_l2(fast, ref) < REL_L2_TOL
    assert rel_l2(exact, ref) <= rel_l2(fast, ref) * 1.05 + 1e-6


def test_attention_mask_with_packed_past_raises(skv):
    rng = np.random.default_rng(3)
    k = rng.standard_normal((1, 2, 40, 64)).astype(np.float32)
    cache = _pack(skv, k, k, np.full((40, 2), 2, dtype=np.int8))
    q = torch.zeros(1, 2, 8, 64, dtype=torch.float16, device="cuda")
    with pytest.raises(ValueError, match="attention_mask is not supported together with kv_cache"):
        skv.packed_attention(q, cache, attention_mask=torch.zeros(8, 40, device="cuda"))


@pytest.mark.parametrize("D,rep,S_new", [(128, 2, 100), (64, 1, 0), (128, 4, 33)])
def test_attention_channel_outliers(skv, D, rep, S_new):
    """K with outlier channels (4 per head, x10) in the packed rows and in this step's own rows:
    the default path (lo part of the 16 largest channels of each KV head) stays within 1e-3 of
    the oracle and is at least as close as K in fp16 only."""
    rng = np.random.default_rng(D + rep + S_new)
    B, H_kv, S, SQ = 2, 2, 700, 190
    k = rng.standard_normal((B, H_kv, S, D)).astype(np.float32)
    v = rng.standard_normal((B, H_kv, S, D)).astype(np.float32)
    kn = rng.standard_normal((B, H_kv, S_new, D)).astype(np.float32)
    vn = rng.standard_normal((B, H_kv, S_new, D)).astype(np.float32)
    for h in range(H_kv):
        ch = rng.choice(D, size=4, replace=False)
        k[:, h, :, ch] *= 10.0
        kn[:, h, :, ch] *= 10.0
    codes = rng.choice(5, size=(S, H_kv), p=(0.05, 0.15, 0.3, 0.45, 0.05)).astype(np.int8)
    q = rng.standard_normal((B, H_kv * rep, SQ, D)).astype(np.float16)
    cache = _pack(skv, k, v, codes)
    kw = dict(k_new=torch.from_numpy(kn).cuda(), v_new=torch.from_numpy(vn).cuda()) if S_new else {}
    ref = O.packed_attention(q.astype(np.float32), O.pack(k, v, O.plan_from_codes(codes), 16),
                             k_new=kn if S_new else None, v_new=vn if S_new else None)
    out = skv.packed_attention(torch.from_numpy(q).cuda(), cache, **kw).cpu().numpy()
    fast = skv.packed_attention(torch.from_numpy(q).cuda(), cache, fast_k=True, **kw).cpu().numpy()
    assert rel_l2(out, ref) < REL_L2_TOL
    assert rel_l2(out, ref) <= rel_l2(fast, ref) + 1e-6


@pytest.mark.parametrize("B,H,S,SQ,D,probs,qs", [CASES[0], CASES[2], CASES[6]])
def test_attention_one_tile_pipeline(skv, B, H, S, SQ, D, probs, qs):
    """The single-query-tile pipeline computes the same attention as the default two-tile one
    (both within 1e-3 of the oracle; they differ only in summation order)."""
    rng = np.random.default_rng(S * 31 + D)
    k = rng.standard_normal((B, H, S, D)).astype(np.float32)
    v = rng.standard_normal((B, H, S, D)).astype(np.float32)
    codes = rng.choice(5, size=(S, H), p=probs).astype(np.int8)
    q = (rng.standard_normal((B, H, SQ, D)) * qs).astype(np.float16)
    cache = _pack(skv, k, v, codes)
    ref = O.packed_attention(q.astype(np.float32), O.pack(k, v, O.plan_from_codes(codes), 16))
    one = skv.packed_attention(torch.from_numpy(q).cuda(), cache).cpu().numpy()
    two = skv.packed_attention(torch.from_numpy(q).cuda(), cache, one_tile=True).cpu().numpy()
    assert rel_l2(one, ref) < REL_L2_TOL and rel_l2(two, ref) < REL_L2_TOL
    assert rel_l2(one, two) < 1e-4


@pytest.mark.parametrize("B,H,S,SQ,D,probs,qs", [CASES[0], CASES[2], CASES[6]])
def test_attention_fma_exponentials(skv, B, H, S, SQ, D, probs, qs):
    """A quarter of the softmax exponentials on the FMA pipe (degree-3 polynomial): same bar."""
    rng = np.random.default_rng(S * 31 + D)
    k = rng.standard_normal((B, H, S, D)).astype(np.float32)
    v = rng.standard_normal((B, H, S, D)).astype(np.float32)
    codes = rng.choice(5, size=(S, H), p=probs).astype(np.int8)
    q = (rng.standard_normal((B, H, SQ, D)) * qs).astype(np.float16)
    cache = _pack(skv, k, v, codes)
    ref = O.packed_attention(q.astype(np.float32), O.pack(k, v, O.plan_from_codes(codes), 16))
    out = skv.packed_attention(torch.from_numpy(q).cuda(), cache, fma_exp=True).cpu().numpy()
    assert rel_l2(out, ref) < REL_L2_TOL


# ---------------------------------------------------------------- the CTA-pair pipeline
PAIR_CASES = [c for c in CASES if c[4] == 128]


# P is rounded to fp16 relative to a running row max; the default pipeline's stream-K parts each
# start their own, so the two pipelines round P differently: about 1.4e-4 relative each (the
# output is an average of random V rows, which does not shrink the relative error), ~2e-4 apart.
PAIR_VS_DEFAULT_TOL = 5e-4


@pytest.mark.parametrize("B,H,S,SQ,D,probs,qs", PAIR_CASES)
@pytest.mark.parametrize("outliers", [False, True])
def test_attention_pair_pipeline(skv, B, H, S, SQ, D, probs, qs, outliers):
    """Two CTAs per unit of 256 queries (tensor-core MMAs over the pair): the same attention as
    the default two-tile pipeline, within 1e-3 of the oracle.  With outlier channels (four K
    channels ten times larger) the lo correction is what keeps the error below 1e-3: K in
    fp16 alone is ~2e-3 off, so a pair that dropped the lo MMA of either CTA's keys fails."""
    rng = np.random.default_rng(S * 31 + D)
    k = rng.standard_normal((B, H, S, D)).astype(np.float32)
    if outliers:
        k[..., [3, 17, 50, 99]] *= 10.0
    v = rng.standard_normal((B, H, S, D)).astype(np.float32)
    codes = rng.choice(5, size=(S, H), p=probs).astype(np.int8)
    q = (rng.standard_normal((B, H, SQ, D)) * qs).astype(np.float16)
    cache = _pack(skv, k, v, codes)
    ref = O.packed_attention(q.astype(np.float32), O.pack(k, v, O.plan_from_codes(codes), 16))
    qd = torch.from_numpy(q).cuda()
    two = skv.packed_attention(qd, cache).cpu().numpy()
    pair = skv.packed_attention(qd, cache, pair=True).cpu().numpy()
    assert rel_l2(pair, ref) < REL_L2_TOL
    assert rel_l2(pair, ref) < 1.5 * rel_l2(two, ref) + 1e-4
    assert rel_l2(pair, two) < PAIR_VS_DEFAULT_TOL
    fast = skv.packed_attention(qd, cache, pair=True, fast_k=True).cpu().numpy()
    assert rel_l2(fast, skv.packed_attention(qd, cache, fast_k=True).cpu().numpy()) < PAIR_VS_DEFAULT_TOL


@pytest.mark.parametrize("B,H_kv,rep,S,SN,SQ,D,probs", [c for c in GQA_CASES if c[6] == 128])
def test_attention_pair_gqa_new_rows(skv, B, H_kv, rep, S, SN, SQ, D, probs):
    rng = np.random.default_rng(S * 7 + SN * 3 + rep)
    k = rng.standard_normal((B, H_kv, S, D)).astype(np.float32)
    v = rng.standard_normal((B, H_kv, S, D)).astype(np.float32)
    codes = rng.choice(5, size=(S, H_kv), p=probs).astype(np.int8)
    kn = rng.standard_normal((B, H_kv, SN, D)).astype(np.float32)
    vn = rng.standard_normal((B, H_kv, SN, D)).astype(np.float32)
    q = rng.standard_normal((B, H_kv * rep, SQ, D)).astype(np.float16)
    cache = _pack(skv, k, v, codes)
    out = skv.packed_attention(torch.from_numpy(q).cuda(), cache, pair=True,
                               k_new=torch.from_numpy(kn).cuda() if SN else None,
                               v_new=torch.from_numpy(vn).cuda() if SN else None).cpu().numpy()
    ref = O.packed_attention(q.astype(np.float32), O.pack(k, v, O.plan_from_codes(codes), 16),
                             k_new=kn if SN else None, v_new=vn if SN else None)
    assert rel_l2(out, ref) < REL_L2_TOL


def test_attention_pair_evicted_head_few_pairs_and_peers(skv):
    """A fully evicted head (zero output), units spread over two pairs only (max_ctas=4), and the
    fused store into two output buffers."""
    rng = np.random.default_rng(9)
    B, H, S, SQ, D = 2, 3, 700, 600, 128
    k = rng.standard_normal((B, H, S, D)).astype(np.float32)
    v = rng.standard_normal((B, H, S, D)).astype(np.float32)
    codes = rng.integers(0, 5, size=(S, H)).astype(np.int8)
    codes[:, 1] = 4
    q = rng.standard_normal((B, H, SQ, D)).astype(np.float16)
    cache = _pack(skv, k, v, codes)
    ref = O.packed_attention(q.astype(np.float32), O.pack(k, v, O.plan_from_codes(codes), 16))
    qd = torch.from_numpy(q).cuda()
    for mc in (0, 4):
        out = skv.packed_attention(qd, cache, pair=True, max_ctas=mc).cpu().numpy()
        assert rel_l2(out, ref) < REL_L2_TOL
        assert np.abs(out[:, 1]).max() == 0.0
    peers = _TwoBuffers((B, H, SQ, D), 0)
    skv.packed_attention(qd, cache, pair=True, peer_outputs=peers, head_offset=0)
    torch.cuda.synchronize()
    assert torch.equal(peers.bufs[0], peers.bufs[1])
    assert rel_l2(peers.bufs[0].cpu().numpy(), ref) < REL_L2_TOL


def test_attention_pair_rejects_other_shapes_and_flags(skv):
    rng = np.random.default_rng(2)
    k = rng.standard_normal((1, 2, 64, 64)).astype(np.float32)
    cache = _pack(skv, k, k, np.full((64, 2), 2, dtype=np.int8))
    with pytest.raises(RuntimeError, match="head_dim 128"):
        skv.packed_attention(torch.zeros(1, 2, 8, 64, dtype=torch.float16, device="cuda"), cache, pair=True)
    k = rng.standard_normal((1, 2, 64, 128)).astype(np.float32)
    cache = _pack(skv, k, k, np.full((64, 2), 2, dtype=np.int8))
    with pytest.raises(ValueError, match="CTA-pair"):
        skv.packed_attention(torch.zeros(1, 2, 8, 128, dtype=torch.float16, device="cuda"), cache, pair=True,
                             one_tile=True)


@pytest.mark.parametrize("S,H", [(1, 1), (77, 3), (1024, 2), (5000, 4), (32768, 4), (2048, 32), (40000, 1)])
def test_head_index_rows_and_counts(skv, S, H):
    """skv_head_index: per head, the slots of the stored entries in token order, fp32 entries first,
    then fp16, int8, int4 (the order staging reads them), and the five counts per head (the four
    precisions and the evicted entries); heads are split over several blocks when there are few."""
    from shadow_infer_b200 import _lib
    rng = np.random.default_rng(S + 7 * H)
    codes = rng.integers(0, 5, size=(S, H))
    slot = np.where(codes == 4, -1, (np.arange(S * H).reshape(S, H) << 2) | np.minimum(codes, 3)).astype(np.int32)
    sd = torch.from_numpy(slot).cuda()
    rows = torch.full((H * S,), -7, dtype=torch.int32, device="cuda")
    counts = torch.empty(H * 5, dtype=torch.int32, device="cuda")
    lib = _lib.load()
    _lib.check(lib.skv_head_index(_lib.ptr(sd), S, H, _lib.ptr(rows), _lib.ptr(counts),
                                  _lib.stream_of(torch.device("cuda"))), "head_index")
    rows, counts = rows.cpu().numpy().reshape(H, S), counts.cpu().numpy().reshape(H, 5)
    for h in range(H):
        want = np.concatenate([slot[codes[:, h] == k, h] for k in range(4)])
        assert np.array_equal(rows[h, :want.size], want)
        assert np.all(rows[h, want.size:] == -7)
        assert counts[h].tolist() == [int(np.sum(codes[:, h] == k)) for k in range(5)]


# ---------------------------------------------------------------- fp16 output
@pytest.mark.parametrize("pipeline", ["default", "one_tile", "pair"])
@pytest.mark.parametrize("B,H,S,SQ,D,probs,qs", [CASES[0], CASES[2], CASES[6]])
def test_attention_fp16_output_is_the_rounded_fp32_output(skv, pipeline, B, H, S, SQ, D, probs, qs):
    """out_dtype=float16 stores the same results rounded to nearest even: bit-identical to
    .half() of the fp32 output, through every epilogue path (whole units, units merged from
    stream-K parts over two and over several CTAs, the two-buffer peer epilogue)."""
    if pipeline == "pair" and D != 128:
        pytest.skip("the CTA-pair pipeline is head_dim 128 only")
    rng = np.random.default_rng(S * 31 + D)
    k = rng.standard_normal((B, H, S, D)).astype(np.float32)
    v = rng.standard_normal((B, H, S, D)).astype(np.float32)
    codes = rng.choice(5, size=(S, H), p=probs).astype(np.int8)
    q = (rng.standard_normal((B, H, SQ, D)) * qs).astype(np.float16)
    cache = _pack(skv, k, v, codes)
    qd = torch.from_numpy(q).cuda()
    kw = {"one_tile": pipeline == "one_tile", "pair": pipeline == "pair"}
    ref = O.packed_attention(q.astype(np.float32), O.pack(k, v, O.plan_from_codes(codes), 16))
    for mc in (0, 2, 4, 7):
        o32 = skv.packed_attention(qd, cache, max_ctas=mc, **kw)
        o16 = skv.packed_attention(qd, cache, max_ctas=mc, out_dtype=torch.float16, **kw)
        assert o16.dtype == torch.float16 and torch.equal(o16, o32.half()), mc
        assert rel_l2(o16.float().cpu().numpy(), ref) < REL_L2_TOL
    peers = _TwoBuffers((B, H, SQ, D), 1, dtype=torch.float16)
    skv.packed_attention(qd, cache, peer_outputs=peers, head_offset=0, out_dtype=torch.float16, **kw)
    torch.cuda.synchronize()
    o32 = skv.packed_attention(qd, cache, **kw)
    assert torch.equal(peers.bufs[0], o32.half()) and torch.equal(peers.bufs[1], o32.half())
    with pytest.raises(ValueError, match="out_dtype"):
        skv.packed_attention(qd, cache, peer_outputs=peers, head_offset=0, **kw)
    with pytest.raises(ValueError, match="out_dtype"):
        skv.packed_attention(qd, cache, out_dtype=torch.bfloat16)
