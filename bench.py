#!/usr/bin/env python
"""Benchmark of the ShadowKV packed-KV data plane on B200.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl b200|reference]

One STEP is one pass of the data plane over one layer of the cfg2 workload
(B=1, H=32, S=8192, D=128 fp32 K/V, inputs resident in HBM):

    allocate_precision_codes -> kv_sensitivity -> admit_codes (30 % fp16 budget,
    hard eviction, 4 sink tokens) -> PrecisionPlan.from_codes (50 % reuse mask)
    -> PackedKVCache.pack -> apply_reuse_mask (previous step's cache) -> unpack

``value`` is algorithmic bytes per step / device time (GB/s).  With N GPUs
(torchrun) every rank packs its own layer (layers are independent objects, so
there is no collective on the data path): weak scaling, value = N layers'
bytes / max-over-ranks time.  ``e2e`` is the same step through the public API
from pinned host buffers (K, V, importance, reuse mask copied in; the packed
payload copied out).  ``roofline`` covers the pack kernel (the dominant
kernel), timed with CUDA events around each launch in the timed region.
``--impl reference`` times the CPU restatement of the reference algorithm
(``oracle/``) over the same layer, its heads split over one single-threaded
worker process per host core (up to 8), on rank 0 only.

The line also carries ``attention``: packed attention over one cfg3 layer
(B=1, H=32, S=4096, D=128, codes 20/50/30 % fp16/int8/int4), heads sharded over
the ranks, the outputs all-gathered by the kernel's own stores into every rank's
buffer (CUDA IPC mappings, NVLink), as tokens/s of the 32-layer
stack and as tensor-core roofline of the kernel; ``global_budget``:
KVCacheManager.enforce_global_budget over 8 packed layers of that shape;
``paged_store``: the PagedKVStore append-mode run of the reference's own paged
benchmark shape plus its gather / append kernels at the cfg2 layer shape; and
``decisions``: decide_reuse_per_token over the cfg2 layer and
compute_irap_importance over cfg3-shaped attention probabilities.
"""

from __future__ import annotations

import argparse
import json
import os
import statistics
import subprocess
import sys
import threading
import time

REPO = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, REPO)

METRIC = "packed-KV GB/s (compress+pack, unpack) & packed-attn tokens/s at 1/2/4/8 B200, % roofline"
FALLBACK_HBM_GBS = 6650.0


def parse_args():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=200)
    ap.add_argument("--warmup", type=int, default=20)
    ap.add_argument("--impl", choices=("b200", "reference"), default="b200")
    ap.add_argument("--ref-heads", type=int, default=8, help="head slice timed by the CPU reference arm")
    ap.add_argument("--no-attention", action="store_true",
                    help="skip the packed-attention, global-budget and paged-store phases")
    ap.add_argument("--phase", choices=("all", "paged", "paged-kernels", "decisions"), default="all",
                    help="'paged' / 'paged-kernels' / 'decisions': print only that phase (the paged store, its "
                         "kernels at the cfg2 shape, the decision inputs) as the JSON line; for profiling")
    return ap.parse_args()


# ----------------------------------------------------------------------------------- peaks
def hbm_peak():
    path = os.path.join(REPO, "MEASURED_PEAKS.json")
    try:
        with open(path) as f:
            return float(json.load(f)["hbm_gbs"]), "measured"
    except Exception:
        return FALLBACK_HBM_GBS, "fallback"


def committed_traffic(name: str):
    """Per-launch DRAM bytes of a kernel from its committed ncu summary (profiles/)."""
    path = os.path.join(REPO, "profiles", name)
    try:
        for line in open(path):
            if line.startswith("traffic_bytes_per_launch:"):
                return int(line.split(":", 1)[1].strip())
    except OSError:
        pass
    return None


# ---------------------------------------------------------------------------------- clocks
class ClockSampler:
    """Samples nvidia-smi SM clocks and throttle reasons while the benchmark runs."""

    FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, index: int):
        self.index = index
        self.rows = []
        self._proc = None
        self._thread = None

    def start(self):
        try:
            self._proc = subprocess.Popen(
                ["nvidia-smi", f"--id={self.index}", f"--query-gpu={self.FIELDS}", "--format=csv,noheader,nounits",
                 "-lms", "100"], stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
        except OSError:
            self._proc = None
            return
        self._thread = threading.Thread(target=self._read, daemon=True)
        self._thread.start()

    def _read(self):
        for line in self._proc.stdout:
            parts = [p.strip() for p in line.split(",")]
            if len(parts) >= 9:
                self.rows.append(parts)

    def stop(self):
        if self._proc is not None:
            self._proc.terminate()
            try:
                self._proc.wait(timeout=5)
            except subprocess.TimeoutExpired:
                self._proc.kill()
        if self._thread is not None:
            self._thread.join(timeout=5)

    def summary(self):
        def num(x):
            try:
                return float(x)
            except ValueError:
                return None
        sm = [num(r[1]) for r in self.rows if num(r[1])]
        mx = [num(r[2]) for r in self.rows if num(r[2])]
        names = ("hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap")
        reasons = sorted({names[i] for r in self.rows for i in range(4) if r[5 + i].lower() == "active"})
        return {"sm_mhz": statistics.median(sm) if sm else None, "sm_max_mhz": max(mx) if mx else None,
                "reasons": reasons, "samples": len(self.rows)}


# ------------------------------------------------------------------------- algorithmic bytes
def step_bytes(B, H, S, D, packed_bytes, n_kept, n_reuse_rows_bytes, n_reuse):
    """Algorithmic HBM bytes of one data-plane step, per kernel."""
    N = S * H
    fp32 = 2 * B * H * S * D * 4
    parts = {
        "allocate": 4 * N + N,
        "sensitivity": fp32 + 4 * N,
        "admission": 9 * N + 4 * N,
        "plan": N + N + 8 * N + 4 * N + 8 * n_reuse,
        "pack": fp32 + N + packed_bytes + 8 * n_kept,
        "reuse": N + 2 * n_reuse_rows_bytes,
        "unpack": packed_bytes + 8 * n_kept + fp32,
    }
    return parts


# ------------------------------------------------------------------------------- reference
def reference_sample(I, heads: int, h0: int = 0):
    """The CPU oracle pipeline on heads [h0, h0 + heads) of the workload (the budget scaled to the
    slice); returns a callable that runs one step and returns (seconds, algorithmic bytes)."""
    import numpy as np
    from oracle import shadowkv_oracle as O

    sl = slice(h0, h0 + heads)
    k = np.ascontiguousarray(I["k"][:, sl].numpy())
    v = np.ascontiguousarray(I["v"][:, sl].numpy())
    imp = np.ascontiguousarray(I["importance"][:, sl].numpy())
    reuse = np.ascontiguousarray(I["reuse"][:, sl].numpy())
    B, H, S, D = k.shape
    budget = I["budget"] * heads // I["k"].shape[1]
    codes0 = O.allocate_precision_codes(imp, "balanced")
    adm, _, _ = O.admit_codes(codes0, imp, O.kv_sensitivity(k, v), budget, B, D, sink_tokens=4,
                              allow_eviction=True)
    prev = O.pack(np.ascontiguousarray(I["k_prev"][:, sl].numpy()),
                  np.ascontiguousarray(I["v_prev"][:, sl].numpy()), O.plan_from_codes(adm), 16)

    def run():
        t0 = time.perf_counter()
        codes = O.allocate_precision_codes(imp, "balanced")
        sens = O.kv_sensitivity(k, v)
        a, _, _ = O.admit_codes(codes, imp, sens, budget, B, D, sink_tokens=4, allow_eviction=True)
        plan = O.plan_from_codes(a, reuse)
        cache = O.pack(k, v, plan, 16)
        st = O.apply_reuse_mask(cache, prev, reuse)
        O.unpack(cache)
        dt = time.perf_counter() - t0
        kept = sum(len(d["indices"]) for d in cache.packed_data.values())
        flagged = reuse & (a < 4)   # previous cache holds the same codes: every flagged entry is copied
        assert st["applied"] == int(flagged.sum())
        reuse_bytes = int(O.code_costs(B, D, 16)[a[flagged].astype(np.int64)].sum())
        parts = step_bytes(B, H, S, D, cache.memory_bytes(), kept, reuse_bytes, int(reuse.sum()))
        return dt, sum(parts.values())

    return run


_REF_RUN = None


def _ref_worker_init(heads: int, h0: int) -> None:
    """Reference-arm worker: one thread, its own copy of the cfg2 inputs, one head slice."""
    global _REF_RUN
    import torch
    torch.set_num_threads(1)
    from shadow_infer_b200 import workloads as W
    I = W.cfg2_inputs()
    _REF_RUN = reference_sample(I, heads, h0)
    del I


def _ref_worker_step(_):
    return _REF_RUN()


def run_reference(args):
    """The CPU restatement of the reference path over the whole cfg2 layer, its heads split over
    one single-threaded worker process per host core (up to 8, heads dividing evenly); a step is
    every worker's pass over its slice, timed on the wall clock around all of them."""
    rank = int(os.environ.get("RANK", "0"))
    if rank != 0:
        return 0
    import multiprocessing as mp
    from shadow_infer_b200 import workloads as W

    H = W.CONFIGS["cfg2"]["H"]
    workers = 1
    for w in (8, 4, 2, 1):
        if w <= (os.cpu_count() or 1) and H % w == 0:
            workers = w
            break
    heads = H // workers
    for var in ("OMP_NUM_THREADS", "OPENBLAS_NUM_THREADS", "MKL_NUM_THREADS"):
        os.environ[var] = "1"           # inherited by the workers: one thread each
    ctx = mp.get_context("spawn")
    # one single-process pool per slice, so that each worker's initializer builds its own slice
    pools = [ctx.Pool(1, initializer=_ref_worker_init, initargs=(heads, i * heads)) for i in range(workers)]
    try:
        def step():
            t0 = time.perf_counter()
            res = [p.apply_async(_ref_worker_step, (0,)) for p in pools]
            out = [r.get() for r in res]
            return time.perf_counter() - t0, sum(b for _, b in out)
        for _ in range(max(args.warmup, 1)):
            step()
        times, nbytes = [], 0
        for _ in range(args.steps):
            dt, nbytes = step()
            times.append(dt)
    finally:
        for p in pools:
            p.close()
            p.join()
    total = sum(times)
    value = nbytes * args.steps / total / 1e9
    sample = (f"CPU oracle (numpy restatement of the reference path) on the whole cfg2 layer (B1 H{H} S8192 "
              f"D128), {workers} single-threaded worker processes of {heads} heads each, per step")
    line = {
        "metric": METRIC, "value": value, "unit": "GB/s", "impl": "reference", "n_gpus": args.gpus,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": 1e3 * total / args.steps,
        "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "f32", "data": "synthetic",
        "config": {"workload": "cfg2 data-plane step", "B": 1, "H": H, "S": 8192, "D": 128},
        "cpu_baseline": {"value": value, "unit": "GB/s", "cores": workers, "kind": "port", "sample": sample},
        "e2e": {"value": value, "unit": "GB/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }
    print(json.dumps(line), flush=True)
    return 0


# ------------------------------------------------------------------------------- attention
def attention_phase(args, world, rank, dev, dist, lib, tensor_peak):
    """Packed attention on one cfg3 layer, heads sharded over ranks, outputs all-gathered.

    One step = the layer's attention over this rank's heads; with N > 1 its epilogue stores
    every output row into all ranks' fp32 [B, H, S, D] buffers (CUDA IPC mappings over NVLink),
    so the all-gather runs inside the kernel, overlapped with the attention math.
    """
    import torch

    from shadow_infer_b200 import workloads as W
    from shadow_infer_b200.shadowkv import PackedKVCache, PrecisionPlan, packed_attention
    from shadow_infer_b200.shadowkv.shadowkv_agent import allocate_precision_codes

    c = W.CONFIGS["cfg3"]
    B, H, S, D, L = c["B"], c["H"], c["S"], c["D"], c["layers"]
    if H % world:
        raise ValueError(f"{H} heads do not shard over {world} GPUs")
    hs, h0 = H // world, rank * (H // world)
    k, v = W.kv_tensors(B, H, S, D, 0)
    imp = W.importance_map(S, H, 0, c["fractions"])
    q = W.queries(B, H, S, D, 0)
    k, v = k[:, h0:h0 + hs].contiguous(), v[:, h0:h0 + hs].contiguous()
    codes = allocate_precision_codes(imp[:, h0:h0 + hs].contiguous().to(dev), "balanced")
    cache = PackedKVCache.pack(k.to(dev), v.to(dev), None, c["group"], plan=PrecisionPlan.from_codes(codes))["packed_kv"]
    qd = q[:, h0:h0 + hs].contiguous().to(dev)
    packed_attention(qd, cache)                        # builds the head index, checks the error word
    # N > 1: the all-gather of the head-sharded outputs is fused into the attention epilogue --
    # every finished row is stored into all ranks' [B, H, S, D] buffers over NVLink
    # (all ranks agree: if any rank cannot map its peers' buffers, every rank falls back to the
    # NCCL all-gather after the kernel, so that all ranks keep taking the same collective steps)
    from shadow_infer_b200.shadowkv.sharding import PeerOutputs, all_gather_heads
    peers, exchange = None, "none"
    if world > 1:
        err = None
        try:
            peers = PeerOutputs((B, H, S, D), device=dev)
        except Exception as e:          # noqa: BLE001 - reported in the line, then the fallback runs
            err = f"{type(e).__name__}: {e}"
        flag = torch.tensor([0 if err else 1], device=dev, dtype=torch.int32)
        dist.all_reduce(flag, op=dist.ReduceOp.MIN)
        if int(flag.item()) == 1:
            exchange = "fused epilogue stores into every rank's buffer (CUDA IPC, NVLink)"
        else:
            if peers is not None:
                dist.barrier()
                peers.close()
                peers = None
            exchange = "NCCL all-gather after the kernel (peer mapping failed" + (f": {err})" if err else " on a peer)")
    gathered = torch.empty(B, H, S, D, dtype=torch.float32, device=dev) if world > 1 and peers is None else None
    steps = max(3, min(args.steps, 32))
    kev = [tuple(torch.cuda.Event(enable_timing=True) for _ in range(3)) for _ in range(steps)]
    sms = torch.cuda.get_device_properties(dev).multi_processor_count

    def step(i=None):
        # events: before the staging kernel, between the two kernels, after the attention kernel
        out = packed_attention(qd, cache, check=False, events=kev[i] if i is not None else None,
                               peer_outputs=peers, head_offset=h0)
        if gathered is not None:
            all_gather_heads(out, out=gathered)
        return out

    for _ in range(3):
        step()
    torch.cuda.synchronize()
    if world > 1:
        dist.barrier()
    t0 = torch.cuda.Event(enable_timing=True)
    t1 = torch.cuda.Event(enable_timing=True)
    n0 = lib.skv_launch_count()
    t0.record()
    for i in range(steps):
        step(i)
    t1.record()
    torch.cuda.synchronize()
    launches = lib.skv_launch_count() - n0
    packed_attention(qd, cache, peer_outputs=peers, head_offset=h0)   # error word of the last launch
    if world > 1:
        dist.barrier()
        if peers is not None:
            peers.close()
    ms = torch.tensor([t0.elapsed_time(t1) / steps], device=dev, dtype=torch.float64)
    if world > 1:
        dist.all_reduce(ms, op=dist.ReduceOp.MAX)
    ms = float(ms.item())
    stage_ms = statistics.mean(a.elapsed_time(b) for a, b, _ in kev)
    kms = statistics.mean(b.elapsed_time(c) for _, b, c in kev)
    flops_rank = 4.0 * B * hs * S * S * D
    # staging kernel: reads the packed rows, writes fp16 K/V tiles (evicted entries skipped)
    stored = int(sum(cache._count.values()))
    stage_bytes = cache.memory_bytes() + stored * 4 + stored * 2 * B * D * 2
    res = {
        "metric": "packed-attn tokens/s (32-layer stack, cfg3)",
        "value": B * S / (L * ms / 1e3), "unit": "tokens/s", "ms_per_layer": ms, "steps": steps,
        "scaling": "strong (heads sharded over GPUs; outputs all-gathered to every rank)",
        "exchange": exchange,
        "attention_ctas": sms,
        "config": {"workload": "cfg3: packed K/V codes 20/50/30 fp16/int8/int4, fp16 queries, non-causal",
                   "B": B, "H": H, "S_q": S, "S_kv": S, "D": D, "layers": L, "heads_per_gpu": hs},
        "roofline": {"kernel": "packed_attention_kernel", "bound": "tensor",
                     "achieved": flops_rank / (kms / 1e3) / 1e12, "peak": tensor_peak[0], "unit": "TFLOP/s",
                     "frac": flops_rank / (kms / 1e3) / 1e12 / tensor_peak[0],
                     "peak_source": tensor_peak[1], "avg_launch_ms": kms, "flops_per_launch": flops_rank,
                     "traffic": committed_traffic("packed_attention_kernel_cfg3.md")},
        "staging": {"kernel": "stage_tiles_kernel", "bound": "hbm", "avg_launch_ms": stage_ms,
                    "algorithmic_bytes": stage_bytes, "achieved_gbs": stage_bytes / (stage_ms / 1e3) / 1e9,
                    "traffic": committed_traffic("stage_tiles_kernel_cfg3.md")},
        "gpu_launches": launches,
        "output_dtype": "f32",
    }
    if world == 1 and rank == 0:
        import numpy as np
        from oracle import shadowkv_oracle as O

        ko, vo = k[:, :1].numpy().copy(), v[:, :1].numpy().copy()
        co = codes[:, :1].cpu().numpy()
        cache_o = O.pack(ko, vo, O.plan_from_codes(co), c["group"])
        qo = q[:, :1].float().numpy()
        t = time.perf_counter()
        O.packed_attention(qo, cache_o)
        dt = time.perf_counter() - t
        res["cpu_baseline"] = {"value": B * S / (dt * H * L), "unit": "tokens/s", "cores": os.cpu_count(),
                               "kind": "port",
                               "sample": "oracle unpack + float64 numpy attention of head 0 of the layer, "
                                         "extrapolated x32 heads x32 layers"}
    res["gqa_block"] = gqa_block_attention(args, rank, dev, tensor_peak, k, v, codes, c["group"]) if world == 1 else None
    return res


def gqa_block_attention(args, rank, dev, tensor_peak, k, v, codes, group):
    """Blockwise decoding shape of the grouped-query model path: a 256-token block's queries
    (32 query heads) attend to the packed cfg3 prefix (8 KV heads of it, 4096 tokens) plus the
    block's own K/V (the reference's cat(past, new) + repeat_kv + attention,
    diffusion_llama.py:376-390).  Events around the two launches; the reference arm for it is
    unpack + cat + repeat_kv + torch attention (fp32) on the same device."""
    import torch

    from shadow_infer_b200.shadowkv import PackedKVCache, PrecisionPlan, packed_attention

    H_kv, rep, W_blk = 8, 4, 256
    B, _, S, D = k.shape
    cache = PackedKVCache.pack(k[:, :H_kv].contiguous().to(dev), v[:, :H_kv].contiguous().to(dev), None, group,
                               plan=PrecisionPlan.from_codes(codes[:, :H_kv].contiguous()))["packed_kv"]
    g = torch.Generator(device=dev).manual_seed(5 + rank)
    q = torch.randn(B, H_kv * rep, W_blk, D, device=dev, generator=g).half()
    kn = torch.randn(B, H_kv, W_blk, D, device=dev, generator=g)
    vn = torch.randn(B, H_kv, W_blk, D, device=dev, generator=g)
    packed_attention(q, cache, k_new=kn, v_new=vn)
    reps = max(3, min(args.steps, 20))
    ev = [tuple(torch.cuda.Event(enable_timing=True) for _ in range(3)) for _ in range(reps + 3)]
    for i in range(reps + 3):
        packed_attention(q, cache, check=False, events=ev[i], k_new=kn, v_new=vn)
    torch.cuda.synchronize()
    ms = statistics.mean(a.elapsed_time(c) for a, _, c in ev[3:])
    kms = statistics.mean(b.elapsed_time(c) for _, b, c in ev[3:])
    flops = 4.0 * B * H_kv * rep * W_blk * (S + W_blk) * D

    def torch_path():
        pk, pv = cache.unpack()
        ka = torch.cat((pk, kn), dim=2).repeat_interleave(rep, dim=1)
        va = torch.cat((pv, vn), dim=2).repeat_interleave(rep, dim=1)
        return torch.softmax(q.float() @ ka.transpose(-2, -1) / D ** 0.5, dim=-1) @ va

    for _ in range(2):
        torch_path()
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record()
    for _ in range(reps):
        torch_path()
    e1.record()
    torch.cuda.synchronize()
    return {
        "workload": f"block of {W_blk} queries x {H_kv * rep} heads over a packed prefix of {S} tokens x {H_kv} KV "
                    f"heads (codes 20/50/30) + the block's own K/V, D={D}",
        "ms": ms, "attention_kernel_ms": kms,
        "roofline": {"kernel": "packed_attention_kernel (GQA, dense tail rows)", "bound": "tensor",
                     "achieved": flops / (kms / 1e3) / 1e12, "peak": tensor_peak[0], "unit": "TFLOP/s",
                     "frac": flops / (kms / 1e3) / 1e12 / tensor_peak[0], "flops_per_launch": flops},
        "torch_unpack_cat_attention_ms": e0.elapsed_time(e1) / reps,
    }


# --------------------------------------------------------------------------- global budget
def budget_phase(args, world, rank, dev, lib):
    """KVCacheManager.enforce_global_budget over 8 packed layers of cfg3's shape.

    Each step re-packs the 8 layers (outside the timed region), then times one
    enforce_global_budget call (budget = 70 % of the usage, 4 sink tokens) with CUDA events:
    candidate listing, the device selection for each batch the reference's loop visits, and
    the in-place eviction of every layer.
    """
    import torch

    from shadow_infer_b200 import workloads as W
    from shadow_infer_b200.shadowkv import KVCacheEntry, KVCacheManager, PackedKVCache, PrecisionPlan
    from shadow_infer_b200.shadowkv.shadowkv_agent import allocate_precision_codes

    c = W.CONFIGS["cfg3"]
    B, H, S, D, layers, sink = c["B"], c["H"], c["S"], c["D"], 8, 4
    kvs, imps, plans = [], [], []
    for L in range(layers):
        k, v = W.kv_tensors(B, H, S, D, 1000 * rank + L)
        imp = W.importance_map(S, H, 1000 * rank + L, c["fractions"]).to(dev)
        kvs.append((k.to(dev), v.to(dev)))
        imps.append(imp)
        plans.append(PrecisionPlan.from_codes(allocate_precision_codes(imp, "balanced")))

    def fresh():
        mgr = KVCacheManager(num_layers=layers)
        for L in range(layers):
            cache = PackedKVCache.pack(kvs[L][0], kvs[L][1], None, c["group"], plan=plans[L])["packed_kv"]
            mgr.store(L, KVCacheEntry(k_tensor=None, v_tensor=None, precision="mixed", packed_kv=cache))
            mgr.set_importance_matrix(L, imps[L])
        return mgr

    steps = max(3, min(args.steps, 10))
    n_cand = layers * (S - sink) * H
    mgr = fresh()
    budget = int(mgr.get_memory_usage() * 0.7)
    for _ in range(2):
        fresh().enforce_global_budget(budget, sink)
    times, processed, launches = [], 0, 0
    for _ in range(steps):
        mgr = fresh()
        torch.cuda.synchronize()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        n0 = lib.skv_launch_count()
        e0.record()
        processed = mgr.enforce_global_budget(budget, sink)
        e1.record()
        torch.cuda.synchronize()
        launches = lib.skv_launch_count() - n0
        times.append(e0.elapsed_time(e1))
    ms = statistics.median(times)
    res = {
        "metric": "enforce_global_budget candidates/s (8 layers, cfg3 shape)",
        "value": n_cand / (ms / 1e3), "unit": "candidates/s", "ms_per_call": ms, "steps": steps,
        "config": {"workload": "8 packed layers B1 H32 S4096 D128 (codes 20/50/30 fp16/int8/int4), "
                               "budget 70% of usage, 4 sink tokens", "candidates": n_cand,
                   "processed": processed},
        "gpu_launches": launches,
    }
    if world == 1 and rank == 0:
        import numpy as np
        from oracle import shadowkv_oracle as O

        k, v = kvs[0]
        codes = plans[0].codes.cpu().numpy()
        layer = {"cache": O.pack(k.cpu().numpy(), v.cpu().numpy(), O.plan_from_codes(codes), c["group"]),
                 "importance": imps[0].cpu().numpy(), "counted": True}
        bud = int(O.manager_usage([layer]) * 0.7)
        t = time.perf_counter()
        O.enforce_global_budget([layer], bud, sink)
        dt = time.perf_counter() - t
        res["cpu_baseline"] = {"value": (S - sink) * H / dt, "unit": "candidates/s", "cores": 1, "kind": "port",
                               "sample": "numpy oracle of enforce_global_budget on one layer of the workload"}
    return res


def paged_phase(args, world, rank, dev, lib, run_mode=True):
    """PagedKVStore (kv_execution="paged"), two measurements.

    * append-mode run: the reference's own paged benchmark shape (B=4, H=8, D=64, 8 layers,
      32-token fp16 pages, 16 steps of 128 new tokens; per step and layer gather the past,
      then append the new tokens), through the public API, timed with CUDA events around
      the whole run (host work included: the GPU waits on it);
    * gather / append kernels at the cfg2 layer shape (B=1, H=32, S=8192, D=128, fp16
      pages): one gather of the full store and one append of all 8192 tokens, each over
      more than L2's worth of bytes, CUDA events around each launch.
    """
    import torch

    from shadow_infer_b200.shadowkv import PagedKVStore

    B, H, D, L, P, n_steps, chunk = 4, 8, 64, 8, 32, 16, 128
    S = n_steps * chunk
    g = torch.Generator().manual_seed(2026 + rank)
    kf = (torch.randn(B, H, S, D, generator=g) * 2.0).to(dev)
    vf = (torch.randn(B, H, S, D, generator=g) * 2.0).to(dev)
    reps = max(3, min(args.steps, 5))
    res = {}

    def run():
        stores = [PagedKVStore(B, H, D, page_size=P, device=dev) for _ in range(L)]
        for step in range(n_steps):
            a = step * chunk
            for st in stores:
                if step:
                    st.gather()
                st.append(kf[:, :, a:a + chunk], vf[:, :, a:a + chunk], "fp16")
        return stores

    if run_mode:
        for _ in range(2):
            run()
        times = []
        n0 = lib.skv_launch_count()
        for _ in range(reps):
            torch.cuda.synchronize()
            e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            e0.record()
            run()
            e1.record()
            torch.cuda.synchronize()
            times.append(e0.elapsed_time(e1))
        launches = (lib.skv_launch_count() - n0) // reps
        ms = statistics.median(times)
        res.update({
            "metric": "paged append-mode run tokens/s (AR014 shape: 8 layers, 16 steps x 128 tokens, "
                      "gather + append)",
            "value": L * S / (ms / 1e3), "unit": "tokens/s", "ms_per_run": ms, "runs": reps,
            "config": {"workload": "B4 H8 D64, 8 layers, 32-token fp16 pages, 16 steps of 128 tokens",
                       "gathers_per_run": L * (n_steps - 1), "appends_per_run": L * n_steps},
            "gpu_launches_per_run": launches,
        })

    # kernels at the cfg2 layer shape
    B2, H2, S2, D2 = 1, 32, 8192, 128
    k2 = (torch.randn(B2, H2, S2, D2, generator=g) * 2.0).to(dev)
    v2 = (torch.randn(B2, H2, S2, D2, generator=g) * 2.0).to(dev)
    flush = torch.empty(256 << 20, dtype=torch.uint8, device=dev)
    gather_ms, append_ms = [], []
    for i in range(2 + reps):
        st = PagedKVStore(B2, H2, D2, page_size=32, device=dev)
        flush.fill_(i & 0xFF)
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        st._kernel_events = (e0, e1)
        st.append(k2, v2, "fp16")
        flush.fill_(i & 0xFF)
        e2, e3 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        st._kernel_events = (e2, e3)
        st.gather()
        torch.cuda.synchronize()
        if i >= 2:
            append_ms.append(e0.elapsed_time(e1))
            gather_ms.append(e2.elapsed_time(e3))
    peak, peak_kind = hbm_peak()
    n_el = B2 * H2 * S2 * D2
    g_bytes = 2 * n_el * (2 + 4)            # fp16 pages read, fp32 K/V written
    a_bytes = 2 * n_el * (4 + 2)            # fp32 rows read, fp16 pages written
    g_ms, a_ms = statistics.mean(gather_ms), statistics.mean(append_ms)
    res.update({
        "gather": {"workload": "B1 H32 S8192 D128 fp16 pages (256 pages of 32)", "ms": g_ms,
                   "GB/s": g_bytes / (g_ms / 1e3) / 1e9,
                   "roofline": {"kernel": "paged_gather_kernel", "bound": "hbm",
                                "achieved": g_bytes / (g_ms / 1e3) / 1e9, "peak": peak, "unit": "GB/s",
                                "frac": g_bytes / (g_ms / 1e3) / 1e9 / peak, "peak_source": f"{peak_kind} hbm_gbs",
                                "algorithmic_bytes": g_bytes,
                                "traffic": committed_traffic("paged_gather_kernel_cfg2.md")}},
        "append": {"workload": "one append of 8192 tokens into 256 new fp16 pages", "ms": a_ms,
                   "GB/s": a_bytes / (a_ms / 1e3) / 1e9,
                   "roofline": {"kernel": "paged_write_vec_kernel", "bound": "hbm",
                                "achieved": a_bytes / (a_ms / 1e3) / 1e9, "peak": peak, "unit": "GB/s",
                                "frac": a_bytes / (a_ms / 1e3) / 1e9 / peak, "peak_source": f"{peak_kind} hbm_gbs",
                                "algorithmic_bytes": a_bytes,
                                "traffic": committed_traffic("paged_write_vec_kernel_cfg2.md")}},
    })
    if run_mode and world == 1 and rank == 0:
        from oracle.paged_store_oracle import OraclePagedStore

        kc, vc = kf.cpu().numpy(), vf.cpu().numpy()
        t = time.perf_counter()
        st = OraclePagedStore(B, H, D, page_size=P)
        for step in range(n_steps):
            a = step * chunk
            if step:
                st.gather()
            st.append(kc[:, :, a:a + chunk], vc[:, :, a:a + chunk], "fp16")
        dt = time.perf_counter() - t
        res["cpu_baseline"] = {"value": S / dt, "unit": "tokens/s", "cores": 1, "kind": "port",
                               "sample": "numpy oracle of the append-mode run on one of the 8 layers"}
    return res


def decision_phase(args, world, rank, dev, lib):
    """Decision inputs: decide_reuse_per_token over the cfg2 layer (current vs previous K/V,
    B=1, H=32, S=8192, D=128) and compute_irap_importance over cfg3-shaped attention
    probabilities (B=1, H=32, 4096 x 4096, 2.1 GB, with the previous step's EMA), CUDA events
    around each call (every launch of it inside), inputs resident and larger than L2."""
    import torch

    from shadow_infer_b200 import workloads as W
    from shadow_infer_b200.shadowkv import compute_irap_importance
    from shadow_infer_b200.shadowkv.shadowkv_agent import decide_reuse_mask

    I = W.cfg2_inputs(seed=rank)
    k, v = I["k"].to(dev), I["v"].to(dev)
    kp, vp = I["k_prev"].to(dev), I["v_prev"].to(dev)
    imp = I["importance"].to(dev)
    B, H, S, D = k.shape
    reps = max(3, min(args.steps, 10))

    def timed(fn):
        out, ts = None, []
        for i in range(2 + reps):
            torch.cuda.synchronize()
            e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            e0.record()
            out = fn()
            e1.record()
            torch.cuda.synchronize()
            if i >= 2:
                ts.append(e0.elapsed_time(e1))
        return out, statistics.median(ts)

    from shadow_infer_b200 import _lib
    from shadow_infer_b200.shadowkv.shadowkv_agent import reuse_threshold

    n0 = lib.skv_launch_count()
    (mask, stats), reuse_ms = timed(lambda: decide_reuse_mask(k, v, kp, vp, 4, 16, 0.2, "balanced", imp))
    reuse_launches = (lib.skv_launch_count() - n0) // (2 + reps)
    reuse_bytes = 4 * B * H * S * D * 4 + S * H * 4 + S * H
    # the kernel alone: the C-ABI call with the buffers already allocated
    m_out = torch.empty(S, H, dtype=torch.uint8, device=dev)
    cnt = torch.empty(4, dtype=torch.int64, device=dev)
    eff = reuse_threshold(4, 16, 0.2, "balanced")
    stream = _lib.stream_of(dev)

    def reuse_kernel():
        _lib.check(lib.skv_reuse_decide(_lib.ptr(k), _lib.ptr(v), _lib.ptr(kp), _lib.ptr(vp), B, H, S, D,
                                        _lib.ptr(imp), eff, _lib.ptr(m_out), None, _lib.ptr(cnt), stream), "bench")

    _, reuse_kms = timed(reuse_kernel)
    c3 = W.CONFIGS["cfg3"]
    Hq, Sq = c3["H"], c3["S"]
    g = torch.Generator(device=dev).manual_seed(77 + rank)
    logits = torch.randn(1, Hq, Sq, Sq, device=dev, generator=g)
    logits[:, :, : (3 * Sq) // 4] *= 6.0
    probs = torch.softmax(logits, dim=-1)
    del logits
    prev = torch.rand(Sq, Hq, device=dev, generator=g) / Sq
    n0 = lib.skv_launch_count()
    (imp3, ema3, da), irap_ms = timed(lambda: compute_irap_importance(probs, prev, 0.9, 0.3, 4, 1, 32))
    irap_launches = (lib.skv_launch_count() - n0) // (2 + reps)
    irap_bytes = probs.numel() * 4
    # the launches alone: the C-ABI call with scratch and outputs already allocated
    scr = torch.empty(lib.skv_irap_scratch_bytes(1, Hq, Sq, Sq), dtype=torch.uint8, device=dev)
    o_imp = torch.empty(Sq, Hq, device=dev)
    o_ema = torch.empty(Sq, Hq, device=dev)
    o_dp = torch.empty(2, dtype=torch.float64, device=dev)

    def irap_kernels():
        _lib.check(lib.skv_irap_importance(_lib.ptr(probs), 1, Hq, Sq, Sq, 0, _lib.ptr(prev), Sq, 0.9, 0.3, 4,
                                           1.0 + 0.1 * (1 / 32), _lib.ptr(scr), scr.numel(), _lib.ptr(o_imp),
                                           _lib.ptr(o_ema), _lib.ptr(o_dp), stream), "bench")

    _, irap_kms = timed(irap_kernels)
    peak, peak_kind = hbm_peak()
    res = {
        "reuse_decision": {
            "workload": "cfg2 layer B1 H32 S8192 D128, current vs previous K/V, balanced, step 4/16",
            "ms": reuse_ms, "GB/s": reuse_bytes / (reuse_ms / 1e3) / 1e9, "gpu_launches": reuse_launches,
            "kernel_ms": reuse_kms, "reuse_ratio": stats["reuse_ratio"],
            "roofline": {"kernel": "reuse_decide_kernel", "bound": "hbm", "algorithmic_bytes": reuse_bytes,
                         "achieved": reuse_bytes / (reuse_kms / 1e3) / 1e9, "peak": peak, "unit": "GB/s",
                         "frac": reuse_bytes / (reuse_kms / 1e3) / 1e9 / peak, "peak_source": f"{peak_kind} hbm_gbs",
                         "traffic": committed_traffic("reuse_decide_kernel_cfg2.md")},
        },
        "irap_importance": {
            "workload": f"attention probabilities [1,{Hq},{Sq},{Sq}] fp32 (cfg3 layer) with the previous EMA",
            "ms": irap_ms, "GB/s": irap_bytes / (irap_ms / 1e3) / 1e9, "gpu_launches": irap_launches,
            "kernels_ms": irap_kms,
            "roofline": {"kernel": "irap_pass_kernel + columns, delta and rank kernels (one ABI call)",
                         "bound": "hbm", "algorithmic_bytes": irap_bytes,
                         "achieved": irap_bytes / (irap_kms / 1e3) / 1e9, "peak": peak, "unit": "GB/s",
                         "frac": irap_bytes / (irap_kms / 1e3) / 1e9 / peak, "peak_source": f"{peak_kind} hbm_gbs",
                         "traffic": committed_traffic("irap_pass_kernel_cfg3.md")},
        },
    }
    if world == 1 and rank == 0:
        import numpy as np

        from oracle import decision_oracle as DO

        hs = 2
        kk, vv, kkp, vvp = (t[:, :hs].cpu().numpy() for t in (k, v, kp, vp))
        ii = imp[:, :hs].cpu().numpy()
        t0 = time.perf_counter()
        DO.decide_reuse_per_token(kk, vv, kkp, vvp, 4, 16, 0.2, "balanced", ii)
        dt_r = time.perf_counter() - t0
        pw = probs[:, :1].cpu().numpy()
        t0 = time.perf_counter()
        DO.compute_irap_importance(pw, prev[:, :1].cpu().numpy(), 0.9, 0.3, 4, 1, 32)
        dt_i = time.perf_counter() - t0
        res["reuse_decision"]["cpu_baseline"] = {
            "value": (reuse_bytes * hs / H) / dt_r / 1e9, "unit": "GB/s", "cores": 1, "kind": "port",
            "sample": f"numpy oracle on heads 0..{hs - 1} of the cfg2 layer"}
        res["irap_importance"]["cpu_baseline"] = {
            "value": (irap_bytes / Hq) / dt_i / 1e9, "unit": "GB/s", "cores": 1, "kind": "port",
            "sample": "numpy oracle on head 0 of the cfg3 probabilities"}
        del np
    return res


def tensor_peak():
    path = os.path.join(REPO, "MEASURED_PEAKS.json")
    try:
        with open(path) as f:
            return float(json.load(f)["bf16_tflops"]), "measured bf16_tflops (burst; fp16 runs at the same rate)"
    except Exception:
        return 1590.0, "fallback"


# ------------------------------------------------------------------------------------ b200
def run_b200(args):
    import torch
    import torch.distributed as dist

    from shadow_infer_b200 import _lib
    from shadow_infer_b200 import workloads as W
    from shadow_infer_b200.shadowkv import PackedKVCache, PrecisionPlan, kv_sensitivity
    from shadow_infer_b200.shadowkv.rd_allocator import admit_codes_device
    from shadow_infer_b200.shadowkv.shadowkv_agent import allocate_precision_codes

    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    if world > 1:
        import datetime
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=120), device_id=dev)
    lib = _lib.load()
    if args.phase != "all":
        if args.phase == "decisions":
            res = decision_phase(args, world, rank, dev, lib)
        else:
            res = paged_phase(args, world, rank, dev, lib, run_mode=args.phase == "paged")
        if world > 1:
            dist.destroy_process_group()
        if rank == 0:
            print(json.dumps({"phase": args.phase, "result": res}), flush=True)
        return 0

    # every rank packs its own layer: seed = rank
    I = W.cfg2_inputs(seed=rank)
    B, H, S, D = I["k"].shape
    k, v = I["k"].to(dev), I["v"].to(dev)
    imp, reuse = I["importance"].to(dev), I["reuse"].to(dev)
    budget, sink = I["budget"], I["sink_tokens"]

    codes0 = allocate_precision_codes(imp, "balanced")
    adm, _ = admit_codes_device(codes0, imp, kv_sensitivity(k, v), budget, B, D, sink, True, True)
    prev = PackedKVCache.pack(I["k_prev"].to(dev), I["v_prev"].to(dev), None, 16,
                              plan=PrecisionPlan.from_codes(adm))["packed_kv"]

    def step(kk, vv, ii, rr):
        codes = allocate_precision_codes(ii, "balanced")
        sens = kv_sensitivity(kk, vv)
        a, res = admit_codes_device(codes, ii, sens, budget, B, D, sink, True, True)
        plan = PrecisionPlan.from_codes(a, reuse_mask=rr)
        cache = PackedKVCache.pack(kk, vv, None, 16, plan=plan)["packed_kv"]
        cache.apply_reuse_mask(prev, rr)
        ku, vu = cache.unpack()
        return cache, res, ku, vu

    # algorithmic bytes of the step (fixed across steps: same inputs)
    cache, res, _, _ = step(k, v, imp, reuse)
    stats = cache.apply_reuse_mask(prev, reuse, return_stats=True)
    kept = sum(cache._count.values())
    from shadow_infer_b200.shadowkv.rd_allocator import entry_bytes
    per_code = {p: int(entry_bytes(p, B, D, 16)) for p in ("fp32", "fp16", "int8", "int4")}
    # reused rows: entries present in both caches with the same precision; same codes here, so
    # every flagged stored entry is copied
    reused_bytes = 0
    slot = cache._slot
    flagged = reuse.reshape(-1).bool() & (slot >= 0)
    for code, p in enumerate(("fp32", "fp16", "int8", "int4")):
        reused_bytes += int(((slot & 3) == code)[flagged].sum().item()) * per_code[p]
    assert stats["applied"] == int(flagged.sum().item())
    parts = step_bytes(B, H, S, D, cache.memory_bytes(), kept, reused_bytes, int(reuse.sum().item()))
    nbytes = sum(parts.values())

    sampler = ClockSampler(local) if rank == 0 else None
    if sampler:
        sampler.start()
    for _ in range(args.warmup):
        step(k, v, imp, reuse)
    # pack-kernel events inside the timed region
    n_ev = args.steps
    evs = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)) for _ in range(n_ev)]
    t0 = torch.cuda.Event(enable_timing=True)
    t1 = torch.cuda.Event(enable_timing=True)
    if world > 1:
        dist.barrier()
    torch.cuda.synchronize()
    launches0 = lib.skv_launch_count()
    t0.record()
    for i in range(args.steps):
        PackedKVCache._pack_events = evs[i]
        step(k, v, imp, reuse)
    PackedKVCache._pack_events = None
    t1.record()
    torch.cuda.synchronize()
    launches = lib.skv_launch_count() - launches0
    if world > 1:
        dist.barrier()
    elapsed_ms = t0.elapsed_time(t1)
    pack_ms_in_step = [a.elapsed_time(b) for a, b in evs]
    # the pack kernel alone, back to back on this step's plan: an L2 flush (a 256 MB fill, ~40 us
    # of GPU work) precedes each launch, so the host's bucket allocation and launch call overlap
    # GPU work and the event pair holds the kernel only (inside a step the GPU idles on the host
    # between the plan's count read-back and the launch, and that gap lands in the events)
    from shadow_infer_b200.shadowkv.packed_kv_cache import run_pack
    plan_last = PrecisionPlan.from_codes(admit_codes_device(allocate_precision_codes(imp, "balanced"), imp,
                                                            kv_sensitivity(k, v), budget, B, D, sink, True,
                                                            True)[0], reuse_mask=reuse)
    flush = torch.empty(256 << 20, dtype=torch.uint8, device=dev)
    pev = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)) for _ in range(10)]
    for i, ev in enumerate(pev):
        flush.fill_(i & 0xFF)
        run_pack(k, v, plan_last, 16, events=ev)
    torch.cuda.synchronize()
    pack_ms = [a.elapsed_time(b) for a, b in pev[2:]]
    # every call of the step alone, the same way: each after two L2-flushing fills (~80 us of GPU
    # work, during which the host enqueues the call), events around the call
    def alone(fn, n=8):
        evp = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)) for _ in range(n)]
        for i, (a, b) in enumerate(evp):
            flush.fill_(i & 0xFF)
            flush.fill_((i + 1) & 0xFF)
            a.record()
            fn()
            b.record()
        torch.cuda.synchronize()
        return statistics.mean(a.elapsed_time(b) for a, b in evp[2:])
    codes_l = allocate_precision_codes(imp, "balanced")
    sens_l = kv_sensitivity(k, v)
    adm_l = admit_codes_device(codes_l, imp, sens_l, budget, B, D, sink, True, True)[0]
    cache_l = PackedKVCache.pack(k, v, None, 16, plan=PrecisionPlan.from_codes(adm_l, reuse_mask=reuse))["packed_kv"]
    kernel_ms = {
        "allocate": alone(lambda: allocate_precision_codes(imp, "balanced")),
        "sensitivity": alone(lambda: kv_sensitivity(k, v)),
        "admission": alone(lambda: admit_codes_device(codes_l, imp, sens_l, budget, B, D, sink, True, True)),
        "plan": alone(lambda: PrecisionPlan.from_codes(adm_l, reuse_mask=reuse)),
        "pack": statistics.mean(pack_ms),
        "reuse": alone(lambda: cache_l.apply_reuse_mask(prev, reuse)),
        "unpack": alone(lambda: cache_l.unpack()),
    }
    # evict: 25 % of the (t, h) entries (seeded Bernoulli mask) from a freshly packed copy of the
    # layer each time; the pack is queued before the fills and is not timed
    gen = torch.Generator(device="cpu").manual_seed(7)
    evict_mask = (torch.rand(S, H, generator=gen) < 0.25).to(dev)
    plan_e = PrecisionPlan.from_codes(adm_l)
    eve = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)) for _ in range(8)]
    evict_after = 0
    for i, (a, b) in enumerate(eve):
        ce = PackedKVCache.pack(k, v, None, 16, plan=plan_e)["packed_kv"]
        flush.fill_(i & 0xFF)
        flush.fill_((i + 1) & 0xFF)
        a.record()
        ce.evict(evict_mask)
        b.record()
        evict_after = ce.memory_bytes()
    torch.cuda.synchronize()
    kernel_ms["evict"] = statistics.mean(a.elapsed_time(b) for a, b in eve[2:])
    parts_k = dict(parts)
    parts_k["evict"] = S * H + 2 * evict_after
    del flush
    tmax = torch.tensor([elapsed_ms], device=dev, dtype=torch.float64)
    if world > 1:
        dist.all_reduce(tmax, op=dist.ReduceOp.MAX)
    elapsed_ms = float(tmax.item())
    ms_per_step = elapsed_ms / args.steps
    value = world * nbytes * args.steps / (elapsed_ms / 1e3) / 1e9

    # ---- e2e: pinned host buffers through the public API
    hk = I["k"].pin_memory()
    hv = I["v"].pin_memory()
    himp = I["importance"].pin_memory()
    hreuse = I["reuse"].pin_memory()
    # Steps are pipelined over full-duplex PCIe: step i+1's inputs travel host -> device on one
    # copy stream and step i's packed payload device -> host on another while the data plane
    # computes on the current stream; device inputs and the host result buffer are double-
    # buffered.  Every step's copies lie inside the timed region.
    out_host = [torch.empty(cache.memory_bytes() + 64, dtype=torch.uint8).pin_memory() for _ in range(2)]
    res_host = [torch.empty(2, dtype=torch.int64).pin_memory() for _ in range(2)]
    dbuf = [tuple(torch.empty(t.shape, dtype=t.dtype, device=dev) for t in (hk, hv, himp, hreuse)) for _ in range(2)]
    cs = torch.cuda.current_stream(dev)
    s_in, s_out = torch.cuda.Stream(device=dev), torch.cuda.Stream(device=dev)
    in_ready = [torch.cuda.Event() for _ in range(2)]
    in_free = [torch.cuda.Event() for _ in range(2)]
    n_e2e = [0]

    def e2e_step():
        j = n_e2e[0] % 2
        n_e2e[0] += 1
        with torch.cuda.stream(s_in):
            s_in.wait_event(in_free[j])            # the compute that read buffer j is done
            for d, h in zip(dbuf[j], (hk, hv, himp, hreuse)):
                d.copy_(h, non_blocking=True)
            in_ready[j].record(s_in)
        cs.wait_event(in_ready[j])
        c, r, _, _ = step(*dbuf[j])
        in_free[j].record(cs)
        done = torch.cuda.Event()
        done.record(cs)
        off = 0
        with torch.cuda.stream(s_out):
            s_out.wait_event(done)
            for d in c.packed_data.values():
                for key in ("k", "v", "scale_k", "scale_v"):
                    t = d[key]
                    if t is None:
                        continue
                    nb = t.numel() * t.element_size()
                    out_host[j][off:off + nb].copy_(t.reshape(-1).view(torch.uint8), non_blocking=True)
                    t.record_stream(s_out)
                    off += nb
            res_host[j].copy_(r, non_blocking=True)
            r.record_stream(s_out)
        return off

    e2e_steps = max(3, min(args.steps, 30))
    for _ in range(3):
        e2e_step()
    if world > 1:
        dist.barrier()
    torch.cuda.synchronize()
    e0 = torch.cuda.Event(enable_timing=True)
    e1 = torch.cuda.Event(enable_timing=True)
    e0.record(cs)
    s_in.wait_event(e0)                            # no copy of the timed steps starts before e0
    d2h = 0
    for _ in range(e2e_steps):
        d2h = e2e_step()
    cs.wait_stream(s_in)
    cs.wait_stream(s_out)
    e1.record(cs)
    torch.cuda.synchronize()
    e2e_ms = torch.tensor([e0.elapsed_time(e1)], device=dev, dtype=torch.float64)
    if world > 1:
        dist.all_reduce(e2e_ms, op=dist.ReduceOp.MAX)
    e2e_ms = float(e2e_ms.item())
    h2d = (hk.numel() + hv.numel() + himp.numel()) * 4 + hreuse.numel()
    attn = attention_phase(args, world, rank, dev, dist, lib, tensor_peak()) if not args.no_attention else None
    gbudget = budget_phase(args, world, rank, dev, lib) if not args.no_attention else None
    paged = paged_phase(args, world, rank, dev, lib) if not args.no_attention else None
    decisions = decision_phase(args, world, rank, dev, lib) if not args.no_attention else None
    if sampler:
        sampler.stop()

    if world > 1:
        dist.barrier()
        dist.destroy_process_group()
    if rank != 0:
        return 0

    peak, peak_kind = hbm_peak()
    pack_avg_ms = statistics.mean(pack_ms)
    achieved = parts["pack"] / (pack_avg_ms / 1e3) / 1e9
    traffic = committed_traffic("pack16_kernel_cfg2.md")
    line = {
        "metric": METRIC, "value": value, "unit": "GB/s", "n_gpus": world, "steps": args.steps,
        "warmup": args.warmup, "ms_per_step": ms_per_step, "higher_is_better": True, "scaling": "weak",
        "vs_baseline": None, "dtype": "f32", "data": "synthetic",
        "config": {"workload": "cfg2 data-plane step: codes, sensitivity, budget admission + hard eviction, "
                               "plan, compress+pack, reuse (50%), unpack",
                   "B": B, "H": H, "S": S, "D": D, "layers_per_gpu": 1, "budget_bytes": budget,
                   "l2": "inputs larger than L2 (K+V 268 MB per layer)",
                   "bytes_per_step": parts},
        "roofline": {"kernel": "pack16_kernel", "bound": "hbm", "achieved": achieved, "peak": peak,
                     "unit": "GB/s", "frac": achieved / peak, "peak_source": f"{peak_kind} hbm_gbs",
                     "traffic": traffic, "algorithmic_bytes": parts["pack"], "avg_launch_ms": pack_avg_ms,
                     "timing": "events around 8 back-to-back launches on the step's plan, each after a 256 MB "
                               "L2-flushing fill",
                     "in_step_avg_launch_ms": statistics.mean(pack_ms_in_step)},
        "e2e": {"value": world * nbytes * e2e_steps / (e2e_ms / 1e3) / 1e9, "unit": "GB/s",
                "h2d_bytes_per_step": h2d, "d2h_bytes_per_step": d2h + 16, "steps": e2e_steps,
                "ms_per_step": e2e_ms / e2e_steps,
                "pipelining": "inputs of step i+1 in and step i's packed payload out on two copy streams "
                              "while step i computes (PCIe is full duplex); double-buffered"},
        "gpu_launches": launches,
        "clocks": sampler.summary() if sampler else None,
        "kernels": {name: {"avg_ms": ms, "algorithmic_bytes": parts_k[name],
                           "achieved_gbs": parts_k[name] / (ms / 1e3) / 1e9,
                           "frac": parts_k[name] / (ms / 1e3) / 1e9 / peak}
                    for name, ms in kernel_ms.items()},
        "kernels_timing": "each call of the step alone through its public API, events around it, after two "
                          "256 MB L2-flushing fills (8 calls, first 2 dropped; pack: the roofline's launches; "
                          "evict: 25 % of the entries of a freshly packed copy, bytes = mask + 2 x packed bytes "
                          "after, count + compaction with the host read of the kept counts between); frac of "
                          "measured HBM",
        "attention": attn,
        "global_budget": gbudget,
        "paged_store": paged,
        "decisions": decisions,
    }
    if world == 1:
        run = reference_sample(I, args.ref_heads)
        run()
        samples = [run() for _ in range(3)]
        ref_val = sum(b for _, b in samples) / sum(t for t, _ in samples) / 1e9
        line["cpu_baseline"] = {
            "value": ref_val, "unit": "GB/s", "cores": 1, "kind": "port",
            "sample": f"numpy oracle pipeline on heads 0..{args.ref_heads - 1} of the cfg2 layer, 3 runs",
        }
    print(json.dumps(line), flush=True)
    return 0


def main():
    args = parse_args()
    if args.impl == "reference":
        return run_reference(args)
    return run_b200(args)


if __name__ == "__main__":
    sys.exit(main())
