"""PagedKVStore on the GPU vs the reference fixtures, the CPU oracle and the packed cache.

Every operation script recorded from the reference store is replayed: return values and
ValueErrors, page layout, slot pool, counters, byte ledgers, the bytes of every page
tensor and the gather result must equal the reference's exactly (integer/byte work and
IEEE-exact quantisation).  Seeded random scripts at larger sizes are checked against the
oracle the same way.
"""

import numpy as np
import pytest
import torch

from golden_lib import array_digest, load_pins, paged_apply, paged_inputs, state_digest
from oracle.paged_store_oracle import OraclePagedStore, store_state

pytestmark = pytest.mark.gpu

PRECISIONS = ("fp32", "fp16", "int8", "int4")


@pytest.fixture(scope="module")
def skv():
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    import shadow_infer_b200.shadowkv as m
    return m


def _np(t):
    return t.detach().cpu().numpy()


def _state(store):
    st = store_state(store, _np)
    st["pages_digest"] = state_digest(st.pop("page_digests"))
    return st


def _replay(skv, pin, device):
    B, H, D = pin["B"], pin["H"], pin["D"]
    store = skv.PagedKVStore(B, H, D, page_size=pin["P"], device=device, int4_group_size=pin["G"])
    conv = lambda x: torch.from_numpy(x).to(device)  # noqa: E731
    for i, (op, want) in enumerate(zip(pin["ops"], pin["results"])):
        try:
            ret, err = paged_apply(store, op, B, H, D, conv), False
        except ValueError:
            ret, err = None, True
        assert (ret, err) == (want["ret"], want["error"]), (i, op)
        assert _state(store) == want["state"], (i, op)
        k, v = store.gather()
        assert k.device.type == torch.device(device).type
        assert [array_digest(k), array_digest(v)] == want["gather"] and k.shape[2] == want["S_out"], (i, op)


_CASES = sorted(c for c, v in load_pins()["cases"].items() if v["kind"] == "paged")


@pytest.mark.parametrize("case", _CASES)
def test_script_matches_reference_fixture(case, skv):
    _replay(skv, load_pins()["cases"][case], "cuda")


@pytest.mark.parametrize("case", ["paged_fp16_evict", "paged_mixed_pool", "paged_random_b2_d64"])
def test_script_matches_reference_fixture_host_device(case, skv):
    """A store created with device='cpu' (the reference's default) keeps its pages on the GPU
    and hands out host tensors."""
    _replay(skv, load_pins()["cases"][case], "cpu")


def _random_script(rng, store, B, H, D, P, n_ops):
    """Yields operations chosen against the oracle store's live state."""
    prec = "fp16"
    for i in range(n_ops):
        r = rng.random()
        seed = int(rng.integers(1 << 30))
        if r < 0.45 or store.max_seq == 0:
            if rng.random() < 0.35:
                prec = PRECISIONS[int(rng.integers(4))]
            yield ["append", int(rng.choice([1, P - 1, P, P + 1, 3 * P + 5, int(rng.integers(1, 4 * P))])), prec, seed]
        elif r < 0.7:
            S = store.max_seq
            pairs = set()
            for _ in range(int(rng.integers(1, 6))):
                t = int(rng.integers(0, S + 2))
                if rng.random() < 0.5:
                    pairs.update((t, h) for h in range(H))
                else:
                    pairs.update((t, int(h)) for h in rng.choice(H, size=int(rng.integers(1, H + 1)), replace=False))
            yield ["evict", sorted([list(p) for p in pairs])]
        else:
            pg = store.pages[store.order[int(rng.integers(len(store.order)))]] if store.order else None
            if pg is None:
                continue
            a = pg.start_token + int(rng.integers(pg.num_tokens))
            yield ["rewrite", a, int(rng.integers(1, pg.end_token - a + 1)), pg.precision, seed]


@pytest.mark.parametrize("B,H,D,P,G,n_ops,seed", [
    (2, 8, 128, 32, 16, 60, 1),
    (1, 4, 64, 16, 32, 80, 2),
    (3, 2, 96, 7, 16, 60, 3),      # page size not a power of two
    (1, 3, 40, 8, 16, 50, 4),      # int4 group falls back to head_dim (40)
    (2, 2, 33, 5, 16, 50, 5),      # odd head_dim: scalar gather path, padded int4 rows
    (1, 2, 64, 12, 4, 50, 6),      # int4 groups of 4 lanes
    (1, 2, 48, 9, 24, 50, 7),      # int4 groups of 24 (shared-memory group maxima)
    (1, 2, 256, 8, 16, 40, 8),     # 8 values per lane in the vector write path
    (2, 2, 32, 4, 8, 40, 9),       # four rows per warp pass
])
def test_random_scripts_match_oracle(skv, B, H, D, P, G, n_ops, seed):
    rng = np.random.default_rng(seed)
    ref = OraclePagedStore(B, H, D, page_size=P, int4_group_size=G)
    dut = skv.PagedKVStore(B, H, D, page_size=P, device="cuda", int4_group_size=G)
    conv = lambda x: torch.from_numpy(x).cuda()  # noqa: E731
    for i, op in enumerate(_random_script(rng, ref, B, H, D, P, n_ops)):
        try:
            want, werr = paged_apply(ref, op, B, H, D, lambda x: x), False
        except ValueError:
            want, werr = None, True
        try:
            got, gerr = paged_apply(dut, op, B, H, D, conv), False
        except ValueError:
            got, gerr = None, True
        assert (got, gerr) == (want, werr), (i, op)
        assert store_state(dut, _np) == store_state(ref), (i, op)
        kr, vr = ref.gather()
        kg, vg = dut.gather()
        np.testing.assert_array_equal(_np(kg), kr, err_msg=f"K after op {i} {op[:2]}")
        np.testing.assert_array_equal(_np(vg), vr, err_msg=f"V after op {i} {op[:2]}")


def _stepwise(store, k, v, precision, split):
    s = 0
    for n in split:
        store.append(k[:, :, s:s + n].contiguous(), v[:, :, s:s + n].contiguous(), precision)
        s += n


def _kv(seed, B=2, H=4, S=19, D=32):
    k, v = paged_inputs(seed, B, H, S, D)
    return torch.from_numpy(k).cuda(), torch.from_numpy(v).cuda()


@pytest.mark.parametrize("precision", PRECISIONS)
def test_gather_equals_packed_cache_roundtrip(skv, precision):
    """Row-local quantisation: paged gather == PackedKVCache.pack(...).unpack() bit for bit."""
    k, v = _kv(2026)
    store = skv.PagedKVStore(2, 4, 32, page_size=8, device="cuda", int4_group_size=16)
    _stepwise(store, k, v, precision, (5, 5, 5, 4))
    pmap = {t: {h: precision for h in range(4)} for t in range(19)}
    kr, vr = skv.PackedKVCache.pack(k, v, pmap, group_size=16)["packed_kv"].unpack()
    kg, vg = store.gather()
    assert torch.equal(kg, kr) and torch.equal(vg, vr)


@pytest.mark.parametrize("precision", PRECISIONS)
def test_evict_equals_packed_cache_evict(skv, precision):
    k, v = _kv(7)
    evict = {(t, h) for t in (2, 4, 5, 17) for h in range(4)} | {(10, 0), (10, 1), (12, 2), (12, 3)}
    pmap = {t: {h: precision for h in range(4)} for t in range(19)}
    cache = skv.PackedKVCache.pack(k, v, pmap, group_size=16)["packed_kv"]
    cache.evict(set(evict))
    kr, vr = cache.unpack()
    store = skv.PagedKVStore(2, 4, 32, page_size=8, device="cuda", int4_group_size=16)
    _stepwise(store, k, v, precision, (5, 5, 5, 4))
    assert store.evict_tokens(set(evict)) == 20
    kg, vg = store.gather()
    assert torch.equal(kg, kr) and torch.equal(vg, vr)


def _ptrs(page):
    return tuple(t.data_ptr() for t in (page.k, page.v, page.scale_k, page.scale_v) if t is not None)


@pytest.mark.parametrize("device", ["cuda", "cpu"])
def test_sealed_pages_keep_identity_and_buffers(skv, device):
    k, v = _kv(11)
    store = skv.PagedKVStore(2, 4, 32, page_size=8, device=device, int4_group_size=16)
    _stepwise(store, k.to(device), v.to(device), "int8", (5, 5))
    sealed, ptrs = store.pages[0], _ptrs(store.pages[0])
    _stepwise(store, k[:, :, 10:].to(device), v[:, :, 10:].to(device), "int8", (5, 4))
    assert store.pages[0] is sealed and _ptrs(store.pages[0]) == ptrs
    page1, ptrs1 = store.pages[1], _ptrs(store.pages[1])
    store.append(k[:, :, :3].to(device), v[:, :, :3].to(device), "int8")
    assert store.appended_tokens == 22 and store.pages[1] is page1 and _ptrs(page1) == ptrs1
    # eviction elsewhere leaves other pages' objects and buffers alone
    assert store.evict_tokens({(1, h) for h in range(4)}) == 4
    assert store.pages[1] is page1 and _ptrs(page1) == ptrs1
    assert store.pages[0].k.device.type == torch.device(device).type


def test_rewrite_equals_append_of_final_content(skv):
    k, v = _kv(13, S=26)
    kn, vn = _kv(14, S=16)
    kf, vf = k.clone(), v.clone()
    kf[:, :, 4:20], vf[:, :, 4:20] = kn, vn
    store = skv.PagedKVStore(2, 4, 32, page_size=8, device="cuda", int4_group_size=16)
    ref = skv.PagedKVStore(2, 4, 32, page_size=8, device="cuda", int4_group_size=16)
    _stepwise(store, k, v, "int4", (8, 8, 8, 2))
    _stepwise(ref, kf, vf, "int4", (8, 8, 8, 2))
    ids = [id(p) for p in store.pages]
    before = store.data_plane_bytes(), store.resident_bytes()
    assert store.rewrite_tokens(4, kn, vn, "int4") == 16
    assert (store.rewritten_tokens, store.rewritten_pages) == (16, 3)
    assert [id(p) for p in store.pages] == ids and (store.data_plane_bytes(), store.resident_bytes()) == before
    for a, b in zip(store.pages, ref.pages):
        for x, y in zip((a.k, a.v, a.scale_k, a.scale_v), (b.k, b.v, b.scale_k, b.scale_v)):
            assert torch.equal(x, y)


def test_long_fp16_store_matches_oracle(skv):
    """The AR014 append-mode shape: 4 x 8 heads x 64 dims, 32-token pages, 16 appends of 128."""
    B, H, D, P = 4, 8, 64, 32
    ref = OraclePagedStore(B, H, D, page_size=P)
    dut = skv.PagedKVStore(B, H, D, page_size=P, device="cuda")
    for step in range(16):
        k, v = paged_inputs(900 + step, B, H, 128, D)
        ref.append(k, v, "fp16")
        dut.append(torch.from_numpy(k).cuda(), torch.from_numpy(v).cuda(), "fp16")
    kr, vr = ref.gather()
    kg, vg = dut.gather()
    np.testing.assert_array_equal(_np(kg), kr)
    np.testing.assert_array_equal(_np(vg), vr)
    assert dut.data_plane_bytes() == ref.data_plane_bytes() == B * H * 2048 * D * 2 * 2


def test_clear_heads_flags_items_outside_the_table(skv):
    """The clear kernel checks every item against the table and its page: a bad item sets the
    error flag and touches nothing."""
    from shadow_infer_b200 import _lib
    store = skv.PagedKVStore(1, 2, 32, page_size=8, device="cuda")
    k, v = _kv(5, B=1, H=2, S=8)
    store.append(k, v, "fp16")
    before = store.gather()
    flag = torch.zeros(1, dtype=torch.int32, device="cuda")
    for item in ([0, 8, 0], [1, 0, 0], [0, 0, 2], [-1, 0, 0]):
        items = torch.tensor(item, dtype=torch.int32, device="cuda")
        st = _lib.load().skv_paged_clear_heads(_lib.ptr(store._table), 1, _lib.ptr(items), 1, 1, 2, 32,
                                               _lib.ptr(flag), _lib.stream_of(torch.device("cuda")))
        assert st == 0 and int(flag.item()) == 1
        flag.zero_()
    after = store.gather()
    assert torch.equal(before[0], after[0]) and torch.equal(before[1], after[1])


def test_misaligned_and_strided_sources(skv):
    """A token slice of a larger tensor is read in place; a source that is not 16-byte aligned
    is copied first; both give the rows an aligned contiguous tensor gives."""
    B, H, T, D = 2, 3, 37, 64
    k, v = _kv(21, B=B, H=H, S=T, D=D)
    base_k = torch.zeros(B * H * T * D + 1, device="cuda")
    base_v = torch.zeros_like(base_k)
    base_k[1:] = k.reshape(-1)
    base_v[1:] = v.reshape(-1)
    odd_k, odd_v = base_k[1:].view(B, H, T, D), base_v[1:].view(B, H, T, D)
    for precision in PRECISIONS:
        a = skv.PagedKVStore(B, H, D, page_size=8, device="cuda")
        b = skv.PagedKVStore(B, H, D, page_size=8, device="cuda")
        c = skv.PagedKVStore(B, H, D, page_size=8, device="cuda")
        a.append(k, v, precision)
        b.append(odd_k, odd_v, precision)
        c.append(k[:, :, :20], v[:, :, :20], precision)
        c.append(k[:, :, 20:], v[:, :, 20:], precision)
        ga, gb, gc = a.gather(), b.gather(), c.gather()
        assert torch.equal(ga[0], gb[0]) and torch.equal(ga[1], gb[1]), precision
        assert torch.equal(ga[0], gc[0]) and torch.equal(ga[1], gc[1]), precision
