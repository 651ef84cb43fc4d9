"""CPU-only checks of the boundary: the C-ABI library loads and exports every
declared symbol, and the host-side logic (argument validation, map/code
conversion, the cost model, lazy packed_data views) behaves like the reference."""

import os
import re

import numpy as np
import pytest
import torch

from oracle import shadowkv_oracle as O

REPO = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def _declared_symbols():
    names = set()
    for fn in os.listdir(os.path.join(REPO, "include")):
        if fn.endswith(".h"):
            text = open(os.path.join(REPO, "include", fn)).read()
            names |= set(re.findall(r"\b(skv_[a-z0-9_]+)\s*\(", text))
    return sorted(names)


def test_library_exports_every_declared_symbol():
    from shadow_infer_b200 import _lib
    lib = _lib.load()
    declared = _declared_symbols()
    assert declared, "no declarations found"
    for name in declared:
        assert hasattr(lib, name), name
    assert set(declared) <= set(_lib.EXPORTED_SYMBOLS)


def test_status_strings_and_scratch_queries():
    from shadow_infer_b200 import _lib
    lib = _lib.load()
    assert lib.skv_version().startswith(b"shadowkv_b200")
    assert lib.skv_status_string(0) == b"ok"
    assert lib.skv_status_string(4) == b"scratch buffer too small"
    assert lib.skv_plan_scratch_bytes(8192, 32) >= 4 * 6 * (8192 * 32 // 2048)
    assert lib.skv_evict_scratch_bytes(1 << 20) >= 4 * 4 * ((1 << 20) // 1024)
    assert lib.skv_admit_scratch_bytes(1, 1) > 2048


def test_null_pointer_errors_without_gpu():
    """Argument validation happens on the host before any launch."""
    from shadow_infer_b200 import _lib
    lib = _lib.load()
    assert lib.skv_plan_bucket(None, None, 4, 4, None, None, None, None, None, 0, None) == _lib.SKV_ERR_INVALID_ARGUMENT
    assert b"null pointer" in lib.skv_last_error()
    assert lib.skv_plan_bucket(None, None, 0, 4, None, None, None, None, None, 0, None) == _lib.SKV_ERR_INVALID_ARGUMENT
    assert lib.skv_allocate_codes(None, -1, 1, None, None) == _lib.SKV_ERR_INVALID_ARGUMENT
    with pytest.raises(ValueError):
        _lib.check(_lib.SKV_ERR_SHAPE, "x")
    with pytest.raises(RuntimeError):
        _lib.check(_lib.SKV_ERR_CUDA, "x")


def test_map_codes_roundtrip_matches_oracle():
    from shadow_infer_b200.shadowkv.precision_plan import codes_to_map, map_to_codes
    rng = np.random.default_rng(3)
    codes = rng.integers(0, 5, size=(9, 5)).astype(np.int8)
    pmap = codes_to_map(torch.from_numpy(codes))
    assert pmap[3][2] == O.CODE_PRECISIONS[int(codes[3, 2])]
    assert np.array_equal(map_to_codes(pmap, 9, 5).numpy(), codes)
    # missing entries default to fp16, unknown names raise when strict
    assert map_to_codes({}, 2, 2).tolist() == [[1, 1], [1, 1]]
    with pytest.raises(ValueError, match="Unsupported precision"):
        map_to_codes({0: {0: "int3"}}, 1, 1)
    assert map_to_codes({0: {0: "INT3"}}, 1, 1, strict=False).tolist() == [[1]]
    assert map_to_codes({0: {0: "INT8"}}, 1, 1).tolist() == [[2]]
    with pytest.raises(ValueError, match="Unsupported precision code"):
        codes_to_map(torch.tensor([[7]], dtype=torch.int8))


def test_entry_bytes_matches_oracle():
    from shadow_infer_b200.shadowkv.rd_allocator import entry_bytes
    for p in ("fp32", "fp16", "int8", "int4", "evicted", "FP16"):
        for (b, d, g) in ((1, 128, 16), (8, 128, 16), (2, 63, 16), (3, 40, 16), (1, 64, 0)):
            assert entry_bytes(p, b, d, g) == O.entry_bytes(p, b, d, g)


def test_plan_validation_before_gpu():
    from shadow_infer_b200.shadowkv.precision_plan import PrecisionPlan
    with pytest.raises(ValueError, match="2-D"):
        PrecisionPlan.from_codes(torch.zeros(4, dtype=torch.int8))
    with pytest.raises(ValueError, match="positive"):
        PrecisionPlan.from_codes(torch.zeros(0, 3, dtype=torch.int8))
    with pytest.raises(TypeError):
        PrecisionPlan()


def test_no_cpu_fallback():
    """Without a CUDA device the data plane raises instead of computing on the host."""
    if torch.cuda.is_available():
        pytest.skip("a CUDA device is present")
    from shadow_infer_b200.shadowkv import PackedKVCache, PrecisionPlan
    with pytest.raises(RuntimeError, match="CUDA"):
        PrecisionPlan.from_codes(torch.zeros(4, 2, dtype=torch.int8))
    with pytest.raises(RuntimeError, match="CUDA"):
        PackedKVCache.pack(torch.zeros(1, 2, 4, 8), torch.zeros(1, 2, 4, 8), {}, 16)


def test_lazy_bucket_dict_behaves_like_dict():
    from shadow_infer_b200.shadowkv.packed_kv_cache import _Bucket
    calls = []
    b = _Bucket({"k": 1, "v": 2}, {"indices": lambda: calls.append(1) or [(0, 1)]})
    assert set(b.keys()) == {"k", "v", "indices"} and "indices" in b and len(b) == 3
    assert calls == []
    assert b["indices"] == [(0, 1)] and b.get("indices") == [(0, 1)] and calls == [1]
    assert dict(b.items())["indices"] == [(0, 1)] and calls == [1]
    assert b.get("missing", 5) == 5
    assert isinstance(b, dict)



@pytest.mark.parametrize("B,D,group", [(1, 128, 16), (8, 128, 16), (2, 64, 32), (1, 256, 16), (3, 96, 48)])
def test_slab_layout_agrees_with_library(B, D, group):
    """The host bucket layout of one pack slab and the library's (device) layout need the same
    bytes for any counts: the host makes its tensor views from the former while the kernel
    writes through the latter."""
    import ctypes
    from shadow_infer_b200 import _lib
    from shadow_infer_b200.shadowkv.packed_kv_cache import _int4_group, _slab_layout
    lib = _lib.load()
    rng = np.random.default_rng(B * 1000 + D)
    G = _int4_group(D, group)
    for _ in range(50):
        counts = [int(x) for x in rng.integers(0, 5000, size=6)]
        counts[rng.integers(0, 4)] = 0                       # an empty bucket
        layout, total = _slab_layout(counts, B, D, G)
        arr = (ctypes.c_int64 * 6)(*counts)
        assert lib.skv_pack_slab_bytes(arr, B, D, group) == total
        for parts in layout:
            for _, _, _, off, nb in parts or ():
                assert off % 256 == 0 and off + nb <= total


@pytest.mark.parametrize("B,D,group", [(1, 128, 16), (8, 128, 16), (2, 64, 32), (3, 96, 48)])
def test_empty_slab_array_matches_its_views(B, D, group):
    """An evicted cache's survivors go into a slab whose ``skv_bucket[4]`` array is built from
    the layout arithmetic alone (the compaction writes through it) while the tensor views are
    made later: every pointer and count of the array must be where the views read."""
    from shadow_infer_b200.shadowkv.packed_kv_cache import _empty_slab, _int4_group, _slab_views
    rng = np.random.default_rng(B * 100 + D)
    G = _int4_group(D, group)
    for _ in range(20):
        counts = [int(x) for x in rng.integers(0, 300, size=4)]
        counts[int(rng.integers(0, 4))] = 0
        slab, layout, flat, arr = _empty_slab(counts, B, D, G, torch.device("cpu"))
        views = _slab_views(slab, layout, counts, flat)
        end = slab.data_ptr() + slab.numel()
        for code in range(4):
            if counts[code] == 0:
                assert views[code] is None
                continue
            b, a = views[code], arr[code]
            assert a.count == counts[code] == b["count"] == b["flat"].numel()
            assert a.flat == b["flat"].data_ptr() and b["flat"].dtype == torch.int64
            for key in ("k", "v", "scale_k", "scale_v"):
                t = b[key]
                if t is None:
                    assert getattr(a, key) is None
                else:
                    assert getattr(a, key) == t.data_ptr()
                    assert t.data_ptr() + t.numel() * t.element_size() <= end
