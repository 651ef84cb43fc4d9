"""PagedKVStore host logic without a GPU: constructor and argument validation (every refusal
happens before any device work, leaving the store untouched), empty-store accounting and
gather, and the C ABI's own checks of page writes (paged_kv_store.py)."""

import ctypes

import numpy as np
import pytest
import torch

from shadow_infer_b200 import _lib
from shadow_infer_b200.shadowkv import PagedKVStore
from shadow_infer_b200.shadowkv.paged_kv_store import _DESC, _DESC_S, _WRITE, _WRITE_S


def _store(**kw):
    return PagedKVStore(2, 4, 32, page_size=kw.pop("page_size", 8), device="cpu", int4_group_size=16, **kw)


def test_constructor_validation_and_initial_state():
    with pytest.raises(ValueError):
        PagedKVStore(1, 1, 8, page_size=0)
    with pytest.raises(ValueError):
        PagedKVStore(1, 1, 8, int4_group_size=0)
    s = _store()
    assert (s.max_seq, s.page_count, s.open_pages, s.appended_tokens, s.page_evictions) == (0, 0, 0, 0, 0)
    assert (s.rewritten_tokens, s.rewritten_pages) == (0, 0)
    assert s.data_plane_bytes() == 0 and s.resident_bytes() == 0
    k, v = s.gather()
    assert k.shape == (2, 4, 0, 32) and v.shape == (2, 4, 0, 32) and k.dtype == torch.float32
    assert s.evict_tokens({(0, 0)}) == 0 and s.evict_tokens(set()) == 0
    assert "page_size=8" in repr(s) and "pages=0" in repr(s)
    assert PagedKVStore(1, 1, 40, int4_group_size=16)._int4_effective_group == 40
    assert PagedKVStore(1, 1, 48, int4_group_size=24)._int4_effective_group == 24


def test_validate_against():
    s = _store()
    s.validate_against(2, 4, 32)
    for bad in ((3, 4, 32), (2, 5, 32), (2, 4, 33)):
        with pytest.raises(ValueError, match="shape mismatch"):
            s.validate_against(*bad)


@pytest.mark.parametrize("k_shape,v_shape,precision", [
    ((2, 4, 3, 32), (2, 4, 3, 32), "bf16"),
    ((2, 4, 3), (2, 4, 3, 32), "fp16"),
    ((2, 4, 3, 32), (2, 4, 2, 32), "fp16"),
    ((3, 4, 3, 32), (3, 4, 3, 32), "fp16"),
    ((2, 5, 3, 32), (2, 5, 3, 32), "int8"),
    ((2, 4, 3, 31), (2, 4, 3, 31), "int4"),
])
def test_append_and_rewrite_refusals_before_device_work(k_shape, v_shape, precision):
    s = _store()
    with pytest.raises(ValueError):
        s.append(torch.zeros(k_shape), torch.zeros(v_shape), precision)
    with pytest.raises(ValueError):
        s.rewrite_tokens(0, torch.zeros(k_shape), torch.zeros(v_shape), precision)
    assert s.max_seq == 0 and s.appended_tokens == 0 and s.page_count == 0


def test_zero_token_append_is_a_noop_and_rewrite_range_checks():
    s = _store()
    s.append(torch.zeros(2, 4, 0, 32), torch.zeros(2, 4, 0, 32), "fp16")
    assert s.max_seq == 0 and s.appended_tokens == 0
    with pytest.raises(ValueError, match="at least one token"):
        s.rewrite_tokens(0, torch.zeros(2, 4, 0, 32), torch.zeros(2, 4, 0, 32), "fp16")
    with pytest.raises(ValueError, match="exceeds stored range"):
        s.rewrite_tokens(0, torch.zeros(2, 4, 1, 32), torch.zeros(2, 4, 1, 32), "fp16")


def test_record_layouts_match_the_c_structs():
    assert _DESC.itemsize == 64 and _WRITE.itemsize == 88 and _DESC_S.size == 64 and _WRITE_S.size == 88
    assert _WRITE.fields["src_token"][1] == 64 and _WRITE.fields["table_pos"][1] == 80
    rec = np.frombuffer(_WRITE_S.pack(1, 2, 3, 4, 5, 6, 7, 3, 0, 0, 0, 8, 9, 10, 11, 0), dtype=_WRITE)[0]
    assert (rec["page"]["k"], rec["page"]["scale_v"], rec["page"]["start_token"], rec["page"]["num_tokens"]) == \
        (1, 4, 5, 6)
    assert (rec["page"]["row_stride"], rec["page"]["precision"], rec["src_token"], rec["dst_row"], rec["rows"],
            rec["table_pos"]) == (7, 3, 8, 9, 10, 11)


def test_abi_page_write_checks():
    lib = _lib.load()
    w = np.zeros(1, dtype=_WRITE)
    w["page"]["k"] = w["page"]["v"] = 1 << 20
    w["page"]["num_tokens"], w["page"]["row_stride"], w["page"]["precision"] = 4, 8, 1
    w["rows"], w["dst_row"], w["src_token"] = 2, 3, 0                  # rows 3..4 of a 4-row page
    args = (1 << 20, 1 << 20, 2, 4, 2, 32, 16, w.ctypes.data, 1, None, None)
    assert lib.skv_paged_write(*args) == _lib.SKV_ERR_SHAPE
    w["dst_row"], w["src_token"] = 0, 1                                   # source rows 1..2 of 2
    assert lib.skv_paged_write(*args) == _lib.SKV_ERR_SHAPE
    w["src_token"], w["page"]["precision"] = 0, 2                         # int8 page without scales
    assert lib.skv_paged_write(*args) == _lib.SKV_ERR_INVALID_ARGUMENT
    w["page"]["precision"] = 7
    assert lib.skv_paged_write(*args) == _lib.SKV_ERR_INVALID_ARGUMENT
    assert lib.skv_paged_write(None, None, 2, 4, 2, 32, 16, w.ctypes.data, 1, None, None) == \
        _lib.SKV_ERR_INVALID_ARGUMENT
    assert lib.skv_paged_write(1, 1, 2, 4, 2, 32, 16, w.ctypes.data, 0, None, None) == _lib.SKV_OK   # nothing to do
    assert lib.skv_paged_gather(None, 0, 2, 4, 32, 16, 8, 8, None, None, None) == _lib.SKV_ERR_INVALID_ARGUMENT
    assert lib.skv_paged_gather(None, 0, 2, 4, 32, 16, 0, 0, ctypes.c_void_p(1), ctypes.c_void_p(1), None) == \
        _lib.SKV_OK                                                       # empty result, no launch
    assert lib.skv_paged_clear_heads(None, 1, None, 1, 2, 4, 32, None, None) == _lib.SKV_ERR_INVALID_ARGUMENT
