"""The allocation-free plan entry point gives the same results as the regular one.

``skv_plan_bucket_static`` exists for callers that cannot allocate device memory (a
runtime that owns the whole device pool, or code that must stay out of the CUDA
allocator) and therefore cannot pass the scratch buffer ``skv_plan_bucket`` needs.
Both are called here through the C ABI on the same inputs, twice in a row with
different codes, and their outputs (integers: compared exactly) must match.  This
file is collected last on purpose.
"""

import numpy as np
import pytest
import torch

pytestmark = pytest.mark.gpu


def _run_regular(lib, _lib, codes, mask, S, H):
    dev = codes.device
    flat = torch.full((S * H,), -7, dtype=torch.int64, device=dev)
    slot = torch.full((S * H,), -7, dtype=torch.int32, device=dev)
    reuse = torch.full((S * H,), -7, dtype=torch.int64, device=dev)
    counts = torch.full((6,), -7, dtype=torch.int64, device=dev)
    scratch = torch.empty(lib.skv_plan_scratch_bytes(S, H), dtype=torch.uint8, device=dev)
    st = lib.skv_plan_bucket(codes.data_ptr(), mask.data_ptr(), S, H, flat.data_ptr(), slot.data_ptr(),
                             reuse.data_ptr(), counts.data_ptr(), scratch.data_ptr(), scratch.numel(),
                             torch.cuda.current_stream().cuda_stream)
    assert st == 0, _lib.last_error()
    return flat, slot, reuse, counts


def _run_static(lib, _lib, codes, mask, S, H):
    dev = codes.device
    flat = torch.full((S * H,), -9, dtype=torch.int64, device=dev)
    slot = torch.full((S * H,), -9, dtype=torch.int32, device=dev)
    reuse = torch.full((S * H,), -9, dtype=torch.int64, device=dev)
    counts = torch.full((6,), -9, dtype=torch.int64, device=dev)
    st = lib.skv_plan_bucket_static(codes.data_ptr(), mask.data_ptr(), S, H, flat.data_ptr(), slot.data_ptr(),
                                    reuse.data_ptr(), counts.data_ptr(), torch.cuda.current_stream().cuda_stream)
    assert st == 0, _lib.last_error()
    return flat, slot, reuse, counts


def test_static_plan_matches_regular_twice():
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    from shadow_infer_b200 import _lib
    lib = _lib.load()
    gen = torch.Generator().manual_seed(99)
    # second call is smaller and uses different codes: stale tile counts must not leak in
    for S, H in ((4096, 32), (777, 12)):
        codes = torch.randint(0, 5, (S, H), generator=gen, dtype=torch.int8).cuda()
        mask = (torch.rand(S, H, generator=gen) < 0.5).to(torch.uint8).cuda()
        a = _run_regular(lib, _lib, codes, mask, S, H)
        b = _run_static(lib, _lib, codes, mask, S, H)
        torch.cuda.synchronize()
        counts = a[3].cpu()
        nstored = int(counts[:5].sum())
        nreuse = int(counts[5])
        assert torch.equal(a[3], b[3])
        assert torch.equal(a[0][:nstored], b[0][:nstored])
        assert torch.equal(a[1], b[1])
        assert torch.equal(a[2][:nreuse], b[2][:nreuse])
        # and both agree with the row-major definition of the buckets
        c = codes.cpu().numpy().reshape(-1)
        t, h = np.divmod(np.arange(S * H), H)
        want = np.concatenate([(h * S + t)[c == k] for k in range(5)])
        assert np.array_equal(b[0][:nstored].cpu().numpy(), want)


def test_static_plan_rejects_oversize():
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    from shadow_infer_b200 import _lib
    lib = _lib.load()
    limit = lib.skv_plan_static_max_entries()
    assert limit == 4194304
    H = 64
    S = limit // H + 1
    dummy = torch.empty(8, dtype=torch.int64, device="cuda")
    st = lib.skv_plan_bucket_static(dummy.data_ptr(), None, S, H, dummy.data_ptr(), dummy.data_ptr(), None,
                                    dummy.data_ptr(), torch.cuda.current_stream().cuda_stream)
    assert st == _lib.SKV_ERR_TOO_LARGE
    assert "exceeds" in _lib.last_error()
