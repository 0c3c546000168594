"""The allocation-free entry point tm_jonker_dense_batch_f32_noalloc.

It exists for callers that cannot allocate device memory (their process has
no cudaMalloc / caching allocator of its own, e.g. a runtime that owns the
GPU's memory).  Here it is called through the C ABI on caller-provided input
and output buffers and must give exactly the mapping of the regular entry
point tm_jonker_dense_batch_f32, on two calls in a row (the shared scratch
keeps the previous call's contents).  Kept in its own file so pytest
collects it last."""

from __future__ import annotations

import numpy as np
import pytest
import torch

pytestmark = pytest.mark.gpu


def _inputs():
    g = torch.Generator().manual_seed(123)
    a = torch.rand(300, 64, 64, generator=g)
    b = torch.rand(97, 40, 70, generator=g) * 10
    b = b.masked_fill(torch.rand(97, 40, 70, generator=g) < 0.3, float("inf"))
    return a, b


def test_noalloc_matches_regular_entry_point_twice():
    from torchmatch_b200 import _loader

    lib = _loader.core()
    stream = torch.cuda.current_stream().cuda_stream
    ws = torch.empty(lib.tm_jv_workspace_bytes(), dtype=torch.uint8, device="cuda")
    for x in _inputs():
        xd = x.cuda()
        b, n, m = x.shape
        ref = torch.empty(b, n, dtype=torch.long, device="cuda")
        got = torch.full((b, n), 7, dtype=torch.long, device="cuda")
        assert lib.tm_jonker_dense_batch_f32(xd.data_ptr(), b, n, m, ref.data_ptr(),
                                             ws.data_ptr(), stream) == 0
        rc = lib.tm_jonker_dense_batch_f32_noalloc(xd.data_ptr(), b, n, m, got.data_ptr(), stream)
        assert rc == 0, lib.tm_status_string(rc)
        torch.cuda.synchronize()
        np.testing.assert_array_equal(got.cpu().numpy(), ref.cpu().numpy())


def test_noalloc_allocates_nothing():
    """Around warm calls, neither the device's free memory nor the torch
    caching allocator's counters move: the entry point allocates nothing."""
    from torchmatch_b200 import _loader

    lib = _loader.core()
    stream = torch.cuda.current_stream().cuda_stream
    x = torch.rand(512, 64, 64, generator=torch.Generator().manual_seed(5)).cuda()
    out = torch.empty(512, 64, dtype=torch.long, device="cuda")
    # the first call loads the module and looks up the scratch address
    assert lib.tm_jonker_dense_batch_f32_noalloc(x.data_ptr(), 512, 64, 64, out.data_ptr(),
                                                 stream) == 0
    torch.cuda.synchronize()
    free0, _ = torch.cuda.mem_get_info()
    stats0 = torch.cuda.memory_stats()
    for _ in range(3):
        assert lib.tm_jonker_dense_batch_f32_noalloc(x.data_ptr(), 512, 64, 64,
                                                     out.data_ptr(), stream) == 0
    torch.cuda.synchronize()
    free1, _ = torch.cuda.mem_get_info()
    stats1 = torch.cuda.memory_stats()
    assert free1 == free0
    for key in ("allocation.all.allocated", "segment.all.allocated", "num_alloc_retries"):
        assert stats1.get(key, 0) == stats0.get(key, 0), key


def test_noalloc_reports_unsolved_rows():
    """The caller cannot read the shared status word, so rows that the loop
    bound left as -1 come back as TM_ERR_UNSOLVED (6)."""
    from torchmatch_b200 import _loader

    lib = _loader.core()
    stream = torch.cuda.current_stream().cuda_stream
    x = torch.rand(64, 64, 64, generator=torch.Generator().manual_seed(6)).cuda()
    out = torch.empty(64, 64, dtype=torch.long, device="cuda")
    lib.tm_jv_debug_set_loop_bound(3)
    try:
        rc = lib.tm_jonker_dense_batch_f32_noalloc(x.data_ptr(), 64, 64, 64, out.data_ptr(),
                                                   stream)
    finally:
        lib.tm_jv_debug_set_loop_bound(0)
    assert rc == 6, lib.tm_status_string(rc)
    assert lib.tm_jonker_dense_batch_f32_noalloc(x.data_ptr(), 64, 64, 64, out.data_ptr(),
                                                 stream) == 0


def test_noalloc_rejects_oversize_and_nan():
    from torchmatch_b200 import _loader

    lib = _loader.core()
    stream = torch.cuda.current_stream().cuda_stream
    x = torch.zeros(1, 257, 257, device="cuda")
    out = torch.empty(1, 257, dtype=torch.long, device="cuda")
    assert lib.tm_jonker_dense_batch_f32_noalloc(x.data_ptr(), 1, 257, 257, out.data_ptr(),
                                                 stream) == 5
    y = torch.ones(2, 3, 3, device="cuda")
    y[1, 1, 1] = float("nan")
    out = torch.empty(2, 3, dtype=torch.long, device="cuda")
    assert lib.tm_jonker_dense_batch_f32_noalloc(y.data_ptr(), 2, 3, 3, out.data_ptr(),
                                                 stream) == 1
