"""The solver's loop-bound failure path, driven from the host without any
GPU fault: a test hook lowers every loop cap, problems that need more steps
come back as rows of -1 with TM_WS_UNSOLVED (bit 4) in the device status, the
rest stay exact, and restoring the bound restores full results."""

from __future__ import annotations

import numpy as np
import pytest
import torch

from cases import config2, config4

pytestmark = pytest.mark.gpu


@pytest.fixture
def lib():
    import torchmatch_b200  # noqa: F401
    from torchmatch_b200 import _loader

    core = _loader.core()
    yield core
    core.tm_jv_debug_set_loop_bound(0)


@pytest.mark.parametrize("make", [lambda: config2(256), lambda: config4(256)])
def test_loop_bound_marks_rows_unsolved(lib, make, oracle_mod):
    x = make()
    ref = oracle_mod.jonker_dense_batch(x.numpy())
    lib.tm_jv_debug_set_loop_bound(3)
    out, status = torch.ops.assignment.jonker_dense_batch_async(x.cuda())
    got = out.cpu().numpy()
    assert int(status.item()) & 4, "no problem reported unsolved under a bound of 3"
    bad = (got != ref).any(axis=1)
    assert bad.any() and (got[bad] == -1).all()  # failed problems are whole rows of -1
    lib.tm_jv_debug_set_loop_bound(0)
    out, status = torch.ops.assignment.jonker_dense_batch_async(x.cuda())
    assert int(status.item()) == 0
    np.testing.assert_array_equal(out.cpu().numpy(), ref)
