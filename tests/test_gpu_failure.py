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


@pytest.fixture
def wait_lib():
    import torchmatch_b200  # noqa: F401
    from torchmatch_b200 import _loader

    core = _loader.core()
    yield core
    core.tm_jv_debug_set_wait_limit(-1)


def _streamed_square(b):
    g = torch.Generator().manual_seed(17)
    return torch.rand(b, 256, 256, generator=g)


@pytest.mark.parametrize("make", [lambda: config2(300), lambda: _streamed_square(64)],
                         ids=["tile64", "ring256"])
def test_tile_wait_timeout_is_reported(wait_lib, oracle_mod, make):
    """A TMA copy whose bounded wait runs out (the hook makes the first wait
    give up at once) -- a 64 x 64 problem's shared-memory tile, or a chunk of
    a streamed 256 x 256 problem's column-reduction ring -- leaves every
    problem as a row of -1, sets TM_WS_TIMEOUT (bit 8) in the async op's
    status and makes the synchronous op raise; the copies in flight still
    land before their shared memory is reused, and resetting the hook brings
    back exact results."""
    lib = wait_lib
    x = make()
    b, n, m = x.shape
    ref = oracle_mod.jonker_dense_batch(x.numpy())
    xd = x.cuda()
    lib.tm_jv_debug_set_wait_limit(0)
    out, status = torch.ops.assignment.jonker_dense_batch_async(xd)
    assert int(status.item()) & 8
    assert (out.cpu().numpy() == -1).all()  # every row written, none left unset
    with pytest.raises(RuntimeError, match="timed out"):
        torch.ops.assignment.jonker_dense_batch(xd)
    # through the C ABI: TM_ERR_TIMEOUT and rows of -1 over a poisoned buffer
    ws = torch.zeros(lib.tm_jv_workspace_bytes(), dtype=torch.uint8, device="cuda")
    got = torch.full((b, n), 7, dtype=torch.long, device="cuda")
    stream = torch.cuda.current_stream().cuda_stream
    rc = lib.tm_jonker_dense_batch_f32(xd.data_ptr(), b, n, m, got.data_ptr(),
                                       ws.data_ptr(), stream)
    assert rc == 7, lib.tm_status_string(rc)
    assert (got.cpu().numpy() == -1).all()
    lib.tm_jv_debug_set_wait_limit(-1)
    np.testing.assert_array_equal(torch.ops.assignment.jonker_dense_batch(xd).cpu().numpy(), ref)
    out, status = torch.ops.assignment.jonker_dense_batch_async(xd)
    assert int(status.item()) == 0
    np.testing.assert_array_equal(out.cpu().numpy(), ref)


def test_sync_op_keeps_unsolved_rows_without_raising(lib, oracle_mod):
    """A loop bound is not an error of the synchronous op: its problems come
    back as rows of -1, as the reference's CPU solver returns them for
    rc != 0 (cpu/ops.cpp:274-278)."""
    x = config2(128)
    ref = oracle_mod.jonker_dense_batch(x.numpy())
    lib.tm_jv_debug_set_loop_bound(3)
    got = torch.ops.assignment.jonker_dense_batch(x.cuda()).cpu().numpy()
    bad = (got != ref).any(axis=1)
    assert bad.any() and (got[bad] == -1).all()
