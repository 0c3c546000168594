"""Fused cost construction on CUDA: jonker_sqeuclidean_batch(x, y).

Bar: bit-exact int64 mappings.  The op must equal (1) the oracle's
restated producer + solver (oracle/jv_oracle.c) and (2) the CUDA
jonker_dense_batch on costs that a sequential fp32 torch producer wrote, on
every storage mode of the solve kernel: problems built in the shared-memory
tile, and larger ones built in per-warp slabs of the workspace (square and
rectangular, vector widths 4 and 1, D across the 8-coordinate chunking)."""

from __future__ import annotations

import numpy as np
import pytest
import torch

from test_points_oracle import seq_costs

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def ops():
    import torchmatch_b200  # noqa: F401

    assert torch.cuda.is_available()
    return torch.ops.assignment


def _points(b, n, m, d, seed, scale=1.0, integer=False):
    g = torch.Generator().manual_seed(seed)
    if integer:
        x = torch.randint(0, 4, (b, n, d), generator=g).float()
        y = torch.randint(0, 4, (b, m, d), generator=g).float()
    else:
        x = torch.randn(b, n, d, generator=g) * scale
        y = torch.randn(b, m, d, generator=g) * scale
    return x, y


SHAPES = [
    # (B, N, M, D)        storage mode of the solve kernel
    (64, 32, 32, 16),     # tile, K = 32
    (512, 64, 64, 16),    # tile, config-2 shape
    (256, 100, 150, 8),   # tile, rectangular
    (96, 128, 128, 16),   # slabs, S = 4, square, vector loads
    (64, 130, 97, 3),     # tile at S = 5, generic producer
    (64, 200, 150, 3),    # slabs, S = 7, rectangular, scalar loads
    (40, 200, 256, 16),   # slabs, S = 8, rectangular, vector loads
    (48, 256, 256, 16),   # slabs, S = 8, square (config-5 shape)
    (24, 256, 255, 33),   # slabs, S = 8, scalar loads, D with a ragged chunk
    (32, 256, 256, 32),   # slabs, blocked producer over two coordinate chunks
    (128, 64, 64, 32),    # tile, blocked producer over two coordinate chunks
    (64, 45, 37, 16),     # tile, blocked producer with a partial row block
    (64, 130, 97, 16),    # tile at S = 5 (rectangular), blocked producer
    (64, 8, 250, 16),     # tile at S = 8 (few rows, wide)
    (32, 180, 60, 7),     # tile at S = 6, generic producer
    (32, 40, 40, 1),
    (16, 24, 30, 0),      # D = 0: every cost is 0
]


@pytest.mark.parametrize("b,n,m,d", SHAPES)
def test_matches_oracle(ops, oracle_mod, b, n, m, d):
    x, y = _points(b, n, m, d, seed=b + n + m + d)
    got = ops.jonker_sqeuclidean_batch(x.cuda(), y.cuda()).cpu().numpy()
    np.testing.assert_array_equal(got, oracle_mod.jonker_sqeuclidean_batch(x, y))


@pytest.mark.parametrize("b,n,m,d", [(256, 64, 64, 16), (64, 128, 128, 16), (32, 256, 256, 16),
                                     (64, 120, 80, 5)])
def test_matches_dense_op_on_materialised_costs(ops, b, n, m, d):
    x, y = _points(b, n, m, d, seed=7 * b + d)
    xc, yc = x.cuda(), y.cuda()
    want = ops.jonker_dense_batch(seq_costs(xc, yc))
    torch.testing.assert_close(ops.jonker_sqeuclidean_batch(xc, yc), want, rtol=0, atol=0)


@pytest.mark.parametrize("n", [64, 128, 256])
def test_integer_points_ties(ops, oracle_mod, n):
    x, y = _points(64, n, n, 2, seed=n, integer=True)
    got = ops.jonker_sqeuclidean_batch(x.cuda(), y.cuda()).cpu().numpy()
    np.testing.assert_array_equal(got, oracle_mod.jonker_sqeuclidean_batch(x, y))


def test_config5_scale_properties(ops, oracle_mod):
    # the config-5 distribution at 2048 problems: a permutation per problem,
    # identical to the oracle on a strided sample
    x, y = _points(2048, 256, 256, 16, seed=5)
    got = ops.jonker_sqeuclidean_batch(x.cuda(), y.cuda()).cpu()
    assert torch.equal(got.sort(dim=1).values, torch.arange(256).expand(2048, 256))
    idx = torch.arange(0, 2048, 37)
    np.testing.assert_array_equal(got[idx].numpy(),
                                  oracle_mod.jonker_sqeuclidean_batch(x[idx], y[idx]))


def test_infinite_coordinates_use_the_sentinel(ops, oracle_mod):
    # a +inf coordinate makes that row's costs +inf: the batch-global
    # sentinel path, as in the dense op
    x, y = _points(32, 70, 90, 4, seed=21)
    x[3, 5, 2] = float("inf")
    y[9, 11, 0] = float("-inf")
    got = ops.jonker_sqeuclidean_batch(x.cuda(), y.cuda()).cpu().numpy()
    np.testing.assert_array_equal(got, oracle_mod.jonker_sqeuclidean_batch(x, y))
    x2, y2 = _points(8, 140, 140, 4, seed=22)   # slab mode
    x2[1, 0, 0] = float("inf")
    got = ops.jonker_sqeuclidean_batch(x2.cuda(), y2.cuda()).cpu().numpy()
    np.testing.assert_array_equal(got, oracle_mod.jonker_sqeuclidean_batch(x2, y2))


def test_nan_raises(ops):
    x, y = _points(4, 16, 16, 3, seed=1)
    x[2, 3, 1] = float("nan")
    with pytest.raises(RuntimeError, match="NaN"):
        ops.jonker_sqeuclidean_batch(x.cuda(), y.cuda())
    # inf - inf is NaN too
    x, y = _points(4, 16, 16, 3, seed=2)
    x[0, 0, 0] = float("inf")
    y[0, 0, 0] = float("inf")
    with pytest.raises(RuntimeError, match="NaN"):
        ops.jonker_sqeuclidean_batch(x.cuda(), y.cuda())


def test_shapes_and_errors(ops):
    e = torch.empty
    assert ops.jonker_sqeuclidean_batch(e(0, 4, 3, device="cuda"),
                                        e(0, 5, 3, device="cuda")).shape == (0, 4)
    out = ops.jonker_sqeuclidean_batch(e(2, 4, 3, device="cuda"), e(2, 0, 3, device="cuda"))
    assert out.shape == (2, 4) and bool((out == -1).all())
    with pytest.raises(RuntimeError, match="agree"):
        ops.jonker_sqeuclidean_batch(e(2, 4, 3, device="cuda"), e(2, 4, 2, device="cuda"))
    with pytest.raises(RuntimeError, match="256"):
        ops.jonker_sqeuclidean_batch(e(1, 257, 3, device="cuda"), e(1, 4, 3, device="cuda"))


def test_float64_and_noncontiguous(ops, oracle_mod):
    x, y = _points(16, 48, 48, 6, seed=3)
    xt = x.double().cuda().transpose(1, 2).contiguous().transpose(1, 2)
    got = ops.jonker_sqeuclidean_batch(xt, y.double().cuda()).cpu().numpy()
    np.testing.assert_array_equal(got, oracle_mod.jonker_sqeuclidean_batch(x, y))


def test_c_abi_small_workspace_and_arguments(oracle_mod):
    # through the C ABI: a workspace holding a single slab runs one warp at
    # a time and still gives the same mapping; bad arguments are refused
    from torchmatch_b200 import _loader

    lib = _loader.core()
    b, n, m, d = 12, 160, 160, 8
    x, y = _points(b, n, m, d, seed=4)
    xc, yc = x.cuda(), y.cuda()
    out = torch.empty(b, n, dtype=torch.long, device="cuda")
    stream = torch.cuda.current_stream().cuda_stream
    full = lib.tm_jv_points_workspace_bytes(b, n, m)
    slab = ((n * m + 63) // 64 * 64) * 4
    assert full >= 256 + slab
    want = oracle_mod.jonker_sqeuclidean_batch(x, y)
    for nbytes in (full, 256 + slab):
        ws = torch.empty(nbytes, dtype=torch.uint8, device="cuda")
        rc = lib.tm_jonker_sqeuclidean_batch_f32(xc.data_ptr(), yc.data_ptr(), b, n, m, d,
                                                 out.data_ptr(), ws.data_ptr(), nbytes, stream)
        assert rc == 0, lib.tm_status_string(rc)
        np.testing.assert_array_equal(out.cpu().numpy(), want)
    ws = torch.empty(full + 256, dtype=torch.uint8, device="cuda")
    args = (xc.data_ptr(), yc.data_ptr(), b, n, m, d, out.data_ptr())
    assert lib.tm_jonker_sqeuclidean_batch_f32(*args, ws.data_ptr() + 16, full, stream) == 3
    assert lib.tm_jonker_sqeuclidean_batch_f32(*args, ws.data_ptr(), 256 + slab - 4,
                                               stream) == 3
    assert lib.tm_jonker_sqeuclidean_batch_f32(xc.data_ptr(), yc.data_ptr(), b, 300, m, d,
                                               out.data_ptr(), ws.data_ptr(), full,
                                               stream) == 5
    # shapes solved in the tile need only the 256-byte header
    assert lib.tm_jv_points_workspace_bytes(64, 64, 64) == 256


@pytest.mark.parametrize("d", [5, 16])
def test_shape_sweep(ops, oracle_mod, d):
    # every slot count, square and rectangular, tile and slab storage
    g = torch.Generator().manual_seed(d)
    for k in range(1, 257, 17):
        for n, m in ((k, k), (k, max(1, k // 2 + 3)), (max(1, k // 3), k)):
            x = torch.randn(6, n, d, generator=g)
            y = torch.randn(6, m, d, generator=g)
            got = ops.jonker_sqeuclidean_batch(x.cuda(), y.cuda()).cpu().numpy()
            np.testing.assert_array_equal(got, oracle_mod.jonker_sqeuclidean_batch(x, y),
                                          err_msg=f"n={n} m={m} d={d}")


def test_opcheck(ops):
    x, y = _points(8, 20, 24, 5, seed=9)
    torch.library.opcheck(ops.jonker_sqeuclidean_batch, (x.cuda(), y.cuda()),
                          test_utils=("test_schema", "test_faketensor"))


SHARDED_SCRIPT = """
import os, sys
sys.path.insert(0, {root!r}); sys.path.insert(0, {root!r} + "/tests")
os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT="29541", RANK="0", WORLD_SIZE="1")
import numpy as np, torch, torch.distributed as dist
import oracle, torchmatch_b200
from torchmatch_b200 import sharded
torch.cuda.set_device(0)
dist.init_process_group("nccl", device_id=torch.device("cuda", 0))
g = torch.Generator().manual_seed(31)
for b, n, m, d, inf in ((64, 64, 64, 16, False), (32, 200, 180, 16, True), (16, 90, 120, 5, True)):
    x = torch.randn(b, n, d, generator=g); y = torch.randn(b, m, d, generator=g)
    if inf:
        x[1, 2, 0] = float("inf")
    got = sharded.solve_points_sharded(x.cuda(), y.cuda()).cpu().numpy()
    assert np.array_equal(got, oracle.jonker_sqeuclidean_batch(x, y)), (b, n, m, d)
x = torch.randn(4, 8, 3, generator=g); x[0, 0, 0] = float("nan")
try:
    sharded.solve_points_sharded(x.cuda(), torch.randn(4, 8, 3).cuda())
    print("NO_RAISE")
except RuntimeError as e:
    assert "NaN" in str(e)
dist.destroy_process_group()
print("POINTS_SHARDED_OK")
"""


def test_solve_points_sharded_one_rank():
    import subprocess
    import sys
    from pathlib import Path

    root = str(Path(__file__).resolve().parent.parent)
    r = subprocess.run([sys.executable, "-c", SHARDED_SCRIPT.format(root=root)],
                       capture_output=True, text=True, timeout=300)
    assert "POINTS_SHARDED_OK" in r.stdout, r.stdout[-2000:] + r.stderr[-3000:]
