"""Host logic of batch sharding (torchmatch_b200/sharded.py) with two gloo
ranks on CPU: the merged statistics of contiguous slices give exactly the
sentinel of the whole batch (reference cpu/ops.cpp:67-93), and NaN / -inf on
any one rank is raised on every rank."""

from __future__ import annotations

import os
import socket

import numpy as np
import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from torchmatch_b200 import sharded


def host_words(x: np.ndarray) -> list[int]:
    """What tm_jv_stats_f32 reports for x, computed on the host."""
    fin = x[np.isfinite(x)]
    flags = (1 if np.isnan(x).any() else 0) | (2 if (x == -np.inf).any() else 0)
    flags |= (4 if fin.size else 0) | (8 if (x == np.inf).any() else 0)
    key = sharded.order_key(float(fin.max())) if fin.size else 0
    return sharded.stats_words(flags, key)


def reference_sentinel(x: np.ndarray, k: int) -> float:
    fin = x[np.isfinite(x)].astype(np.float32)
    if not fin.size:
        return 1.0
    return float((fin.max() + np.float32(1)) * np.float32(k + 1))


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _worker(rank, world, port, batch, q):
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        lo, hi = sharded.shard_bounds(batch.shape[0], world)[rank]
        words = sharded.merge_words(host_words(batch[lo:hi]))
        try:
            q.put((rank, "ok", sharded.sentinel_from_words(words, max(batch.shape[1:]))))
        except RuntimeError as e:
            q.put((rank, "err", str(e)))
    finally:
        dist.destroy_process_group()


def _run(batch: np.ndarray):
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, 2, port, batch, q)) for r in range(2)]
    for p in procs:
        p.start()
    res = [q.get(timeout=120) for _ in procs]
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    return sorted(res)


def test_merged_sentinel_equals_whole_batch():
    g = np.random.default_rng(0)
    x = (g.random((6, 5, 7)) * 10).astype(np.float32)
    x[4, 1, 2] = 42.5  # the max sits in rank 1's slice
    x[0, 0, 0] = np.inf  # +inf only in rank 0's slice
    res = _run(x)
    want = reference_sentinel(x, 7)
    for rank, kind, val in res:
        assert kind == "ok"
        sentinel, pinf = val
        assert np.float32(sentinel) == np.float32(want) and pinf


@pytest.mark.parametrize("bad,msg", [(np.nan, "NaN"), (-np.inf, "-inf")])
def test_error_on_one_rank_raises_everywhere(bad, msg):
    x = np.ones((4, 3, 3), np.float32)
    x[3, 2, 2] = bad  # in rank 1's slice only
    res = _run(x)
    assert [r[1] for r in res] == ["err", "err"]
    assert all(msg in r[2] for r in res)


def test_shard_bounds():
    assert sharded.shard_bounds(10, 4) == [(0, 3), (3, 6), (6, 9), (9, 10)]
    assert sharded.shard_bounds(2, 4) == [(0, 1), (1, 2), (2, 2), (2, 2)]
    assert sharded.shard_bounds(65536, 8)[7] == (57344, 65536)


def test_solve_points_sharded_rejects_bad_shapes():
    # shape checks run before any device work
    with pytest.raises(RuntimeError, match="x must be"):
        sharded.solve_points_sharded(torch.zeros(2, 3, 4), torch.zeros(2, 3, 5))
    with pytest.raises(RuntimeError, match="x must be"):
        sharded.solve_points_sharded(torch.zeros(2, 3, 4), torch.zeros(3, 3, 4))
    with pytest.raises(RuntimeError, match="x must be"):
        sharded.solve_points_sharded(torch.zeros(3, 4), torch.zeros(3, 4))
