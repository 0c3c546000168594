"""GPU checks of the sharded entry points and of the check-mode solve.

* tm_jv_solve_checked_f32: all-finite problems solved exactly, problems with
  non-finite cells left as rows of -1, batch statistics accumulated.
* sharded.solve_sharded on a one-rank NCCL group (in a subprocess), with and
  without +inf cells, against the oracle.
* sharded.solve_multi_gpu over every visible GPU against the oracle.
"""

from __future__ import annotations

import subprocess
import sys
import textwrap
from pathlib import Path

import numpy as np
import pytest
import torch

from cases import config2, config4

pytestmark = pytest.mark.gpu
ROOT = Path(__file__).resolve().parent.parent


def test_checked_solve_semantics(oracle_mod):
    from torchmatch_b200 import _loader

    lib = _loader.core()
    x = config2(64)
    x[5, 3, 7] = float("inf")
    x[9, 0, 0] = float("nan")
    xd = x.cuda()
    out = torch.empty(64, 64, dtype=torch.long, device="cuda")
    ws = torch.zeros(lib.tm_jv_workspace_bytes() // 4, dtype=torch.int32, device="cuda")
    rc = lib.tm_jv_solve_checked_f32(xd.data_ptr(), 64, 64, 64, out.data_ptr(), ws.data_ptr(),
                                     torch.cuda.current_stream().cuda_stream)
    assert rc == 0
    got = out.cpu().numpy()
    flags = int(ws[0].item()) & 0xFFFFFFFF
    assert flags & 1 and flags & 8 and flags & 4 and not flags & 2
    assert (got[5] == -1).all() and (got[9] == -1).all()
    keep = [b for b in range(64) if b not in (5, 9)]
    np.testing.assert_array_equal(got[keep], oracle_mod.jonker_dense_batch(x.numpy()[keep]))


SCRIPT = textwrap.dedent(
    """
    import os, sys
    sys.path.insert(0, {root!r}); sys.path.insert(0, {root!r} + "/tests/golden")
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT="29533", RANK="0", WORLD_SIZE="1")
    import numpy as np, torch, torch.distributed as dist
    import oracle, torchmatch_b200
    from torchmatch_b200 import sharded
    from cases import config2, config4
    torch.cuda.set_device(0)
    dist.init_process_group("nccl", device_id=torch.device("cuda", 0))
    for x in (config2(512), config4(512)):
        got = sharded.solve_sharded(x.cuda()).cpu().numpy()
        assert np.array_equal(got, oracle.jonker_dense_batch(x.numpy())), x.shape
    bad = config2(8).cuda(); bad[3, 1, 1] = float("-inf")
    try:
        sharded.solve_sharded(bad)
        print("NO_RAISE")
    except RuntimeError as e:
        assert "-inf" in str(e)
    dist.destroy_process_group()
    print("SHARDED_OK")
    """
)


def test_solve_sharded_one_rank():
    r = subprocess.run([sys.executable, "-c", SCRIPT.format(root=str(ROOT))],
                       capture_output=True, text=True, timeout=300)
    assert "SHARDED_OK" in r.stdout, r.stdout[-2000:] + r.stderr[-3000:]


def test_solve_multi_gpu(oracle_mod):
    from torchmatch_b200 import sharded

    x = config4(300)
    got = sharded.solve_multi_gpu(x.cuda(0)).cpu().numpy()
    np.testing.assert_array_equal(got, oracle_mod.jonker_dense_batch(x.numpy()))
