"""The op refuses CUDA graph capture (reference tests/test_cudagraph_guard.py:
the statistics pass syncs the host, so capture must fail loudly).  Runs in a
subprocess with a wall-clock limit so a regression cannot hang the session."""

from __future__ import annotations

import subprocess
import sys
import textwrap
from pathlib import Path

import pytest

pytestmark = pytest.mark.gpu

ROOT = Path(__file__).resolve().parent.parent

SCRIPT = textwrap.dedent(
    """
    import sys
    sys.path.insert(0, {root!r})
    import torch
    import torchmatch_b200  # noqa: F401
    cost = torch.rand(4, 8, 8, device="cuda")
    static_cost = cost.clone()
    torch.ops.assignment.jonker_dense_batch(static_cost)  # warm-up outside capture
    graph = torch.cuda.CUDAGraph()
    try:
        with torch.cuda.graph(graph):
            torch.ops.assignment.jonker_dense_batch(static_cost)
    except RuntimeError as exc:
        msg = str(exc)
        ok = "CUDA graph capture" in msg and "jonker_dense_batch" in msg
        print("GUARD_RAISED_OK" if ok else "GUARD_RAISED_WRONG_MESSAGE: " + msg)
        sys.exit(0)
    print("GUARD_DID_NOT_RAISE")
    sys.exit(1)
    """
)


def test_op_rejects_cuda_graph_capture():
    r = subprocess.run([sys.executable, "-c", SCRIPT.format(root=str(ROOT))],
                       capture_output=True, text=True, timeout=120)
    assert "GUARD_RAISED_OK" in r.stdout, f"stdout={r.stdout!r} stderr={r.stderr[-2000:]!r}"
