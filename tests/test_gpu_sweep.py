"""Seeded random sweep: many small shapes and cost distributions, dense and
compact, CUDA against the oracle (bit-exact).  Distributions cover the
paths that are hard to reach with the fixed configurations: heavy integer
ties (Dijkstra events), +inf masks (sentinel), negative costs, huge costs
(the LARGE / FLT_MAX fallbacks) and extreme aspect ratios."""

from __future__ import annotations

import numpy as np
import pytest
import torch

pytestmark = pytest.mark.gpu


def _batch(rng: np.random.Generator, kind: str, b: int, n: int, m: int) -> np.ndarray:
    if kind == "uniform":
        x = rng.random((b, n, m))
    elif kind == "ties":
        x = rng.integers(0, 3, (b, n, m)).astype(np.float64)
    elif kind == "inf":
        x = rng.random((b, n, m)) * 5
        x[rng.random((b, n, m)) < 0.4] = np.inf
    elif kind == "negative":
        x = rng.normal(size=(b, n, m)) * 100
    elif kind == "huge":
        x = rng.random((b, n, m)) * 3e18
    else:
        x = np.round(rng.random((b, n, m)) * 4) / 4 - 0.5
    return x.astype(np.float32)


KINDS = ("uniform", "ties", "inf", "negative", "huge", "quarters")
CASES = [(seed, kind) for seed in range(6) for kind in KINDS]


@pytest.mark.parametrize("seed,kind", CASES)
@pytest.mark.parametrize("variant", ["dense", "compact"])
def test_random_shapes(seed, kind, variant, oracle_mod):
    import torchmatch_b200  # noqa: F401

    rng = np.random.default_rng(1000 * seed + KINDS.index(kind))
    op = getattr(torch.ops.assignment, f"jonker_{variant}_batch")
    ref = getattr(oracle_mod, f"jonker_{variant}_batch")
    for _ in range(4):
        n, m = (int(v) for v in rng.integers(1, 41, 2))
        if rng.random() < 0.2:
            n = int(rng.integers(1, 200))
        b = int(rng.integers(1, 40))
        x = _batch(rng, kind, b, n, m)
        np.testing.assert_array_equal(op(torch.from_numpy(x).cuda()).cpu().numpy(), ref(x),
                                      err_msg=f"{variant} {kind} shape {x.shape}")
