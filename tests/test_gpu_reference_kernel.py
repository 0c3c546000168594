"""The reference's own batched CUDA kernel (cuda/jonker_tiled.cuh, built from
its sources into oracle/_ref by oracle/Makefile) against this package on the
shapes it supports (square K <= 64, finite costs).  It runs a different
algorithm (successive shortest paths), so the bar is the optimal total: the
float64 totals of both mappings agree to fp32 rounding, and both are
permutations."""

from __future__ import annotations

import numpy as np
import pytest
import torch

from cases import config1, config2

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize("make", [lambda: config1(), lambda: config2(4096)])
def test_reference_cuda_kernel_same_optimum(make, oracle_mod):
    import torchmatch_b200  # noqa: F401

    if not oracle_mod.reference_cuda_available():
        pytest.skip("oracle/_ref/libtmref_cuda.so not built (reference tree absent)")
    x = make().cuda().contiguous()
    ref = oracle_mod.reference_cuda_jonker_dense_batch(x).cpu()
    ours = torch.ops.assignment.jonker_dense_batch(x).cpu()
    k = x.shape[1]
    assert torch.equal(ref.sort(dim=1).values, torch.arange(k).expand_as(ref))
    c = x.double().cpu()
    tot = lambda m: c.gather(2, m[:, :, None]).sum(dim=(1, 2)).numpy()  # noqa: E731
    np.testing.assert_allclose(tot(ref), tot(ours), rtol=1e-5, atol=1e-6)
    # on continuous costs the optimum is unique: the mappings coincide almost always
    assert (ref == ours).all(dim=1).float().mean() > 0.99
