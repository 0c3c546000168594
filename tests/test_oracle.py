"""The CPU oracle (oracle/jv_oracle.c) pinned against the reference.

Golden vectors come from the reference's own jonker_dense_batch
(tests/golden/make_golden.py); oracle/_ref is the reference's solver core
compiled from its sources, checked where it was built.
"""

from __future__ import annotations

import numpy as np
import pytest
import torch

from cases import CASES, config2, config3, config4, config5_chunk, digest


@pytest.mark.parametrize("name", sorted(CASES))
def test_oracle_matches_golden(name, golden, oracle_mod):
    outs, meta = golden
    x = CASES[name]()
    assert digest(x) == meta[name]["sha256"], "input recipe drifted"
    got = oracle_mod.jonker_dense_batch(x.numpy())
    np.testing.assert_array_equal(got, outs[name])


def _ref_cases():
    return {
        "config2": config2(256),
        "config3": config3(64),
        "config4": config4(128),
        "config5": config5_chunk(8, 3),
        "ties": torch.randint(0, 5, (256, 24, 24), generator=torch.Generator().manual_seed(11)).float(),
    }


@pytest.mark.parametrize("name", ["config2", "config3", "config4", "config5", "ties"])
def test_oracle_matches_compiled_reference(name, oracle_mod):
    if not oracle_mod.reference_available():
        pytest.skip("oracle/_ref not built (reference tree absent)")
    x = _ref_cases()[name].numpy()
    np.testing.assert_array_equal(
        oracle_mod.jonker_dense_batch(x), oracle_mod.reference_jonker_dense_batch(x)
    )


def test_oracle_rejects_nan_and_neg_inf(oracle_mod):
    x = np.ones((2, 3, 3), np.float32)
    x[1, 0, 2] = np.nan
    with pytest.raises(RuntimeError, match="NaN"):
        oracle_mod.jonker_dense_batch(x)
    x[1, 0, 2] = -np.inf
    with pytest.raises(RuntimeError, match="-inf"):
        oracle_mod.jonker_dense_batch(x)


def test_oracle_empty_shapes(oracle_mod):
    assert oracle_mod.jonker_dense_batch(np.zeros((0, 3, 3), np.float32)).shape == (0, 3)
    out = oracle_mod.jonker_dense_batch(np.zeros((2, 3, 0), np.float32))
    assert out.shape == (2, 3) and (out == -1).all()


def test_oracle_is_a_valid_optimum(oracle_mod):
    scipy = pytest.importorskip("scipy.optimize")
    x = config2(32).numpy()
    out = oracle_mod.jonker_dense_batch(x)
    for b in range(x.shape[0]):
        assert sorted(out[b]) == list(range(64))
        r, c = scipy.linear_sum_assignment(x[b].astype(np.float64))
        opt = x[b].astype(np.float64)[r, c].sum()
        got = x[b].astype(np.float64)[np.arange(64), out[b]].sum()
        assert abs(got - opt) < 1e-5


@pytest.mark.parametrize("name", sorted(CASES))
def test_compact_oracle_matches_golden(name, golden, oracle_mod):
    outs, _ = golden
    got = oracle_mod.jonker_compact_batch(CASES[name]().numpy())
    np.testing.assert_array_equal(got, outs["compact__" + name])


@pytest.mark.parametrize("name", ["config2", "config3", "config4", "config5", "ties"])
def test_compact_oracle_matches_compiled_reference(name, oracle_mod):
    if not oracle_mod.reference_available():
        pytest.skip("oracle/_ref not built (reference tree absent)")
    x = _ref_cases()[name].numpy()
    np.testing.assert_array_equal(
        oracle_mod.jonker_compact_batch(x), oracle_mod.reference_jonker_compact_batch(x)
    )
