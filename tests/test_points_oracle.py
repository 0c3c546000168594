"""The oracle's squared-Euclidean producer (the checker of the fused
jonker_sqeuclidean_batch op) against a sequential fp32 torch producer.

The fused op defines cell (i, j) as the fp32 sum over d, in order, of
(x_i,d - y_j,d)^2 with every operation rounded on its own.  Elementwise torch
ops on CPU round each operation, so a loop over d gives the same bits;
bar: bit-exact costs, and identical mappings through the oracle solver."""

from __future__ import annotations

import numpy as np
import pytest
import torch


def seq_costs(x: torch.Tensor, y: torch.Tensor) -> torch.Tensor:
    c = torch.zeros(x.shape[0], x.shape[1], y.shape[1], dtype=torch.float32, device=x.device)
    for d in range(x.shape[2]):
        df = x[:, :, None, d] - y[:, None, :, d]
        c = c + df * df
    return c


@pytest.mark.parametrize("b,n,m,d", [(4, 5, 6, 7), (3, 8, 8, 0), (2, 9, 4, 1), (2, 16, 20, 17),
                                     (1, 33, 31, 8), (2, 12, 12, 16)])
def test_producer_bit_exact(oracle_mod, b, n, m, d):
    g = torch.Generator().manual_seed(b * 1000 + n * 10 + d)
    x = torch.randn(b, n, d, generator=g) * 3
    y = torch.randn(b, m, d, generator=g) * 3
    np.testing.assert_array_equal(oracle_mod.sqeuclidean_costs(x, y), seq_costs(x, y).numpy())


def test_fused_oracle_is_dense_oracle_on_costs(oracle_mod):
    g = torch.Generator().manual_seed(11)
    x = torch.randn(64, 24, 16, generator=g)
    y = torch.randn(64, 30, 16, generator=g)
    np.testing.assert_array_equal(oracle_mod.jonker_sqeuclidean_batch(x, y),
                                  oracle_mod.jonker_dense_batch(seq_costs(x, y)))


def test_fused_oracle_integer_ties(oracle_mod):
    # integer coordinates: many equal costs, so tie rules decide the mapping
    g = torch.Generator().manual_seed(12)
    x = torch.randint(0, 3, (32, 20, 2), generator=g).float()
    y = torch.randint(0, 3, (32, 20, 2), generator=g).float()
    np.testing.assert_array_equal(oracle_mod.jonker_sqeuclidean_batch(x, y),
                                  oracle_mod.jonker_dense_batch(seq_costs(x, y)))


def test_producer_rejects_bad_shapes(oracle_mod):
    with pytest.raises(ValueError):
        oracle_mod.sqeuclidean_costs(np.zeros((2, 3, 4)), np.zeros((2, 3, 5)))
