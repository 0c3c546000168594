"""Direct op handles (reference sources/torchmatch/assignment/ops.py).

``jonker_dense_batch`` is the operator this package implements on CUDA; the
other reference ops are bound only when the reference extension registered
them in this process.
"""

from __future__ import annotations

import torch

_OPS = torch.ops.assignment

jonker_dense_batch = _OPS.jonker_dense_batch
jonker_dense_batch_unpacked = _OPS.jonker_dense_batch_unpacked
# graph-capturable variant: (mapping, device status) without a host sync
jonker_dense_batch_async = _OPS.jonker_dense_batch_async

jonker_compact_batch = _OPS.jonker_compact_batch
jonker_compact_batch_unpacked = _OPS.jonker_compact_batch_unpacked
# fused squared-Euclidean costs from two point sets (x (B, N, D), y (B, M, D))
jonker_sqeuclidean_batch = _OPS.jonker_sqeuclidean_batch

__all__ = ["jonker_compact_batch", "jonker_compact_batch_unpacked", "jonker_dense_batch",
           "jonker_dense_batch_async", "jonker_dense_batch_unpacked",
           "jonker_sqeuclidean_batch"]

for _name in (
    "jonker_scalar", "jonker_dense", "jonker_compact",
    "munkres", "hybrid", "lawler", "greedy",
):
    if hasattr(_OPS, _name):
        globals()[_name] = getattr(_OPS, _name)
        __all__.append(_name)
