"""Dispatcher over ``torch.ops.assignment`` -- the reference's ``solve`` surface.

Same public names, arguments and error types as tue-p8n/torchmatch 1.0.3
``torchmatch.assignment.solve`` / ``resolve_backend`` / ``Backend``
(sources/torchmatch/assignment/_solve.py:25-330).  One routing change, the
point of this package: on CUDA every 3-D problem with max(N, M) <= 256 --
square or rectangular -- goes to ``jonker_dense_batch`` (the reference
capped it at square K <= 64, _solve.py:95-97 and :180-201, and looped a 2-D
op over the batch otherwise), and a 2-D CUDA problem under
``Backend.JONKER`` is solved as a batch of one instead of raising.

CPU tensors and the Hungarian / greedy backends are not reimplemented: they
are forwarded to ``torch.ops.assignment`` when the reference's extensions
are loaded in the process, and raise ``ValueError`` otherwise.
"""

from __future__ import annotations

import types
from enum import Enum
from typing import Literal, overload

import torch

__all__ = ["Backend", "resolve_backend", "solve"]


class Backend(str, Enum):
    AUTO = "auto"
    JONKER = "jonker"
    MUNKRES = "munkres"
    LAWLER = "lawler"
    GREEDY = "greedy"

    def __str__(self) -> str:
        return self.value


def _op(name: str):
    return getattr(torch.ops.assignment, name, None)


# Indirection so tests can substitute recording stubs (the reference's
# tests/test_match_dispatch.py:35-71 patch the same namespace).
_OPS = types.SimpleNamespace(
    jonker_dense_batch=torch.ops.assignment.jonker_dense_batch,
    jonker_scalar=_op("jonker_scalar"),
    jonker_dense=_op("jonker_dense"),
    jonker_compact=_op("jonker_compact"),
    jonker_compact_batch=torch.ops.assignment.jonker_compact_batch,
    jonker_dense_batch_unpacked=torch.ops.assignment.jonker_dense_batch_unpacked,
    jonker_compact_batch_unpacked=torch.ops.assignment.jonker_compact_batch_unpacked,
    munkres=_op("munkres"),
    lawler=_op("lawler"),
    greedy=_op("greedy"),
)

# Thresholds (reference _solve.py:62-64); the CUDA batch limit is the
# kernel's, not the reference's 64.
_JONKER_SCALAR_MAX_CELLS = 64
_CUDA_2D_LAWLER_N = 32
_CUDA_BATCH_MAX_K = 256


def _coerce_backend(value: Backend | str) -> Backend:
    try:
        return Backend(value)
    except ValueError as err:
        msg = (
            f"torchmatch.assignment.solve: unknown backend {value!r}; "
            f"valid values are {[b.value for b in Backend]}"
        )
        raise ValueError(msg) from err


def _require(name: str):
    op = getattr(_OPS, name)
    if op is None:
        msg = (
            f"torchmatch.assignment.solve: {name} is unavailable "
            "(the reference torchmatch extension providing it is not loaded)"
        )
        raise ValueError(msg)
    return op


def _pick_jonker_cpu_2d(n: int, m: int) -> str:
    if n * m <= _JONKER_SCALAR_MAX_CELLS:
        return "jonker_scalar"
    return "jonker_compact" if n == m else "jonker_dense"


def _pick_jonker_cpu_3d(n: int, m: int) -> str:
    return "jonker_compact_batch" if n == m else "jonker_dense_batch"


def _pick_auto_cuda_2d(n: int) -> str:
    return "munkres" if n < _CUDA_2D_LAWLER_N else "lawler"


def _cuda_batch_fits(n: int, m: int) -> bool:
    return max(n, m) <= _CUDA_BATCH_MAX_K


def _dense_batch(cost: torch.Tensor) -> torch.Tensor:
    return _OPS.jonker_dense_batch(cost)


def _dense_batch_result(cost: torch.Tensor, m: int, unpack: bool):
    """CUDA 3-D: packed op, or the native unpacked op when unpack=True."""
    if unpack and _ALLOW_NATIVE_UNPACK and _OPS.jonker_dense_batch_unpacked is not None:
        return _OPS.jonker_dense_batch_unpacked(cost)
    packed = _dense_batch(cost)
    return _unpack_packed(packed, m) if unpack else packed


def _dispatch_auto(cost: torch.Tensor, *, unpack: bool):
    is_cuda = cost.device.type == "cuda"
    if cost.ndim == 2:
        if is_cuda:
            name = _pick_auto_cuda_2d(cost.size(0))
            if getattr(_OPS, name) is not None:
                packed = _dispatch_primed(cost, name)
            elif _cuda_batch_fits(cost.size(0), cost.size(1)):
                packed = _dense_batch(cost.unsqueeze(0))[0]
            else:
                packed = _dispatch_primed(cost, name)
            return _unpack_packed(packed, cost.size(1)) if unpack else packed
        return _dispatch_jonker(cost, unpack=unpack)
    b, n, m = cost.shape
    if not is_cuda:
        return _dispatch_jonker(cost, unpack=unpack)
    if _cuda_batch_fits(n, m):
        return _dense_batch_result(cost, m, unpack)
    op = _require(_pick_auto_cuda_2d(n))
    packed = torch.stack([op(cost[i]) for i in range(b)], dim=0)
    return _unpack_packed(packed, m) if unpack else packed


def _dispatch_primed(cost: torch.Tensor, op_name: str) -> torch.Tensor:
    if cost.device.type != "cuda":
        msg = f"torchmatch.assignment.solve: {op_name} is CUDA-only"
        raise ValueError(msg)
    op = getattr(_OPS, op_name)
    if op is None:
        msg = (
            f"torchmatch.assignment.solve: {op_name} is unavailable "
            "(CUDA extension not loaded)"
        )
        raise ValueError(msg)
    if cost.ndim == 2:
        return op(cost)
    return torch.stack([op(cost[b]) for b in range(cost.size(0))], dim=0)


_ALLOW_NATIVE_UNPACK = True


def _unpack_packed_3d(packed: torch.Tensor, m: int):
    """Compacts a packed (B, N) row->col tensor into
    (matches (B, N, 2), unmatched_rows (B, N), unmatched_cols (B, M),
    n_matched (B,)); entries past each problem's count are unspecified
    (reference _solve.py:124-164)."""
    b, n = packed.shape
    dev = packed.device
    hit = packed >= 0
    n_matched = hit.sum(dim=-1)
    rows = torch.arange(n, device=dev).expand(b, n)
    # stable sort on the miss flag brings matched rows to the front in order
    by_hit = torch.argsort((~hit).to(torch.int8), dim=-1, stable=True)
    matches = torch.stack(
        [torch.gather(rows, 1, by_hit), torch.gather(packed, 1, by_hit)], dim=-1
    )
    by_miss = torch.argsort(hit.to(torch.int8), dim=-1, stable=True)
    unmatched_rows = torch.gather(rows, 1, by_miss)
    # unmatched rows scatter into a spare column m, so they can never clear
    # the mark a matched row set on the same column
    used = torch.zeros(b, m + 1, dtype=torch.bool, device=dev)
    used.scatter_(1, torch.where(hit, packed, m), hit)
    used = used[:, :m]
    by_free = torch.argsort(used.to(torch.int8), dim=-1, stable=True)
    unmatched_cols = torch.gather(torch.arange(m, device=dev).expand(b, m), 1, by_free)
    return matches, unmatched_rows, unmatched_cols, n_matched


def _unpack_packed(packed: torch.Tensor, m: int):
    if packed.ndim == 1:
        matches, ur, uc, nm = _unpack_packed_3d(packed.unsqueeze(0), m)
        k = int(nm.item())
        n = packed.size(0)
        return matches[0, :k], ur[0, : n - k], uc[0, : m - k]
    return _unpack_packed_3d(packed, m)


def _dispatch_jonker(cost: torch.Tensor, *, unpack: bool):
    if cost.device.type == "cuda":
        if cost.ndim == 2:
            n, m = cost.shape
            if not _cuda_batch_fits(n, m):
                msg = (
                    "torchmatch.assignment.solve: CUDA batched JV requires "
                    f"max(N, M) <= {_CUDA_BATCH_MAX_K}, got shape {tuple(cost.shape)}; "
                    "transfer to CPU"
                )
                raise ValueError(msg)
            packed = _dense_batch(cost.unsqueeze(0))[0]
            return _unpack_packed(packed, m) if unpack else packed
        _b, n, m = cost.shape
        if not _cuda_batch_fits(n, m):
            msg = (
                "torchmatch.assignment.solve: CUDA batched JV requires "
                f"K <= {_CUDA_BATCH_MAX_K}, got K={max(n, m)}; transfer to CPU"
            )
            raise ValueError(msg)
        return _dense_batch_result(cost, m, unpack)
    # CPU: the reference's own CPU ops, when its extension is loaded.
    if cost.ndim == 2:
        packed = _require(_pick_jonker_cpu_2d(cost.size(0), cost.size(1)))(cost)
        return _unpack_packed(packed, cost.size(1)) if unpack else packed
    name = _pick_jonker_cpu_3d(cost.size(1), cost.size(2))
    if unpack and _ALLOW_NATIVE_UNPACK and getattr(_OPS, f"{name}_unpacked") is not None:
        return getattr(_OPS, f"{name}_unpacked")(cost)
    if name == "jonker_compact_batch" and _OPS.jonker_compact_batch is None:
        name = "jonker_dense_batch"
    packed = _require(name)(cost)
    return _unpack_packed(packed, cost.size(2)) if unpack else packed


def _validate(cost: torch.Tensor) -> None:
    if cost.ndim not in (2, 3):
        msg = f"torchmatch.assignment.solve: cost.ndim must be 2 or 3, got {cost.ndim}"
        raise ValueError(msg)
    if cost.dtype not in (torch.float32, torch.float64):
        msg = (
            "torchmatch.assignment.solve: cost.dtype must be float32 or float64, "
            f"got {cost.dtype}"
        )
        raise ValueError(msg)
    if cost.device.type not in ("cpu", "cuda"):
        msg = (
            "torchmatch.assignment.solve: cost.device must be cpu or cuda, "
            f"got {cost.device}"
        )
        raise ValueError(msg)
    # The CUDA op checks NaN / -inf itself in its single statistics pass
    # (RuntimeError with "NaN" / "-inf"), so a CUDA input is not scanned
    # twice here; CPU inputs keep the reference's early check.
    if cost.device.type == "cpu":
        if torch.isnan(cost).any():
            msg = "torchmatch.assignment.solve: cost contains NaN"
            raise RuntimeError(msg)
        if (cost == float("-inf")).any():
            msg = "torchmatch.assignment.solve: cost contains -inf"
            raise RuntimeError(msg)


@overload
def solve(
    cost: torch.Tensor, *, backend: Backend | str = ..., unpack: Literal[False] = False
) -> torch.Tensor: ...


@overload
def solve(
    cost: torch.Tensor, *, backend: Backend | str = ..., unpack: Literal[True]
) -> tuple[torch.Tensor, ...]: ...


def solve(cost: torch.Tensor, *, backend: Backend | str = Backend.AUTO, unpack: bool = False):
    """Solve the linear assignment problem(s) in ``cost`` ((N, M) or (B, N, M)).

    Returns the int64 row->col mapping (``-1`` = unmatched row), or with
    ``unpack=True`` the compacted tuple of the reference's ``*_unpacked`` ops.
    """
    backend = _coerce_backend(backend)
    _validate(cost)
    if backend == Backend.AUTO:
        return _dispatch_auto(cost, unpack=unpack)
    if backend == Backend.JONKER:
        return _dispatch_jonker(cost, unpack=unpack)
    if backend in (Backend.MUNKRES, Backend.LAWLER):
        packed = _dispatch_primed(cost, backend.value)
        return _unpack_packed(packed, cost.size(-1)) if unpack else packed
    if backend == Backend.GREEDY:
        packed = _require("greedy")(cost)
        return _unpack_packed(packed, cost.size(-1)) if unpack else packed
    msg = f"torchmatch.assignment.solve: backend {backend!r} not dispatched"
    raise RuntimeError(msg)


def resolve_backend(cost: torch.Tensor, *, backend: Backend | str = Backend.AUTO) -> str:
    """Name of the ``torch.ops.assignment`` op ``solve()`` would call."""
    backend = _coerce_backend(backend)
    if backend != Backend.AUTO:
        return backend.value
    is_cuda = cost.device.type == "cuda"
    if cost.ndim == 2:
        if is_cuda:
            name = _pick_auto_cuda_2d(cost.size(0))
            if getattr(_OPS, name) is None and _cuda_batch_fits(cost.size(0), cost.size(1)):
                return "jonker_dense_batch"
            return name
        return _pick_jonker_cpu_2d(cost.size(0), cost.size(1))
    _b, n, m = cost.shape
    if not is_cuda:
        return _pick_jonker_cpu_3d(n, m)
    if _cuda_batch_fits(n, m):
        return "jonker_dense_batch"
    return _pick_auto_cuda_2d(n)
