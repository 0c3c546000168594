"""Loads the native libraries and wires ``torch.ops.assignment.jonker_dense_batch``.

Mirrors the role of the reference loaders (tue-p8n/torchmatch 1.0.3,
sources/torchmatch/assignment/_loader.py:111-169, _cpu.py:58-74,
_cuda.py:54-73) for the one operator this package provides:

* the schema ``assignment::jonker_dense_batch(Tensor costs) -> Tensor`` is
  defined here unless the reference's CPU extension already defined it
  (cpu/ops.cpp:486-496 owns it when both are loaded; load it first);
* the fake kernel ``(B, N, M) -> (B, N) int64`` (_loader.py:160-169) is
  registered unless one exists;
* ``lib/libtmjv_torch.so`` registers the CUDA kernel.

There is no fallback: if the library is missing or fails to load, importing
raises, so a GPU run can never silently take another path.
"""

from __future__ import annotations

import ctypes
import functools
from pathlib import Path

import torch

PKG = Path(__file__).resolve().parent
LIBDIR = PKG / "lib"
CORE_LIB = LIBDIR / "libtmjv.so"
TORCH_LIB = LIBDIR / "libtmjv_torch.so"

OP = "assignment::jonker_dense_batch"
SCHEMA = "(Tensor costs) -> Tensor"
OP_ASYNC = "assignment::jonker_dense_batch_async"
SCHEMA_ASYNC = "(Tensor costs) -> (Tensor, Tensor)"
OP_UNPACKED = "assignment::jonker_dense_batch_unpacked"
OP_COMPACT = "assignment::jonker_compact_batch"
OP_COMPACT_UNPACKED = "assignment::jonker_compact_batch_unpacked"
SCHEMA_UNPACKED = "(Tensor costs) -> (Tensor, Tensor, Tensor, Tensor)"

# fused squared-Euclidean costs; no counterpart op in the reference
OP_POINTS = "assignment::jonker_sqeuclidean_batch"
SCHEMA_POINTS = "(Tensor x, Tensor y) -> Tensor"

_LIB_HANDLES: list[object] = []


def _has_op(name: str = OP) -> bool:
    try:
        torch._C._dispatch_find_schema_or_throw(name, "")
        return True
    except RuntimeError:
        return False


def _fake(costs: torch.Tensor) -> torch.Tensor:
    torch._check(costs.dim() == 3, lambda: "costs must be 3D (B, N, M)")
    return costs.new_empty(costs.size(0), costs.size(1), dtype=torch.long)


def _fake_unpacked(costs: torch.Tensor):
    torch._check(costs.dim() == 3, lambda: "costs must be 3D (B, N, M)")
    b, n, m = costs.size(0), costs.size(1), costs.size(2)
    return (
        costs.new_empty(b, n, 2, dtype=torch.long),
        costs.new_empty(b, n, dtype=torch.long),
        costs.new_empty(b, m, dtype=torch.long),
        costs.new_empty(b, dtype=torch.long),
    )


def _fake_points(x: torch.Tensor, y: torch.Tensor) -> torch.Tensor:
    torch._check(x.dim() == 3 and y.dim() == 3, lambda: "x must be (B, N, D) and y (B, M, D)")
    return x.new_empty(x.size(0), x.size(1), dtype=torch.long)


def _fake_async(costs: torch.Tensor):
    torch._check(costs.dim() == 3, lambda: "costs must be 3D (B, N, M)")
    return (costs.new_empty(costs.size(0), costs.size(1), dtype=torch.long),
            costs.new_empty(1, dtype=torch.int32))


@functools.cache
def load() -> None:
    """Define the op (if needed), register its fake and load the CUDA impl."""
    if not TORCH_LIB.exists():
        raise ImportError(
            f"{TORCH_LIB} is not built; run `python torchmatch_b200/_build.py`"
        )
    for name, schema, fake in ((OP, SCHEMA, _fake), (OP_UNPACKED, SCHEMA_UNPACKED, _fake_unpacked),
                               (OP_ASYNC, SCHEMA_ASYNC, _fake_async),
                               (OP_COMPACT, SCHEMA, _fake),
                               (OP_COMPACT_UNPACKED, SCHEMA_UNPACKED, _fake_unpacked),
                               (OP_POINTS, SCHEMA_POINTS, _fake_points)):
        if not _has_op(name):
            lib = torch.library.Library("assignment", "FRAGMENT")
            lib.define(name.split("::")[1] + schema)
            _LIB_HANDLES.append(lib)
        try:
            torch.library.register_fake(name)(fake)
        except RuntimeError:
            pass  # the reference's loader registered the same fake already
    torch.ops.load_library(str(TORCH_LIB))


@functools.cache
def core() -> ctypes.CDLL:
    """The plain C ABI (include/torchmatch_b200.h) through ctypes."""
    lib = ctypes.CDLL(str(CORE_LIB))
    i64, i32, vp = ctypes.c_int64, ctypes.c_int, ctypes.c_void_p
    lib.tm_jv_max_k.restype = i32
    lib.tm_jv_stats_f32.argtypes = [vp, i64, vp, vp]
    lib.tm_jv_sentinel.argtypes = [vp, i32, vp, vp]
    lib.tm_jv_solve_f32.argtypes = [vp, i64, i32, i32, ctypes.c_float, i32, vp, vp, vp]
    lib.tm_jv_solve_checked_f32.argtypes = [vp, i64, i32, i32, vp, vp, vp]
    lib.tm_jv_solve_checked_f32.restype = i32
    lib.tm_jv_workspace_bytes.restype = ctypes.c_size_t
    lib.tm_jonker_dense_batch_f32.argtypes = [vp, i64, i32, i32, vp, vp, vp]
    lib.tm_jonker_dense_batch_f32_noalloc.argtypes = [vp, i64, i32, i32, vp, vp]
    lib.tm_jonker_dense_batch_f32_noalloc.restype = i32
    lib.tm_jonker_dense_batch_unpacked_f32.argtypes = [vp, i64, i32, i32, vp, vp, vp]
    lib.tm_jonker_dense_batch_unpacked_f32.restype = i32
    lib.tm_jonker_dense_batch_async_f32.argtypes = [vp, i64, i32, i32, vp, vp, vp]
    lib.tm_jonker_dense_batch_async_f32.restype = i32
    lib.tm_jonker_compact_batch_f32.argtypes = [vp, i64, i32, i32, vp, vp, vp]
    lib.tm_jonker_compact_batch_f32.restype = i32
    lib.tm_jonker_compact_batch_unpacked_f32.argtypes = [vp, i64, i32, i32, vp, vp, vp]
    lib.tm_jonker_compact_batch_unpacked_f32.restype = i32
    lib.tm_jv_points_workspace_bytes.argtypes = [i64, i32, i32]
    lib.tm_jv_points_workspace_bytes.restype = ctypes.c_size_t
    lib.tm_jonker_sqeuclidean_batch_f32.argtypes = [vp, vp, i64, i32, i32, i32, vp, vp,
                                                   ctypes.c_size_t, vp]
    lib.tm_jonker_sqeuclidean_batch_f32.restype = i32
    lib.tm_jv_points_solve_f32.argtypes = [vp, vp, i64, i32, i32, i32, ctypes.c_float, i32, i32,
                                          vp, vp, ctypes.c_size_t, vp]
    lib.tm_jv_points_solve_f32.restype = i32
    lib.tm_jv_debug_set_loop_bound.argtypes = [i32]
    lib.tm_jv_debug_set_loop_bound.restype = None
    lib.tm_jv_debug_set_wait_limit.argtypes = [i32]
    lib.tm_jv_debug_set_wait_limit.restype = None
    lib.tm_status_string.restype = ctypes.c_char_p
    lib.tm_status_string.argtypes = [i32]
    for name in ("tm_jv_stats_f32", "tm_jv_sentinel", "tm_jv_solve_f32",
                 "tm_jonker_dense_batch_f32", "tm_last_cuda_error"):
        getattr(lib, name).restype = i32
    return lib


# Every symbol include/torchmatch_b200.h declares.
EXPORTED = (
    "tm_jv_max_k",
    "tm_jv_stats_f32",
    "tm_jv_sentinel",
    "tm_jv_solve_f32",
    "tm_jv_solve_checked_f32",
    "tm_jv_workspace_bytes",
    "tm_jonker_dense_batch_f32",
    "tm_jonker_dense_batch_f32_noalloc",
    "tm_jonker_dense_batch_unpacked_f32",
    "tm_jonker_dense_batch_async_f32",
    "tm_jonker_compact_batch_f32",
    "tm_jonker_compact_batch_unpacked_f32",
    "tm_jv_points_workspace_bytes",
    "tm_jonker_sqeuclidean_batch_f32",
    "tm_jv_points_solve_f32",
    "tm_last_cuda_error",
    "tm_jv_debug_set_loop_bound",
    "tm_jv_debug_set_wait_limit",
    "tm_status_string",
)
