"""TEST INFRASTRUCTURE ONLY: ctypes bindings of the CPU oracle.

``jonker_dense_batch`` runs ``jv_oracle.c`` (this repository's C restatement of
the reference's CPU path, cpu/ops.cpp:176-289 + cpu/jonker_dense_flat.h).
``reference_jonker_dense_batch`` runs the reference's own solver core compiled
from its sources into ``oracle/_ref/`` (absent where the reference tree was
never available to build it).  Only tests, ``__graft_entry__.smoke()`` and
bench.py's CPU-baseline leg import this module.
"""

from __future__ import annotations

import ctypes
import os
import subprocess
from pathlib import Path

import numpy as np

HERE = Path(__file__).resolve().parent
LIB = HERE / "libtmoracle.so"
REF_LIB = HERE / "_ref" / "libtmref.so"

_ERRORS = {
    1: "jonker: cost matrix contains NaN. Use +inf for forbidden pairs",
    2: "jonker: cost matrix contains -inf. Use +inf for forbidden pairs",
    3: "jonker oracle: allocation failure",
}


def build() -> None:
    """Compile the oracle (and oracle/_ref where the reference tree exists)."""
    subprocess.run(["make", "-s", "-C", str(HERE)], check=True)


def _load(path: Path, symbol: str):
    if not path.exists():
        raise FileNotFoundError(f"{path} is not built (run make -C {HERE})")
    lib = ctypes.CDLL(str(path))
    fn = getattr(lib, symbol)
    fn.restype = ctypes.c_int
    fn.argtypes = [
        ctypes.c_void_p,
        ctypes.c_int64,
        ctypes.c_int,
        ctypes.c_int,
        ctypes.c_void_p,
        ctypes.c_int,
    ]
    return fn


_fns: dict[str, object] = {}


def _call(path: Path, symbol: str, costs, threads: int) -> np.ndarray:
    key = f"{path}:{symbol}"
    if key not in _fns:
        _fns[key] = _load(path, symbol)
    fn = _fns[key]
    a = np.ascontiguousarray(np.asarray(costs, dtype=np.float32))
    if a.ndim != 3:
        raise ValueError("costs must be 3D (B, N, M)")
    b, n, m = a.shape
    out = np.full((b, n), -1, dtype=np.int64)
    rc = fn(a.ctypes.data, b, n, m, out.ctypes.data, int(threads))
    if rc != 0:
        raise RuntimeError(_ERRORS.get(rc, f"oracle failed with code {rc}"))
    return out


def jonker_dense_batch(costs, threads: int = 0) -> np.ndarray:
    """Oracle restatement: (B, N, M) float32 -> (B, N) int64, -1 = unmatched."""
    return _call(LIB, "tmo_jonker_dense_batch_f32", costs, threads)


def jonker_compact_batch(costs, threads: int = 0) -> np.ndarray:
    """Oracle restatement of jonker_compact_batch (cpu/jonker_compact_core.h)."""
    return _call(LIB, "tmo_jonker_compact_batch_f32", costs, threads)


def reference_jonker_compact_batch(costs, threads: int = 0) -> np.ndarray:
    """The reference's compact solver behind the same batch driver."""
    return _call(REF_LIB, "tmref_jonker_compact_batch_f32", costs, threads)


def reference_available() -> bool:
    return REF_LIB.exists()


def reference_jonker_dense_batch(costs, threads: int = 0) -> np.ndarray:
    """The reference's compiled solver core behind the same batch driver."""
    return _call(REF_LIB, "tmref_jonker_dense_batch_f32", costs, threads)


def host_threads() -> int:
    return len(os.sched_getaffinity(0))


def sqeuclidean_costs(x, y) -> np.ndarray:
    """Squared-Euclidean (B, N, M) fp32 costs of x (B, N, D) and y (B, M, D),
    summed over d in order with every operation rounded (jv_oracle.c)."""
    key = f"{LIB}:tmo_sqeuclidean_costs_f32"
    if key not in _fns:
        lib = ctypes.CDLL(str(LIB))
        fn = lib.tmo_sqeuclidean_costs_f32
        fn.restype = None
        fn.argtypes = [ctypes.c_void_p, ctypes.c_void_p, ctypes.c_int64, ctypes.c_int,
                       ctypes.c_int, ctypes.c_int, ctypes.c_void_p]
        _fns[key] = fn
    xa = np.ascontiguousarray(np.asarray(x, dtype=np.float32))
    ya = np.ascontiguousarray(np.asarray(y, dtype=np.float32))
    if xa.ndim != 3 or ya.ndim != 3 or xa.shape[0] != ya.shape[0] or xa.shape[2] != ya.shape[2]:
        raise ValueError("x must be (B, N, D) and y (B, M, D)")
    b, n, d = xa.shape
    m = ya.shape[1]
    out = np.empty((b, n, m), dtype=np.float32)
    _fns[key](xa.ctypes.data, ya.ctypes.data, b, n, m, d, out.ctypes.data)
    return out


def jonker_sqeuclidean_batch(x, y, threads: int = 0) -> np.ndarray:
    """Oracle of the fused op: the restated producer, then jonker_dense_batch."""
    return jonker_dense_batch(sqeuclidean_costs(x, y), threads)


REF_CUDA_LIB = HERE / "_ref" / "libtmref_cuda.so"


def reference_cuda_available() -> bool:
    return REF_CUDA_LIB.exists()


def reference_cuda_jonker_dense_batch(costs):
    """The reference's own batched CUDA kernel (cuda/jonker_tiled.cuh, built
    from its sources for sm_100a) on a contiguous finite (B, K, K) float32
    CUDA tensor, K <= 64, on the current stream.  Kernel only: the reference
    op first scans for NaN / +-inf and rewrites +inf (absent here)."""
    import torch

    key = f"{REF_CUDA_LIB}:tmref_cuda_jonker_dense_batch"
    if key not in _fns:
        lib = ctypes.CDLL(str(REF_CUDA_LIB))
        fn = lib.tmref_cuda_jonker_dense_batch
        fn.restype = ctypes.c_int
        fn.argtypes = [ctypes.c_void_p, ctypes.c_int, ctypes.c_int, ctypes.c_void_p,
                       ctypes.c_void_p]
        _fns[key] = fn
    b, k, k2 = costs.shape
    if k != k2 or costs.dtype != torch.float32 or not costs.is_contiguous():
        raise ValueError("costs must be a contiguous float32 (B, K, K) CUDA tensor")
    out = torch.empty(b, k, dtype=torch.int64, device=costs.device)
    rc = _fns[key](costs.data_ptr(), b, k, out.data_ptr(), torch.cuda.current_stream().cuda_stream)
    if rc != 0:
        raise RuntimeError(f"reference CUDA kernel failed with code {rc}")
    return out
