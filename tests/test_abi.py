"""The C ABI library: loads without a GPU, exports what the header declares,
and its host-only logic (argument checks, sentinel) behaves like the
reference's compute_inf_sentinel (cuda/cuda_common.cuh:215-255)."""

from __future__ import annotations

import ctypes
import re
import struct
from pathlib import Path

import numpy as np
import pytest

ROOT = Path(__file__).resolve().parent.parent
HEADER = ROOT / "include" / "torchmatch_b200.h"


def _core():
    from torchmatch_b200 import _loader

    return _loader.core()


def test_library_exports_every_declared_symbol():
    from torchmatch_b200 import _loader

    declared = set(re.findall(r"^\s*(?:int|void|size_t|const char \*)\s*(tm_\w+)\(",
                              HEADER.read_text(), re.M))
    assert declared == set(_loader.EXPORTED)
    lib = ctypes.CDLL(str(_loader.CORE_LIB))
    for name in declared:
        assert hasattr(lib, name), name


def test_torch_library_registers_cuda_kernel():
    import torch
    import torchmatch_b200  # noqa: F401

    dump = torch._C._dispatch_dump("assignment::jonker_dense_batch")
    assert "jonker_dense_batch(Tensor costs) -> Tensor" in dump
    assert "CUDA: registered" in dump


def test_max_k_and_status_strings():
    lib = _core()
    assert lib.tm_jv_max_k() == 256
    assert b"NaN" in lib.tm_status_string(1)
    assert b"-inf" in lib.tm_status_string(2)


def _key(f: float) -> int:
    u = struct.unpack("<I", struct.pack("<f", f))[0]
    return (~u & 0xFFFFFFFF) if (u & 0x80000000) else (u | 0x80000000)


class Stats(ctypes.Structure):
    _fields_ = [("flags", ctypes.c_uint32), ("max_key", ctypes.c_uint32)]


@pytest.mark.parametrize("mx", [0.5, 9.99, -3.25, 0.0, 1e30, -1e-20])
@pytest.mark.parametrize("k", [1, 2, 64, 150, 256])
def test_sentinel_formula_matches_oracle(mx, k, oracle_mod):
    lib = _core()
    st = Stats(4, _key(mx))
    out = ctypes.c_float()
    pinf = ctypes.c_int(-1)
    rc = lib.tm_jv_sentinel(ctypes.byref(st), k, ctypes.byref(out), ctypes.byref(pinf))
    assert rc == 0 and pinf.value == 0
    expect = (np.float32(mx) + np.float32(1)) * np.float32(k + 1)
    assert np.float32(out.value) == expect


def test_sentinel_flags():
    lib = _core()
    out = ctypes.c_float()
    pinf = ctypes.c_int()
    assert lib.tm_jv_sentinel(ctypes.byref(Stats(1 | 4, _key(1.0))), 4, ctypes.byref(out), None) == 1
    assert lib.tm_jv_sentinel(ctypes.byref(Stats(2 | 8, 0)), 4, ctypes.byref(out), None) == 2
    assert lib.tm_jv_sentinel(ctypes.byref(Stats(8, 0)), 4, ctypes.byref(out), ctypes.byref(pinf)) == 0
    assert out.value == 1.0 and pinf.value == 1


def test_solve_argument_checks_need_no_gpu():
    lib = _core()
    assert lib.tm_jv_solve_f32(None, -1, 2, 2, 1.0, 0, None, None, None) == 3
    assert lib.tm_jv_solve_f32(None, 0, 2, 2, 1.0, 0, None, None, None) == 0
    assert lib.tm_jv_solve_f32(ctypes.c_void_p(16), 1, 2, 2, 1.0, 0, ctypes.c_void_p(16),
                               None, None) == 3  # no workspace
    assert lib.tm_jv_solve_f32(ctypes.c_void_p(16), 1, 257, 3, 1.0, 0, ctypes.c_void_p(16),
                               ctypes.c_void_p(64), None) == 5
    assert lib.tm_jv_workspace_bytes() == 64
    assert lib.tm_jonker_dense_batch_f32(None, 2, 3, 3, None, None, None) == 3


def test_points_workspace_sizing_needs_no_gpu():
    # TILE shapes need only the 256-byte header; streaming shapes take one
    # N*M slab (rounded to 64 floats) per resident warp, at most one per problem
    from torchmatch_b200 import _loader

    lib = _loader.core()
    assert lib.tm_jv_points_workspace_bytes(4096, 64, 64) == 256
    assert lib.tm_jv_points_workspace_bytes(64, 130, 97) == 256
    assert lib.tm_jv_points_workspace_bytes(1, 1, 256) == 256
    assert lib.tm_jv_points_workspace_bytes(10, 256, 256) == 256 + 10 * 65536 * 4
    slab = (200 * 150 + 63) // 64 * 64 * 4
    assert lib.tm_jv_points_workspace_bytes(64, 200, 150) == 256 + 64 * slab
    big = lib.tm_jv_points_workspace_bytes(65536, 256, 256) - 256
    assert big % (65536 * 4) == 0 and 0 < big // (65536 * 4) <= 148 * 16
    assert lib.tm_jv_points_workspace_bytes(0, 8, 8) == 256
    assert lib.tm_jv_points_workspace_bytes(4, 300, 8) == 256
