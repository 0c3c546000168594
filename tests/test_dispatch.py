"""Routing of ``torchmatch_b200.assignment.solve`` (reference
tests/test_match_dispatch.py, with the CUDA thresholds this package lifts).

CUDA routing is exercised without a GPU through a stand-in tensor that only
reports device/shape, and the recording stubs the reference tests use."""

from __future__ import annotations

import pytest
import torch

import torchmatch_b200  # noqa: F401
from torchmatch_b200.assignment import Backend, _solve, resolve_backend, solve


class FakeCuda:
    """Shape/device stand-in for a CUDA tensor (no GPU needed)."""

    def __init__(self, *shape):
        self.shape = torch.Size(shape)
        self.ndim = len(shape)
        self.dtype = torch.float32
        self.device = torch.device("cuda", 0)

    def size(self, i=None):
        return self.shape if i is None else self.shape[i]

    def unsqueeze(self, d):
        assert d == 0
        return FakeCuda(1, *self.shape)

    def __getitem__(self, i):
        return FakeCuda(*self.shape[1:])


@pytest.fixture
def record_ops(monkeypatch):
    calls = []

    def stub(name):
        def f(cost):
            calls.append((name, tuple(cost.shape)))
            b = cost.shape[:-1]
            return torch.zeros(*b, dtype=torch.long)

        return f

    for name in vars(_solve._OPS):
        monkeypatch.setattr(_solve._OPS, name, stub(name))
    return calls


@pytest.mark.parametrize("shape", [(2, 8, 8), (3, 64, 64), (2, 8, 12), (4, 100, 150),
                                   (2, 128, 128), (1, 256, 256), (2, 256, 3)])
def test_auto_cuda_3d_uses_dense_batch(record_ops, shape):
    solve(FakeCuda(*shape))
    assert record_ops == [("jonker_dense_batch", shape)]
    assert resolve_backend(FakeCuda(*shape)) == "jonker_dense_batch"


@pytest.mark.parametrize("shape", [(2, 8, 8), (2, 8, 12), (2, 200, 100)])
def test_jonker_cuda_3d_uses_dense_batch(record_ops, shape):
    solve(FakeCuda(*shape), backend="jonker")
    assert record_ops == [("jonker_dense_batch", shape)]


def test_jonker_cuda_too_large_errors(record_ops):
    with pytest.raises(ValueError, match="K <= 256"):
        solve(FakeCuda(2, 257, 257), backend="jonker")


def test_jonker_cuda_2d_is_a_batch_of_one(record_ops):
    solve(FakeCuda(8, 8), backend="jonker")
    assert record_ops == [("jonker_dense_batch", (1, 8, 8))]


def test_auto_cuda_3d_too_large_loops_2d_op(record_ops):
    solve(FakeCuda(3, 300, 300))
    assert [c[0] for c in record_ops] == ["lawler"] * 3


def test_auto_cuda_2d_prefers_hungarian_when_loaded(record_ops):
    solve(FakeCuda(8, 8))
    assert record_ops[-1][0] == "munkres"
    solve(FakeCuda(128, 128))
    assert record_ops[-1][0] == "lawler"


def test_auto_cuda_2d_without_hungarian_uses_dense_batch(record_ops, monkeypatch):
    monkeypatch.setattr(_solve._OPS, "munkres", None)
    solve(FakeCuda(8, 8))
    assert record_ops[-1] == ("jonker_dense_batch", (1, 8, 8))
    assert resolve_backend(FakeCuda(8, 8)) == "jonker_dense_batch"


def test_unknown_backend():
    with pytest.raises(ValueError, match="unknown backend"):
        solve(torch.zeros(2, 2), backend="nope")
    assert Backend("jonker") is Backend.JONKER
    assert resolve_backend(torch.zeros(2, 2), backend="munkres") == "munkres"


def test_validation_errors():
    with pytest.raises(ValueError, match="ndim"):
        solve(torch.zeros(2))
    with pytest.raises(ValueError, match="dtype"):
        solve(torch.zeros(2, 2, dtype=torch.int64))
    with pytest.raises(RuntimeError, match="NaN"):
        solve(torch.tensor([[1.0, float("nan")], [0.0, 1.0]]))
    with pytest.raises(RuntimeError, match="-inf"):
        solve(torch.tensor([[1.0, float("-inf")], [0.0, 1.0]]))


def test_cpu_without_reference_extension_raises(monkeypatch):
    for name in ("jonker_compact_batch", "jonker_compact_batch_unpacked",
                 "jonker_dense_batch_unpacked"):
        monkeypatch.setattr(_solve._OPS, name, None)
    # the op exists, but only a CUDA kernel is registered in this package
    if "CPU: registered" in torch._C._dispatch_dump("assignment::jonker_dense_batch"):
        pytest.skip("the reference CPU extension is loaded in this process")
    with pytest.raises((RuntimeError, NotImplementedError)):
        solve(torch.zeros(2, 3, 3))


def test_unpack_packed_3d_layout():
    packed = torch.tensor([[2, -1, 0], [1, 0, -1]])
    matches, ur, uc, nm = _solve._unpack_packed_3d(packed, 4)
    assert nm.tolist() == [2, 2]
    assert matches[0, :2].tolist() == [[0, 2], [2, 0]]
    assert matches[1, :2].tolist() == [[0, 1], [1, 0]]
    assert ur[0, :1].tolist() == [1] and ur[1, :1].tolist() == [2]
    assert uc[0, :2].tolist() == [1, 3] and uc[1, :2].tolist() == [2, 3]


def test_unpack_packed_2d():
    m, ur, uc = _solve._unpack_packed(torch.tensor([1, -1]), 3)
    assert m.tolist() == [[0, 1]] and ur.tolist() == [1] and uc.tolist() == [0, 2]


def test_assignment_cost():
    from torchmatch_b200.assignment import assignment_cost

    c = torch.tensor([[[1.0, 2.0], [3.0, 4.0]]], dtype=torch.float64)
    m = torch.tensor([[1, -1]])
    assert assignment_cost(c, m).tolist() == [2.0]
    assert assignment_cost(c, m, reduction="mean").tolist() == [2.0]
    assert assignment_cost(c, m, reduction="none").tolist() == [[2.0, 0.0]]
    assert float(assignment_cost(c[0], m[0])) == 2.0


def test_fake_kernel_shape():
    from torch._subclasses.fake_tensor import FakeTensorMode

    with FakeTensorMode():
        out = torch.ops.assignment.jonker_dense_batch(torch.empty(3, 5, 7))
    assert out.shape == (3, 5) and out.dtype == torch.long


def test_cuda_unpack_uses_native_unpacked_op(record_ops):
    solve(FakeCuda(2, 8, 12), unpack=True)
    assert record_ops == [("jonker_dense_batch_unpacked", (2, 8, 12))]
