"""CUDA jonker_dense_batch vs the oracle and the reference's golden vectors.

Bar: bit-exact int64 mappings (index work).  Golden vectors come from the
reference's own CPU op; larger seeded batches are checked against the oracle
(oracle/jv_oracle.c, itself pinned to the reference by test_oracle.py); the
full-size configurations are checked through size-independent properties
(valid permutation / partial matching, forbidden edges never used, float64
totals equal to the oracle's on a strided sample)."""

from __future__ import annotations

import numpy as np
import pytest
import torch

from cases import CASES, config2, config3, config4, config5, config5_chunk

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def op():
    import torchmatch_b200  # noqa: F401

    assert torch.cuda.is_available()
    return torch.ops.assignment.jonker_dense_batch


def _run(op, x: torch.Tensor) -> np.ndarray:
    return op(x.cuda()).cpu().numpy()


@pytest.mark.parametrize("name", sorted(CASES))
def test_golden(name, op, golden):
    outs, _ = golden
    np.testing.assert_array_equal(_run(op, CASES[name]()), outs[name])


@pytest.mark.parametrize(
    "name,make",
    [
        ("config2_full", lambda: config2(4096)),
        ("config3_b2048", lambda: config3(2048)),
        ("config4_b2048", lambda: config4(2048)),
        ("config5_b512", lambda: config5_chunk(512, 5)),
        ("ties_k96", lambda: torch.randint(0, 6, (1024, 96, 96),
                                           generator=torch.Generator().manual_seed(3)).float()),
        ("gamma_rect", lambda: torch.distributions.Gamma(2.0, 2.0).sample((512, 70, 90))),
    ],
)
def test_matches_oracle(name, make, op, oracle_mod):
    x = make().contiguous()
    np.testing.assert_array_equal(_run(op, x), oracle_mod.jonker_dense_batch(x.numpy()))


def _check_matching(x: np.ndarray, out: np.ndarray):
    b, n, m = x.shape
    assert out.shape == (b, n)
    assert ((out >= -1) & (out < m)).all()
    for k in range(b):
        cols = out[k][out[k] >= 0]
        assert len(np.unique(cols)) == len(cols), "column used twice"
    if n <= m:
        assert (out >= 0).all()


@pytest.mark.parametrize("cfg", ["config2", "config3", "config4", "config5"])
def test_full_size_properties(cfg, op, oracle_mod):
    if cfg == "config5":
        x = config5(16384)  # a quarter of B=65536 keeps host RAM bounded
    else:
        x = {"config2": config2, "config3": config3, "config4": config4}[cfg]()
    out = _run(op, x)
    xn = x.numpy()
    _check_matching(xn, out)
    if cfg == "config4":
        b, n, _ = xn.shape
        used = np.take_along_axis(xn, np.maximum(out, 0)[..., None], 2)[..., 0]
        assert np.isfinite(used[out >= 0]).all(), "a forbidden (+inf) edge was used"
    # float64 totals of a strided sample equal the oracle's exactly
    idx = np.arange(0, xn.shape[0], max(1, xn.shape[0] // 256))
    ref = oracle_mod.jonker_dense_batch(xn[idx])
    got = out[idx]
    x64 = xn[idx].astype(np.float64)
    rows = np.arange(xn.shape[1])
    for k in range(len(idx)):
        hit_g, hit_r = got[k] >= 0, ref[k] >= 0
        tg = x64[k][rows[hit_g], got[k][hit_g]].sum()
        tr = x64[k][rows[hit_r], ref[k][hit_r]].sum()
        assert tg == tr
    np.testing.assert_array_equal(got, ref)


def test_float64_input_is_cast_to_float32(op, oracle_mod):
    x = torch.rand(64, 24, 24, dtype=torch.float64, generator=torch.Generator().manual_seed(1))
    ref = oracle_mod.jonker_dense_batch(x.float().numpy())
    np.testing.assert_array_equal(_run(op, x), ref)


def test_non_contiguous_input(op, oracle_mod):
    x = torch.rand(32, 40, 40, generator=torch.Generator().manual_seed(2))
    xt = x.cuda().transpose(1, 2)
    ref = oracle_mod.jonker_dense_batch(x.transpose(1, 2).contiguous().numpy())
    np.testing.assert_array_equal(op(xt).cpu().numpy(), ref)


def test_unaligned_storage_offset(op, oracle_mod):
    base = torch.rand(1 + 16 * 7 * 5, generator=torch.Generator().manual_seed(4))
    x = base.cuda()[1:].view(16, 7, 5)  # 4-byte aligned only
    ref = oracle_mod.jonker_dense_batch(base[1:].view(16, 7, 5).numpy())
    np.testing.assert_array_equal(op(x).cpu().numpy(), ref)


def test_known_answer_inf_mask(op):
    cost = torch.tensor([[[1.0, float("inf")], [float("inf"), 1.0]],
                         [[2.0, float("inf")], [float("inf"), 3.0]]], device="cuda")
    assert op(cost).cpu().tolist() == [[0, 1], [0, 1]]


def test_nan_rejected(op):
    cost = torch.tensor([[[1.0, 2.0], [3.0, 4.0]], [[1.0, float("nan")], [3.0, 4.0]]], device="cuda")
    with pytest.raises(RuntimeError, match="NaN"):
        op(cost)


def test_neg_inf_rejected(op):
    cost = torch.tensor([[[1.0, 2.0], [3.0, 4.0]], [[1.0, float("-inf")], [3.0, 4.0]]], device="cuda")
    with pytest.raises(RuntimeError, match="-inf"):
        op(cost)


@pytest.mark.parametrize("shape", [(0, 4, 4), (3, 0, 4), (3, 4, 0)])
def test_empty(op, shape):
    out = op(torch.zeros(shape, device="cuda"))
    assert out.shape == shape[:2] and out.dtype == torch.long and (out == -1).all()


def test_k_above_limit_raises(op):
    with pytest.raises(RuntimeError, match="256"):
        op(torch.zeros(1, 257, 257, device="cuda"))


def test_input_not_mutated(op):
    x = CASES["mixed_inf_rect"]().cuda()
    before = x.clone()
    op(x)
    assert torch.equal(x, before)


def test_runs_on_current_stream(op, oracle_mod):
    x = config2(64)
    s = torch.cuda.Stream()
    with torch.cuda.stream(s):
        out = op(x.cuda())
    s.synchronize()
    np.testing.assert_array_equal(out.cpu().numpy(), oracle_mod.jonker_dense_batch(x.numpy()))


def test_opcheck(op):
    x = torch.rand(4, 16, 16, device="cuda", generator=torch.Generator("cuda").manual_seed(0))
    torch.library.opcheck(op, (x,), test_utils=("test_schema", "test_faketensor"))


def test_torch_compile(oracle_mod):
    from torchmatch_b200.assignment import solve

    f = torch.compile(lambda c: solve(c, backend="jonker"), fullgraph=True)
    x = config2(32)
    np.testing.assert_array_equal(f(x.cuda()).cpu().numpy(), oracle_mod.jonker_dense_batch(x.numpy()))


def test_solve_routes_rectangular_cuda(oracle_mod):
    from torchmatch_b200.assignment import resolve_backend, solve

    x = CASES["rect100x150"]()
    assert resolve_backend(x.cuda()) == "jonker_dense_batch"
    np.testing.assert_array_equal(solve(x.cuda()).cpu().numpy(),
                                  oracle_mod.jonker_dense_batch(x.numpy()))
    m, ur, uc, nm = solve(x.cuda(), unpack=True)
    assert nm.tolist() == [100] * 4 and uc.shape == (4, 150)


def test_c_abi_direct(oracle_mod):
    """tm_jonker_dense_batch_f32 through ctypes, torch only for memory."""
    from torchmatch_b200 import _loader

    lib = _loader.core()
    x = CASES["config4_b256"]()
    xd = x.cuda()
    out = torch.empty(x.shape[0], x.shape[1], dtype=torch.long, device="cuda")
    ws = torch.empty(lib.tm_jv_workspace_bytes(), dtype=torch.uint8, device="cuda")
    stream = torch.cuda.current_stream().cuda_stream
    rc = lib.tm_jonker_dense_batch_f32(xd.data_ptr(), x.shape[0], x.shape[1], x.shape[2],
                                       out.data_ptr(), ws.data_ptr(), stream)
    assert rc == 0, lib.tm_status_string(rc)
    torch.cuda.synchronize()
    np.testing.assert_array_equal(out.cpu().numpy(), oracle_mod.jonker_dense_batch(x.numpy()))
    bad = xd.clone()
    bad[3, 4, 5] = float("nan")
    assert lib.tm_jonker_dense_batch_f32(bad.data_ptr(), x.shape[0], x.shape[1], x.shape[2],
                                         out.data_ptr(), ws.data_ptr(), stream) == 1


def test_stats_kernel(oracle_mod):
    from torchmatch_b200 import _loader

    lib = _loader.core()
    x = torch.randn(1000003, generator=torch.Generator().manual_seed(5)) * 100
    for special, flag in ((float("inf"), 8), (float("-inf"), 2), (float("nan"), 1)):
        y = x.clone()
        y[77777] = special
        st = torch.zeros(2, dtype=torch.int32, device="cuda")
        yd = y.cuda()
        assert lib.tm_jv_stats_f32(yd.data_ptr(), y.numel(), st.data_ptr(),
                                   torch.cuda.current_stream().cuda_stream) == 0
        flags, key = st.cpu().tolist()
        assert flags & flag and flags & 4
        u = key & 0xFFFFFFFF
        u = (u & 0x7FFFFFFF) if (u & 0x80000000) else (~u & 0xFFFFFFFF)
        mx = np.frombuffer(np.uint32(u).tobytes(), np.float32)[0]
        fin = y.numpy()[np.isfinite(y.numpy())]
        assert mx == fin.max()


def _unpack_like_reference(packed: np.ndarray, m: int):
    """cpu/ops.cpp:378-414 restated: pairs in row order, unmatched rows, unused
    columns in column order, -1 past every count."""
    b, n = packed.shape
    mt = np.full((b, n, 2), -1, np.int64)
    ur = np.full((b, n), -1, np.int64)
    uc = np.full((b, m), -1, np.int64)
    nm = np.zeros(b, np.int64)
    for k in range(b):
        rows = np.nonzero(packed[k] >= 0)[0]
        nm[k] = len(rows)
        mt[k, : len(rows), 0] = rows
        mt[k, : len(rows), 1] = packed[k, rows]
        miss = np.nonzero(packed[k] < 0)[0]
        ur[k, : len(miss)] = miss
        free = np.setdiff1d(np.arange(m), packed[k, rows])
        uc[k, : len(free)] = free
    return mt, ur, uc, nm


@pytest.mark.parametrize("name", ["config4_b256", "tall9x5", "wide5x9", "ties_small",
                                  "gated32", "rect250x6", "sq256", "inf_known_answer"])
def test_unpacked_matches_reference_layout(name, golden):
    outs, _ = golden
    x = CASES[name]()
    got = torch.ops.assignment.jonker_dense_batch_unpacked(x.cuda())
    want = _unpack_like_reference(outs[name], x.shape[2])
    for g, w in zip(got, want):
        np.testing.assert_array_equal(g.cpu().numpy(), w)


def test_unpacked_empty_and_errors():
    op = torch.ops.assignment.jonker_dense_batch_unpacked
    m, ur, uc, nm = op(torch.zeros(3, 0, 4, device="cuda"))
    assert m.shape == (3, 0, 2) and uc.shape == (3, 4) and nm.tolist() == [0, 0, 0]
    bad = torch.ones(2, 3, 3, device="cuda")
    bad[1, 2, 0] = float("nan")
    with pytest.raises(RuntimeError, match="NaN"):
        op(bad)


def test_unpacked_opcheck_and_solve_route():
    from torchmatch_b200.assignment import solve

    x = torch.rand(4, 12, 17, device="cuda", generator=torch.Generator("cuda").manual_seed(1))
    torch.library.opcheck(torch.ops.assignment.jonker_dense_batch_unpacked, (x,),
                          test_utils=("test_schema", "test_faketensor"))
    native = solve(x, unpack=True)
    packed = solve(x).cpu().numpy()
    for g, w in zip(native, _unpack_like_reference(packed, 17)):
        np.testing.assert_array_equal(g.cpu().numpy(), w)


@pytest.mark.parametrize("name", sorted(CASES))
def test_compact_golden(name, golden):
    outs, _ = golden
    got = torch.ops.assignment.jonker_compact_batch(CASES[name]().cuda()).cpu().numpy()
    np.testing.assert_array_equal(got, outs["compact__" + name])


@pytest.mark.parametrize("make", [lambda: config2(2048), lambda: config3(1024),
                                  lambda: config4(1024), lambda: config5_chunk(256, 7)])
def test_compact_matches_oracle(make, oracle_mod):
    x = make().contiguous()
    got = torch.ops.assignment.jonker_compact_batch(x.cuda()).cpu().numpy()
    np.testing.assert_array_equal(got, oracle_mod.jonker_compact_batch(x.numpy()))


def test_compact_unpacked_layout(golden):
    outs, _ = golden
    x = CASES["config4_b256"]()
    got = torch.ops.assignment.jonker_compact_batch_unpacked(x.cuda())
    want = _unpack_like_reference(outs["compact__config4_b256"], x.shape[2])
    for g, w in zip(got, want):
        np.testing.assert_array_equal(g.cpu().numpy(), w)
