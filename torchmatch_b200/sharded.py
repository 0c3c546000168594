"""Batch sharding across GPUs for jonker_dense_batch.

The B problems of one batch are independent; the only quantity coupling
them is the batch-global +inf sentinel (max_finite + 1) * (K + 1)
(reference cpu/ops.cpp:67-93, cuda/cuda_common.cuh:215-255).  Two ways to
spread one batch over several GPUs:

* ``solve_sharded(local, group)`` -- one process per GPU (torchrun).  Each
  rank holds a contiguous slice of the batch; the per-slice statistics are
  combined with one all-reduce (MAX over five int64 words: the NaN / -inf /
  finite / +inf flags and the order-preserving key of the largest finite
  cell), after which every rank solves its slice locally.  No other data
  crosses between GPUs.
* ``solve_multi_gpu(costs, devices)`` -- one process driving several GPUs:
  contiguous slices are peer-copied (NVLink) from the caller's device to
  each GPU on that GPU's own stream, solved there, and the int64 results are
  copied back into one output on the caller's device.

Both produce exactly what ``torch.ops.assignment.jonker_dense_batch`` gives
on the whole batch.  ``solve_points_sharded`` is the one-process-per-GPU
form of the fused squared-Euclidean op (point sets in, no cost tensor).
"""

from __future__ import annotations

import ctypes
import struct

import torch

from torchmatch_b200 import _loader

_NAN, _NEG_INF, _FINITE, _POS_INF = 1, 2, 4, 8


class _Stats(ctypes.Structure):
    _fields_ = [("flags", ctypes.c_uint32), ("max_key", ctypes.c_uint32)]


def stats_words(flags: int, key: int) -> list[int]:
    """Device statistics -> the five words that are all-reduced with MAX."""
    return [
        int(bool(flags & _NAN)),
        int(bool(flags & _NEG_INF)),
        int(bool(flags & _FINITE)),
        int(bool(flags & _POS_INF)),
        int(key),
    ]


def sentinel_from_words(words: list[int], k: int) -> tuple[float, bool]:
    """Merged words -> (sentinel, has_pos_inf); raises like the reference
    (cuda/cuda_common.cuh:245-249) on NaN / -inf."""
    lib = _loader.core()
    flags = (_NAN if words[0] else 0) | (_NEG_INF if words[1] else 0)
    flags |= (_FINITE if words[2] else 0) | (_POS_INF if words[3] else 0)
    st = _Stats(flags, words[4] & 0xFFFFFFFF)
    out = ctypes.c_float()
    pinf = ctypes.c_int()
    rc = lib.tm_jv_sentinel(ctypes.byref(st), k, ctypes.byref(out), ctypes.byref(pinf))
    if rc != 0:
        raise RuntimeError("jonker_dense_batch: " + lib.tm_status_string(rc).decode())
    return out.value, bool(pinf.value)


def order_key(x: float) -> int:
    """Host copy of the kernel's order-preserving float -> uint32 key."""
    u = struct.unpack("<I", struct.pack("<f", x))[0]
    return (~u & 0xFFFFFFFF) if (u & 0x80000000) else (u | 0x80000000)


def _stream(dev: torch.device) -> int:
    return torch.cuda.current_stream(dev).cuda_stream


def _local_stats(c: torch.Tensor) -> list[int]:
    lib = _loader.core()
    st = torch.empty(lib.tm_jv_workspace_bytes() // 4, dtype=torch.int32, device=c.device)
    rc = lib.tm_jv_stats_f32(c.data_ptr(), c.numel(), st.data_ptr(), _stream(c.device))
    if rc != 0:
        raise RuntimeError("jonker_dense_batch statistics: " + lib.tm_status_string(rc).decode())
    flags, key = (int(v) & 0xFFFFFFFF for v in st[:2].cpu().tolist())
    return stats_words(flags, key)


def _solve_local(c: torch.Tensor, sentinel: float, pinf: bool) -> torch.Tensor:
    lib = _loader.core()
    b, n, m = c.shape
    out = torch.empty(b, n, dtype=torch.long, device=c.device)
    if b == 0 or n == 0:
        return out
    ws = torch.empty(lib.tm_jv_workspace_bytes(), dtype=torch.uint8, device=c.device)
    rc = lib.tm_jv_solve_f32(c.data_ptr(), b, n, m, sentinel, int(pinf), out.data_ptr(),
                             ws.data_ptr(), _stream(c.device))
    if rc != 0:
        raise RuntimeError("batched JV kernel launch failed: " + lib.tm_status_string(rc).decode())
    return out


def merge_words(words: list[int], group=None, device=None) -> list[int]:
    """The one exchange of a sharded solve: element-wise MAX of every rank's
    five statistics words (flags are 0/1, the key is order-preserving, so
    MAX is OR of the flags and max of the largest finite cell)."""
    import torch.distributed as dist

    dev = device if dist.get_backend(group) == "nccl" else torch.device("cpu")
    t = torch.tensor(words, dtype=torch.int64, device=dev)
    dist.all_reduce(t, op=dist.ReduceOp.MAX, group=group)
    return t.cpu().tolist()


def _device_words(st: torch.Tensor) -> torch.Tensor:
    """tm_jv_stats (first two int32 of a workspace) -> the five int64 words."""
    raw = st[:2].to(torch.int64) & 0xFFFFFFFF
    t = torch.empty(5, dtype=torch.int64, device=st.device)
    # flag bits 1, 2, 4, 8 (NaN, -inf, finite, +inf) -> words 0..3
    t[:4] = (raw[0] >> torch.arange(4, device=st.device)) & 1
    t[4] = raw[1]
    return t


def solve_sharded(local: torch.Tensor, group=None) -> torch.Tensor:
    """Solve this rank's contiguous slice (B_r, N, M) of one global batch.

    Collective over ``group`` (every rank calls it with the same N, M).  The
    slice is solved in check mode, which also yields its statistics; one
    all-reduce merges them, the host raises on NaN / -inf anywhere, and only
    if some slice holds +inf is the slice solved again with the global
    sentinel.  Returns the (B_r, N) int64 mapping of the local slice.
    """
    import torch.distributed as dist

    if local.dim() != 3:
        raise RuntimeError("costs must be 3D (B, N, M)")
    c = local.to(torch.float32).contiguous()
    b, n, m = c.shape
    k = max(n, m)
    lib = _loader.core()
    if k > lib.tm_jv_max_k():
        raise RuntimeError(f"Batched JV (CUDA) supports max(N, M) <= 256, got K={k}")
    ws = torch.zeros(lib.tm_jv_workspace_bytes() // 4, dtype=torch.int32, device=c.device)
    out = torch.full((b, n), -1, dtype=torch.long, device=c.device)
    if b and n and m:
        rc = lib.tm_jv_solve_checked_f32(c.data_ptr(), b, n, m, out.data_ptr(), ws.data_ptr(),
                                         _stream(c.device))
        if rc != 0:
            raise RuntimeError("batched JV kernel launch failed: "
                               + lib.tm_status_string(rc).decode())
    if dist.get_backend(group) == "nccl":
        t = _device_words(ws)
        dist.all_reduce(t, op=dist.ReduceOp.MAX, group=group)
        words = t.cpu().tolist()
    else:
        flags, key = (int(v) & 0xFFFFFFFF for v in ws[:2].cpu().tolist())
        words = merge_words(stats_words(flags, key), group)
    sentinel, pinf = sentinel_from_words(words, k)
    if pinf and b and n and m:
        rc = lib.tm_jv_solve_f32(c.data_ptr(), b, n, m, sentinel, 1, out.data_ptr(),
                                 ws.data_ptr(), _stream(c.device))
        if rc != 0:
            raise RuntimeError("batched JV kernel launch failed: "
                               + lib.tm_status_string(rc).decode())
    return out


def solve_points_sharded(x_local: torch.Tensor, y_local: torch.Tensor, group=None) -> torch.Tensor:
    """``solve_sharded`` for the fused squared-Euclidean op: this rank's
    contiguous slices x (B_r, N, D) and y (B_r, M, D) of one global batch of
    point sets.  The costs are built inside the solve kernel on every rank
    (tm_jv_points_solve_f32); the statistics of the computed cells are merged
    with one all-reduce, exactly as for a cost batch, so the result equals
    ``torch.ops.assignment.jonker_sqeuclidean_batch`` on the whole batch.
    Collective over ``group``."""
    import torch.distributed as dist

    if x_local.dim() != 3 or y_local.dim() != 3 or x_local.shape[0] != y_local.shape[0] \
            or x_local.shape[2] != y_local.shape[2]:
        raise RuntimeError("x must be (B, N, D) and y (B, M, D)")
    x = x_local.to(torch.float32).contiguous()
    y = y_local.to(torch.float32).contiguous()
    b, n, d = x.shape
    m = y.shape[1]
    k = max(n, m)
    lib = _loader.core()
    if k > lib.tm_jv_max_k():
        raise RuntimeError(f"Batched JV (CUDA) supports max(N, M) <= 256, got K={k}")
    nbytes = lib.tm_jv_points_workspace_bytes(b, n, m)
    ws = torch.zeros(nbytes, dtype=torch.uint8, device=x.device)
    out = torch.full((b, n), -1, dtype=torch.long, device=x.device)
    stream = _stream(x.device)

    def launch(sentinel: float, pinf: int, check: int) -> None:
        rc = lib.tm_jv_points_solve_f32(x.data_ptr(), y.data_ptr(), b, n, m, d, sentinel, pinf,
                                        check, out.data_ptr(), ws.data_ptr(), nbytes, stream)
        if rc != 0:
            raise RuntimeError("batched JV kernel launch failed: "
                               + lib.tm_status_string(rc).decode())

    if b and n and m:
        launch(0.0, 0, 1)
    st = ws[:8].view(torch.int32)
    if dist.get_backend(group) == "nccl":
        t = _device_words(st)
        dist.all_reduce(t, op=dist.ReduceOp.MAX, group=group)
        words = t.cpu().tolist()
    else:
        flags, key = (int(v) & 0xFFFFFFFF for v in st.cpu().tolist())
        words = merge_words(stats_words(flags, key), group)
    sentinel, pinf = sentinel_from_words(words, k)
    if pinf and b and n and m:
        launch(sentinel, 1, 0)
    return out


_PEER_STREAMS: dict[int, torch.cuda.Stream] = {}


def _peer_stream(dev: torch.device) -> torch.cuda.Stream:
    """One long-lived stream per GPU for solve_multi_gpu.  The caching
    allocator keeps freed blocks per stream, so a fresh stream per call would
    allocate every slice anew (and free the cache, which synchronises the
    device, once memory runs short)."""
    if dev.index not in _PEER_STREAMS:
        _PEER_STREAMS[dev.index] = torch.cuda.Stream(dev)
    return _PEER_STREAMS[dev.index]


def shard_bounds(b: int, parts: int) -> list[tuple[int, int]]:
    """Contiguous slices [g * ceil(B / G), ...) of a batch of B problems."""
    step = -(-b // parts) if parts else 0
    return [(min(g * step, b), min((g + 1) * step, b)) for g in range(parts)]


def solve_multi_gpu(costs: torch.Tensor, devices: list[int] | None = None) -> torch.Tensor:
    """Solve one batch on several GPUs from a single process.

    ``costs`` lives on one CUDA device (the caller's); the result comes back
    there.  Slices travel by peer copies on each target GPU's stream; the
    statistics pass runs once on the caller's device.
    """
    if costs.device.type != "cuda" or costs.dim() != 3:
        raise RuntimeError("costs must be a 3D CUDA tensor")
    home = costs.device
    if devices is None:
        devices = list(range(torch.cuda.device_count()))
    c = costs.to(torch.float32).contiguous()
    b, n, m = c.shape
    k = max(n, m)
    if b == 0 or n == 0 or m == 0:
        return torch.full((b, n), -1, dtype=torch.long, device=home)
    if k > _loader.core().tm_jv_max_k():
        raise RuntimeError(f"Batched JV (CUDA) supports max(N, M) <= 256, got K={k}")
    sentinel, pinf = sentinel_from_words(_local_stats(c), k)
    out = torch.empty(b, n, dtype=torch.long, device=home)
    home_stream = torch.cuda.current_stream(home)
    ready = torch.cuda.Event()
    ready.record(home_stream)
    done = []
    local = None
    for (lo, hi), d in zip(shard_bounds(b, len(devices)), devices):
        if hi <= lo:
            continue
        dev = torch.device("cuda", d)
        if dev == home:
            local = (lo, hi)  # solved last, after the peers are under way
            continue
        s = _peer_stream(dev)
        with torch.cuda.device(dev), torch.cuda.stream(s):
            s.wait_event(ready)
            c.record_stream(s)  # s reads c: keep its block until s is done
            part = c[lo:hi].to(dev, non_blocking=True)
            res = _solve_local(part, sentinel, pinf)
            ev = torch.cuda.Event()
            ev.record(s)
            done.append((ev, res, lo, hi))
    if local is not None:
        lo, hi = local
        out[lo:hi] = _solve_local(c[lo:hi], sentinel, pinf)
    for ev, res, lo, hi in done:
        home_stream.wait_event(ev)
        out[lo:hi].copy_(res, non_blocking=True)
        res.record_stream(home_stream)  # read by the home stream after s
    return out
