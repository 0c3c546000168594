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
  each GPU in pieces, each piece solved as soon as it has arrived while the
  next one crosses the link, and the int64 results are copied back into one
  output on the caller's device.

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
_WS_TIMEOUT, _ERR_TIMEOUT = 8, 7  # TM_WS_TIMEOUT, TM_ERR_TIMEOUT


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


_PEER_STREAMS: dict[tuple[int, str], torch.cuda.Stream] = {}
_WORKSPACES: dict[int, torch.Tensor] = {}


def _peer_stream(dev: torch.device, role: str) -> torch.cuda.Stream:
    """Long-lived streams per GPU for solve_multi_gpu (a copy stream and two
    solve streams).  The caching allocator keeps freed blocks per stream, so
    a fresh stream per call would allocate every slice anew (and free the
    cache, which synchronises the device, once memory runs short)."""
    key = (dev.index, role)
    if key not in _PEER_STREAMS:
        _PEER_STREAMS[key] = torch.cuda.Stream(dev)
    return _PEER_STREAMS[key]


def _workspaces(dev: torch.device, count: int) -> torch.Tensor:
    """`count` solve workspaces (one tm_jv_workspace each) on `dev`, kept
    across calls and grown on demand."""
    words = _loader.core().tm_jv_workspace_bytes() // 4
    ws = _WORKSPACES.get(dev.index)
    if ws is None or ws.shape[0] < count:
        ws = torch.zeros(max(count, 16), words, dtype=torch.int32, device=dev)
        _WORKSPACES[dev.index] = ws
    return ws


def shard_bounds(b: int, parts: int) -> list[tuple[int, int]]:
    """Contiguous slices [g * ceil(B / G), ...) of a batch of B problems."""
    step = -(-b // parts) if parts else 0
    return [(min(g * step, b), min((g + 1) * step, b)) for g in range(parts)]


def _launch(lib, fn: str, *args) -> None:
    rc = getattr(lib, fn)(*args)
    if rc != 0:
        raise RuntimeError("batched JV kernel launch failed: " + lib.tm_status_string(rc).decode())


def solve_multi_gpu(costs: torch.Tensor, devices: list[int] | None = None,
                    chunks: int = 4) -> torch.Tensor:
    """Solve one batch on several GPUs from a single process.

    ``costs`` lives on one CUDA device (the caller's); the result comes back
    there.  The batch is split into contiguous slices, one per device, and
    every slice into ``chunks`` pieces.  On each GPU a copy stream brings the
    pieces over NVLink one after another while two solve streams take turns
    solving the pieces that have arrived, in check mode (each piece into its
    own workspace), so piece k + 1 crosses the link while piece k is solved
    and a piece's last problems overlap the next piece's first.  There is no
    separate statistics pass: after one host read of every piece's
    statistics (the reference raises on NaN / -inf after one host check as
    well, cuda/cuda_common.cuh:245-249), a batch holding +inf is solved again
    slice by slice with the global sentinel, from the slices already on their
    GPUs.  The int64 results go back to the caller's device on the copy
    streams.  The result equals ``torch.ops.assignment.jonker_dense_batch``
    on the whole batch.
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
    lib = _loader.core()
    if k > lib.tm_jv_max_k():
        raise RuntimeError(f"Batched JV (CUDA) supports max(N, M) <= 256, got K={k}")
    out = torch.empty(b, n, dtype=torch.long, device=home)
    home_stream = torch.cuda.current_stream(home)
    ready = torch.cuda.Event()
    ready.record(home_stream)
    jobs = []
    for (lo, hi), d in zip(shard_bounds(b, len(devices)), devices):
        if hi <= lo:
            continue
        dev = torch.device("cuda", d)
        pieces = [(p0, p1) for p0, p1 in shard_bounds(hi - lo, max(1, chunks)) if p1 > p0]
        ws = _workspaces(dev, len(pieces))
        cs = _peer_stream(dev, "copy")
        solvers = (_peer_stream(dev, "solve0"), _peer_stream(dev, "solve1"))
        with torch.cuda.device(dev), torch.cuda.stream(cs):
            cs.wait_event(ready)
            for st in solvers:
                st.wait_stream(cs)  # earlier users of this GPU's workspaces are done
            if dev == home:
                part = c[lo:hi]
                c.record_stream(solvers[0])
                c.record_stream(solvers[1])
            else:
                part = torch.empty(hi - lo, n, m, dtype=torch.float32, device=dev)
                c.record_stream(cs)  # cs reads c: keep its block until cs is done
            res = torch.empty(hi - lo, n, dtype=torch.long, device=dev)
            for q, (p0, p1) in enumerate(pieces):
                st = solvers[q % 2]
                if dev != home:
                    part[p0:p1].copy_(c[lo + p0:lo + p1], non_blocking=True)
                    arrived = torch.cuda.Event()
                    arrived.record(cs)
                    st.wait_event(arrived)
                _launch(lib, "tm_jv_solve_checked_f32", part[p0:].data_ptr(), p1 - p0, n, m,
                        res[p0:].data_ptr(), ws[q].data_ptr(), st.cuda_stream)
            for st in solvers:
                cs.wait_stream(st)
                part.record_stream(st)
                res.record_stream(st)
        jobs.append((dev, part, res, lo, hi, ws[:len(pieces)]))
    # one host read of every piece's statistics and status, after its solves
    flags, key = 0, 0
    for dev, part, res, lo, hi, ws in jobs:
        torch.cuda.current_stream(dev).wait_stream(_peer_stream(dev, "copy"))
        with torch.cuda.device(dev):
            # words 0, 1: tm_jv_stats; word 4: the status (TM_WS_* bits)
            for f, kk, status in ws[:, [0, 1, 4]].cpu().tolist():
                flags |= int(f) & 0xFFFFFFFF
                key = max(key, int(kk) & 0xFFFFFFFF)
                if status & _WS_TIMEOUT:
                    raise RuntimeError("jonker_dense_batch: "
                                       + lib.tm_status_string(_ERR_TIMEOUT).decode())
    sentinel, pinf = sentinel_from_words(stats_words(flags, key), k)
    for dev, part, res, lo, hi, ws in jobs:
        cs = _peer_stream(dev, "copy")
        with torch.cuda.device(dev), torch.cuda.stream(cs):
            if pinf:
                _launch(lib, "tm_jv_solve_f32", part.data_ptr(), hi - lo, n, m, sentinel, 1,
                        res.data_ptr(), ws[0].data_ptr(), cs.cuda_stream)
            out[lo:hi].copy_(res, non_blocking=True)
            out.record_stream(cs)
            done = torch.cuda.Event()
            done.record(cs)
        home_stream.wait_event(done)
    return out
