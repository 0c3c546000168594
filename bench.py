#!/usr/bin/env python
"""Throughput of the batched Jonker-Volgenant op (problems solved per second).

    python bench.py [--gpus N] [--steps K] [--warmup W] [--config c2] [--impl ours|reference]

One step = one call of torch.ops.assignment.jonker_dense_batch on a resident
(B, N, M) fp32 batch (statistics pass, host check of the NaN / -inf verdict,
solve).  At N > 1 (torchrun, one rank per GPU) every rank holds a contiguous
slice of one global batch and runs torchmatch_b200.sharded.solve_sharded (one
all-reduce of the statistics words, then a local solve): the per-rank work is
fixed, so scaling is weak.  Rank 0 prints one JSON line.

Workloads (synthetic, seeded; tests/golden/cases.py holds the recipes):
  c1  B=64     N=M=32   uniform[0,1)                (configs[0], CPU case)
  c2  B=4096   N=M=64   uniform[0,1)                (configs[1], default)
  c3  B=16384  N=M=128  integers in {0..15}
  c4  B=8192   N=100 M=150 uniform[0,10), 20% +inf
  c5  B=65536  N=M=256  |x_i - y_j|^2, x, y ~ N(0, I16)  (B split over ranks)

`value` is device time (CUDA events, max over ranks) with inputs resident in
HBM; consecutive steps rotate over enough input copies that their total
exceeds twice the 126 MB L2, so every step reads its batch from HBM.  `e2e`
is the same op with a pinned host batch copied in (four pieces, double-
buffered on a copy stream) and the result copied out to pinned memory inside
each timed step.  `roofline` is measured live: the solve kernel alone,
launched through the C ABI between CUDA events on its stream, against the
measured HBM copy bandwidth.  `cpu_baseline` times the reference's own CPU
solver (oracle/_ref, built from the reference sources) on the host cores.

Every named shape is reported in the same line: `per_config` (one GPU) gives,
for c1, c3, c4 and c5, the op's problems/s on the whole named batch, its solve
launch's roofline fraction and the reference CPU solver on this host (and
`c5_fused`: the config-5 problems built from point sets inside the kernel), and
`strong_c5` (every N) gives config 5 as strong scaling -- the fixed
B = 65536 batch split over the N ranks, max over ranks.
"""

from __future__ import annotations

import argparse
import ctypes
import json
import os
import statistics
import subprocess
import sys
import threading
import time
from pathlib import Path

ROOT = Path(__file__).resolve().parent
sys.path.insert(0, str(ROOT))
sys.path.insert(0, str(ROOT / "tests" / "golden"))

METRIC = ("LAPs solved/sec (B×N×M fp32 batch) at 1/2/4/8 B200; "
          "% of HBM roofline")
UNIT = "problems/s"
L2_BYTES = 126 * 1024 * 1024
FALLBACK_HBM_GBS = 6650.0

CONFIGS = {
    "c1": dict(B=64, N=32, M=32, desc="config1: B=64 N=M=32 uniform[0,1) fp32"),
    "c2": dict(B=4096, N=64, M=64, desc="config2: B=4096 N=M=64 uniform[0,1) fp32"),
    "c3": dict(B=16384, N=128, M=128, desc="config3: B=16384 N=M=128 integers {0..15} fp32"),
    "c4": dict(B=8192, N=100, M=150, desc="config4: B=8192 N=100 M=150 uniform[0,10) 20% +inf"),
    "c5": dict(B=65536, N=256, M=256, desc="config5: B=65536 N=M=256 |x-y|^2, x,y~N(0,I16)",
               split=True),
}


def make_batch(cfg: str, b: int, seed: int):
    """Seeded CPU batch of workload `cfg` with b problems."""
    import torch

    import cases

    if cfg == "c1":
        return cases.config1()[:b]
    if cfg == "c2":
        return torch.rand(b, 64, 64, generator=torch.Generator().manual_seed(seed))
    if cfg == "c3":
        return torch.randint(0, 16, (b, 128, 128),
                             generator=torch.Generator().manual_seed(seed)).float()
    if cfg == "c4":
        g = torch.Generator().manual_seed(seed)
        c = torch.rand(b, 100, 150, generator=g) * 10
        mask = torch.rand(b, 100, 150, generator=g) < 0.2
        i = torch.arange(100)
        mask[:, i, i] = False
        return c.masked_fill(mask, float("inf"))
    if cfg == "c5":
        return cases.config5_chunk(b, seed)
    raise ValueError(cfg)


def make_batch_device(cfg: str, b: int, seed: int, device):
    """Same distribution generated on the GPU (timing only; parity runs use
    the CPU recipes)."""
    import torch

    g = torch.Generator(device=device).manual_seed(seed)
    if cfg == "c5":
        out = torch.empty(b, 256, 256, device=device)
        for s in range(0, b, 512):
            e = min(b, s + 512)
            x = torch.randn(e - s, 256, 16, device=device, generator=g)
            y = torch.randn(e - s, 256, 16, device=device, generator=g)
            out[s:e] = ((x[:, :, None] - y[:, None]) ** 2).sum(-1)
        return out
    if cfg == "c3":
        return torch.randint(0, 16, (b, 128, 128), device=device, generator=g).float()
    if cfg == "c4":
        c = torch.rand(b, 100, 150, device=device, generator=g) * 10
        mask = torch.rand(b, 100, 150, device=device, generator=g) < 0.2
        i = torch.arange(100, device=device)
        mask[:, i, i] = False
        return c.masked_fill(mask, float("inf"))
    return make_batch(cfg, b, seed).to(device)


def peak_hbm():
    p = ROOT / "MEASURED_PEAKS.json"
    try:
        v = float(json.loads(p.read_text())["hbm_gbs"])
        return v, "MEASURED_PEAKS.json hbm_gbs (of measured)"
    except Exception:
        return FALLBACK_HBM_GBS, "profiling-recipe fallback 6.65 TB/s (of fallback)"


def traffic_for(cfg: str):
    """DRAM bytes per solve launch from the committed ncu summary, if any."""
    p = ROOT / "profiles" / "traffic.json"
    try:
        return json.loads(p.read_text()).get(cfg)
    except Exception:
        return None


class ClockSampler:
    """nvidia-smi clocks / throttle reasons sampled every 100 ms."""

    FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, gpu_index: int):
        self.gpu = gpu_index
        self.rows: list[list[str]] = []
        self.proc = None
        self.thread = None

    def start(self):
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", f"--query-gpu={self.FIELDS}", "--format=csv,noheader,nounits",
                 "-lms", "100", "-i", str(self.gpu)],
                stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
        except OSError:
            self.proc = None
            return
        self.thread = threading.Thread(target=self._read, daemon=True)
        self.thread.start()

    def _read(self):
        for line in self.proc.stdout:
            parts = [p.strip() for p in line.split(",")]
            if len(parts) >= 9:
                self.rows.append(parts)

    def stop(self):
        if self.proc is None:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["nvidia-smi unavailable"]}
        time.sleep(0.25)
        self.proc.terminate()
        try:
            self.proc.wait(timeout=5)
        except subprocess.TimeoutExpired:
            self.proc.kill()
        self.thread.join(timeout=2)
        sm = [float(r[1]) for r in self.rows if r[1].replace(".", "").isdigit()]
        mx = [float(r[2]) for r in self.rows if r[2].replace(".", "").isdigit()]
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        reasons = sorted({names[k] for r in self.rows for k in range(4) if r[5 + k] == "Active"})
        return {"sm_mhz": statistics.median(sm) if sm else None,
                "sm_max_mhz": max(mx) if mx else None, "reasons": reasons,
                "samples": len(self.rows)}


def cpu_baseline(cfg: str, seconds: float = 6.0):
    """The reference's CPU solver (oracle/_ref) -- else the oracle port -- on
    all host threads over a bounded sample of the workload."""
    import oracle

    kind = "reference" if oracle.reference_available() else "port"
    fn = oracle.reference_jonker_dense_batch if kind == "reference" else oracle.jonker_dense_batch
    spec = CONFIGS[cfg]
    b = min(spec["B"], {"c3": 2048, "c4": 2048, "c5": 512}.get(cfg, spec["B"]))
    x = make_batch(cfg, b, 0).numpy()
    threads = oracle.host_threads()
    fn(x[: min(b, 64)], threads)
    times = []
    t_end = time.perf_counter() + seconds
    while len(times) < 3 or (time.perf_counter() < t_end and len(times) < 50):
        t0 = time.perf_counter()
        fn(x, threads)
        times.append(time.perf_counter() - t0)
    med = statistics.median(times)
    return {"value": b / med, "unit": UNIT, "cores": threads, "kind": kind,
            "sample": f"{spec['desc'].split(':')[0]} first {b} problems x {len(times)} runs, "
                      f"median {med * 1e3:.1f} ms, {threads} threads"}


def run_reference(args):
    rank = int(os.environ.get("RANK", "0"))
    if rank != 0:
        return
    import oracle

    kind = "reference" if oracle.reference_available() else "port"
    fn = oracle.reference_jonker_dense_batch if kind == "reference" else oracle.jonker_dense_batch
    spec = CONFIGS[args.config]
    b = min(spec["B"], {"c3": 2048, "c4": 2048, "c5": 512}.get(args.config, spec["B"]))
    x = make_batch(args.config, b, 0).numpy()
    threads = oracle.host_threads()
    for _ in range(args.warmup):
        fn(x, threads)
    t0 = time.perf_counter()
    for _ in range(args.steps):
        fn(x, threads)
    dt = time.perf_counter() - t0
    value = b * args.steps / dt
    line = {
        "impl": "reference", "metric": METRIC, "value": value, "unit": UNIT,
        "n_gpus": args.gpus, "steps": args.steps, "warmup": args.warmup,
        "ms_per_step": dt / args.steps * 1e3, "higher_is_better": True, "scaling": "weak",
        "vs_baseline": None, "dtype": "f32", "data": "synthetic",
        "config": {"workload": spec["desc"], "sample_problems": b},
        "cpu_baseline": {"value": value, "unit": UNIT, "cores": threads, "kind": kind,
                         "sample": f"first {b} problems of the workload per step"},
        "e2e": {"value": value, "unit": UNIT, "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
        "reference_gpu_kernel": reference_gpu_kernel(args, spec),
    }
    print(json.dumps(line), flush=True)


def reference_gpu_kernel(args, spec):
    """The reference's own batched CUDA kernel (cuda/jonker_tiled.cuh, built
    from its sources into oracle/_ref for sm_100a) on the same resident
    workload, CUDA events around K launches.  Kernel only: the reference op
    also runs a statistics scan and an +inf rewrite first.  Its kernel takes
    square K <= 64 (configs 1 and 2); otherwise None."""
    import oracle

    try:
        import torch
    except ImportError:
        return None
    if spec["N"] != spec["M"] or spec["N"] > 64 or not torch.cuda.is_available() \
            or not oracle.reference_cuda_available():
        return None
    dev = torch.device("cuda", 0)
    b = spec["B"]
    per_bytes = b * spec["N"] * spec["M"] * 4
    nbuf = max(1, min(8, -(-2 * L2_BYTES // per_bytes) + 1))
    bufs = [make_batch_device(args.config, b, k, dev).contiguous() for k in range(nbuf)]
    for k in range(args.warmup):
        oracle.reference_cuda_jonker_dense_batch(bufs[k % nbuf])
    torch.cuda.synchronize()
    t0 = torch.cuda.Event(enable_timing=True)
    t1 = torch.cuda.Event(enable_timing=True)
    t0.record()
    for k in range(args.steps):
        oracle.reference_cuda_jonker_dense_batch(bufs[k % nbuf])
    t1.record()
    torch.cuda.synchronize()
    ms = t0.elapsed_time(t1) / args.steps
    return {"value": b / (ms / 1e3), "unit": UNIT, "ms_per_launch": ms,
            "kernel": "match_batch::lap_batch_kernel (reference cuda/jonker_tiled.cuh, "
                      "nvcc sm_100a)", "inputs": "resident in HBM, rotating copies > 2x L2"}


class _near_gpu:
    """Binds this thread to the CPUs of the GPU's NUMA node (from sysfs) for
    the scope of the block, then restores the previous set; a no-op where
    sysfs does not list them."""

    def __init__(self, dev):
        self.dev = dev
        self.prev = None

    def __enter__(self):
        import torch

        try:
            pr = torch.cuda.get_device_properties(self.dev)
            bus = f"{pr.pci_domain_id:04x}:{pr.pci_bus_id:02x}:{pr.pci_device_id:02x}.0"
            text = Path(f"/sys/bus/pci/devices/{bus}/local_cpulist").read_text().strip()
            cpus = set()
            for part in text.split(","):
                lo, _, hi = part.partition("-")
                cpus.update(range(int(lo), int(hi or lo) + 1))
            cpus &= os.sched_getaffinity(0)
            if cpus:
                self.prev = os.sched_getaffinity(0)
                os.sched_setaffinity(0, cpus)
        except (OSError, ValueError, AttributeError, TypeError):
            self.prev = None
        return self

    def __exit__(self, *exc):
        if self.prev:
            os.sched_setaffinity(0, self.prev)
        return False


def _device_ms(fn, steps: int, warmup: int) -> float:
    """Mean ms per call of fn() between CUDA events on the current stream."""
    import torch

    for _ in range(warmup):
        fn()
    torch.cuda.synchronize()
    t0 = torch.cuda.Event(enable_timing=True)
    t1 = torch.cuda.Event(enable_timing=True)
    t0.record()
    for _ in range(steps):
        fn()
    t1.record()
    torch.cuda.synchronize()
    return t0.elapsed_time(t1) / steps


def per_config_record(cfg: str, dev, lib, args, peak: float) -> dict:
    """One GPU, the whole named batch of `cfg` resident in HBM: the op
    (device-timed per call), its dominant solve launch alone through the C
    ABI (the roofline kernel), and the reference's CPU solver on a bounded
    sample on this host.  Inputs: one batch larger than 2x L2 for c3-c5;
    c1 is a 256 KB launch-bound case that stays in L2."""
    import torch

    spec = CONFIGS[cfg]
    b, n, m = spec["B"], spec["N"], spec["M"]
    x = make_batch_device(cfg, b, 11, dev).contiguous()
    op = torch.ops.assignment.jonker_dense_batch
    steps = {"c1": 50, "c3": 20, "c4": 20, "c5": 3}.get(cfg, 20)
    op_ms = _device_ms(lambda: op(x), steps, 2)
    ws = torch.zeros(lib.tm_jv_workspace_bytes() // 4, dtype=torch.int32, device=dev)
    out = torch.empty(b, n, dtype=torch.long, device=dev)
    stream = torch.cuda.current_stream().cuda_stream
    has_inf = bool(torch.isinf(x).any())
    if has_inf:
        # the op's second launch, with the batch-global sentinel, is the one
        # that solves every problem; time that launch
        fin = x[torch.isfinite(x)]
        sent = (float(fin.max()) + 1.0) * float(max(n, m) + 1) if fin.numel() else 1.0
        sent = float(torch.tensor(sent, dtype=torch.float32))

        def kern():
            rc = lib.tm_jv_solve_f32(x.data_ptr(), b, n, m, ctypes.c_float(sent), 1,
                                     out.data_ptr(), ws.data_ptr(), stream)
            assert rc == 0, lib.tm_status_string(rc)
        kname = "jv_batch_kernel (sentinel solve; the op runs a check-mode pass first)"
    else:
        def kern():
            rc = lib.tm_jv_solve_checked_f32(x.data_ptr(), b, n, m, out.data_ptr(),
                                             ws.data_ptr(), stream)
            assert rc == 0, lib.tm_status_string(rc)
        kname = "jv_batch_kernel (check mode; the op's only launch)"
    k_ms = _device_ms(kern, steps, 1)
    del x, out
    torch.cuda.empty_cache()
    alg = b * (n * m * 4 + n * 8)
    rec = {"workload": spec["desc"], "B": b, "value": b / (op_ms / 1e3), "unit": UNIT,
           "ms_per_step": op_ms, "steps": steps,
           "roofline": {"bound": "hbm", "kernel": kname, "avg_launch_us": k_ms * 1e3,
                        "alg_bytes_per_launch": alg,
                        "achieved": alg / (k_ms / 1e3) / 1e9, "peak": peak, "unit": "GB/s",
                        "frac": alg / (k_ms / 1e3) / 1e9 / peak,
                        "traffic": traffic_for(cfg)},
           "gpu_launches_per_step": 2 if has_inf else 1}
    if not args.no_cpu:
        rec["cpu_baseline"] = cpu_baseline(cfg, seconds=3.0)
    return rec


def fused_c5_record(dev, lib, peak: float) -> dict:
    """Config-5 problems from point sets through the fused op
    (jonker_sqeuclidean_batch: the costs are built inside the solve kernel),
    B=65536, x, y ~ N(0, I16): the op per call and its launch through the C
    ABI, CUDA events.  Algorithmic bytes are the points and the mapping."""
    import torch

    b, n, d = 65536, 256, 16
    g = torch.Generator(device=dev).manual_seed(1)
    x = torch.randn(b, n, d, device=dev, generator=g)
    y = torch.randn(b, n, d, device=dev, generator=g)
    op_ms = _device_ms(lambda: torch.ops.assignment.jonker_sqeuclidean_batch(x, y), 3, 1)
    nbytes = lib.tm_jv_points_workspace_bytes(b, n, n)
    ws = torch.empty(nbytes, dtype=torch.uint8, device=dev)
    out = torch.empty(b, n, dtype=torch.long, device=dev)
    stream = torch.cuda.current_stream().cuda_stream

    def kern():
        rc = lib.tm_jv_points_solve_f32(x.data_ptr(), y.data_ptr(), b, n, n, d, 0.0, 0, 1,
                                        out.data_ptr(), ws.data_ptr(), nbytes, stream)
        assert rc == 0, lib.tm_status_string(rc)
    k_ms = _device_ms(kern, 3, 1)
    del x, y, ws, out
    torch.cuda.empty_cache()
    alg = b * (2 * n * d * 4 + n * 8)
    return {"workload": f"config5 problems from points: B={b} N=M={n} D={d}, x,y~N(0,I16)",
            "value": b / (op_ms / 1e3), "unit": UNIT, "ms_per_step": op_ms,
            "roofline": {"bound": "hbm", "kernel": "jv_batch_kernel (points, check mode)",
                         "avg_launch_us": k_ms * 1e3, "alg_bytes_per_launch": alg,
                         "achieved": alg / (k_ms / 1e3) / 1e9, "peak": peak, "unit": "GB/s",
                         "frac": alg / (k_ms / 1e3) / 1e9 / peak,
                         "traffic": traffic_for("c5_fused")},
            "cost_tensor_bytes_avoided": b * n * n * 4}


def strong_c5_record(dev, world: int, rank: int, args) -> dict:
    """Config 5 as strong scaling: the fixed B=65536 batch split into
    `world` contiguous slices, one per rank (each generated on its GPU),
    solved by sharded.solve_sharded (one all-reduce of the statistics words,
    then the local solve) every step; max over ranks of the CUDA-event time."""
    import torch
    import torch.distributed as dist

    from torchmatch_b200 import sharded

    spec = CONFIGS["c5"]
    b = spec["B"] // world
    x = make_batch_device("c5", b, 500 + rank, dev).contiguous()
    steps = 3
    step = (lambda: sharded.solve_sharded(x)) if world > 1 else \
        (lambda: torch.ops.assignment.jonker_dense_batch(x))
    step()
    torch.cuda.synchronize()
    if world > 1:
        dist.barrier()
    torch.cuda.synchronize()
    t0 = torch.cuda.Event(enable_timing=True)
    t1 = torch.cuda.Event(enable_timing=True)
    t0.record()
    for _ in range(steps):
        step()
    t1.record()
    torch.cuda.synchronize()
    ms = t0.elapsed_time(t1) / steps
    if world > 1:
        t = torch.tensor([ms], device=dev)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        ms = float(t.item())
    del x
    torch.cuda.empty_cache()
    return {"workload": spec["desc"], "global_batch": spec["B"], "per_gpu_batch": b,
            "n_gpus": world, "scaling": "strong", "value": spec["B"] / (ms / 1e3),
            "unit": UNIT, "ms_per_step": ms, "steps": steps,
            "timing": "CUDA events per rank, max over ranks"}


def run_ours(args):
    import torch
    import torch.distributed as dist

    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    if world > 1:
        dist.init_process_group("nccl", device_id=dev)

    import torchmatch_b200  # noqa: F401
    from torchmatch_b200 import _loader, sharded

    lib = _loader.core()
    spec = CONFIGS[args.config]
    n, m = spec["N"], spec["M"]
    b = spec["B"] // world if spec.get("split") else spec["B"]
    per_bytes = b * n * m * 4
    nbuf = max(1, min(8, -(-2 * L2_BYTES // per_bytes) + 1)) if per_bytes < 2 * L2_BYTES else 1
    bufs = [make_batch_device(args.config, b, 1000 * rank + k, dev) for k in range(nbuf)]
    op = torch.ops.assignment.jonker_dense_batch

    def step(x):
        if world > 1:
            return sharded.solve_sharded(x)
        return op(x)

    def barrier():
        torch.cuda.synchronize()
        if world > 1:
            dist.barrier()
        torch.cuda.synchronize()

    gpu_index = local
    vis = os.environ.get("CUDA_VISIBLE_DEVICES")
    if vis:
        try:
            gpu_index = int(vis.split(",")[local])
        except ValueError:
            pass
    clocks = ClockSampler(gpu_index) if rank == 0 else None

    for k in range(args.warmup):
        step(bufs[k % nbuf])
    barrier()
    # Keep the GPU loaded for ~0.5 s on both sides of the timed region so the
    # clock sampler sees it under load.  Every rank runs the same number of
    # steps (each step of a sharded solve is a collective).
    tw = time.perf_counter()
    step(bufs[0])
    barrier()
    per = torch.tensor([time.perf_counter() - tw], dtype=torch.float64, device=dev)
    if world > 1:
        dist.all_reduce(per, op=dist.ReduceOp.MAX)
    n_load = max(1, min(2000, int(0.5 / max(float(per.item()), 1e-6))))
    if clocks:
        clocks.start()
    for _ in range(n_load):
        step(bufs[0])
    barrier()
    t0 = torch.cuda.Event(enable_timing=True)
    t1 = torch.cuda.Event(enable_timing=True)
    t0.record()
    for k in range(args.steps):
        step(bufs[k % nbuf])
    t1.record()
    barrier()
    ms = t0.elapsed_time(t1)
    for _ in range(max(1, n_load // 2)):
        step(bufs[0])
    barrier()
    if clocks:
        clk = clocks.stop()
    if world > 1:
        t = torch.tensor([ms], device=dev)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        ms = float(t.item())
    value = b * world * args.steps / (ms / 1e3)

    # ---- kernel-only timing of the op's solve launch (roofline) ------------
    # The op runs one kernel per step: the check-mode solve, which also
    # gathers the batch statistics (a second, sentinel launch happens only for
    # batches holding +inf).  It is timed alone here, through the C ABI,
    # between CUDA events on the stream it is launched on.
    ws = torch.zeros(lib.tm_jv_workspace_bytes() // 4, dtype=torch.int32, device=dev)
    out = torch.empty(b, n, dtype=torch.long, device=dev)
    stream = torch.cuda.current_stream().cuda_stream
    reps = max(3, min(args.steps, 50))
    evs = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True))
           for _ in range(reps)]
    for r in range(reps):
        x = bufs[r % nbuf]
        evs[r][0].record()
        rc = lib.tm_jv_solve_checked_f32(x.data_ptr(), b, n, m, out.data_ptr(), ws.data_ptr(),
                                         stream)
        evs[r][1].record()
        assert rc == 0, lib.tm_status_string(rc)
    torch.cuda.synchronize()
    solve_ms = statistics.mean(a.elapsed_time(z) for a, z in evs)
    # ---- pipelined: batches in flight on several streams (one GPU) ---------
    # jonker_dense_batch_async does the same work (check-mode solve, gated
    # sentinel re-solve on the device) without a host synchronisation, so the
    # next batch's warps fill the SMs that a batch's last problems leave idle.
    # The device statuses (NaN / -inf / loop bound) are read after the timed
    # region and must all be 0.
    pipelined = None
    if world == 1:
        aop = torch.ops.assignment.jonker_dense_batch_async
        nstreams = args.streams
        streams = [torch.cuda.Stream(dev) for _ in range(nstreams)]

        def pipe(nsteps):
            cur = torch.cuda.current_stream()
            for st_ in streams:
                st_.wait_stream(cur)
            stats = []
            for k in range(nsteps):
                with torch.cuda.stream(streams[k % nstreams]):
                    stats.append(aop(bufs[k % nbuf])[1])
            for st_ in streams:
                cur.wait_stream(st_)
            return stats

        pipe(max(3, args.warmup))
        barrier()
        p0 = torch.cuda.Event(enable_timing=True)
        p1 = torch.cuda.Event(enable_timing=True)
        p0.record()
        stats = pipe(args.steps)
        p1.record()
        barrier()
        p_ms = p0.elapsed_time(p1)
        assert int(torch.stack(stats).max()) == 0, "a pipelined batch reported a status"
        pipelined = {"value": b * args.steps / (p_ms / 1e3), "unit": UNIT,
                     "ms_per_step": p_ms / args.steps, "streams": nstreams,
                     "op": "jonker_dense_batch_async", "launches_per_step": 2}

    alg_bytes = b * (n * m * 4 + n * 8)
    achieved = alg_bytes / (solve_ms / 1e3) / 1e9
    peak, peak_src = peak_hbm()

    # ---- end to end: pinned host batch in, mapping out ---------------------
    # The pinned buffers are filled by a thread bound to the CPUs next to the
    # GPU, so their pages sit in the GPU's NUMA node (first touch), as a
    # caller feeding this GPU would place them.
    with _near_gpu(dev):
        host = make_batch(args.config, min(b, 8192), 7).pin_memory() if args.config != "c5" \
            else bufs[0][: min(b, 4096)].cpu().pin_memory()
        res = torch.empty(host.shape[0], n, dtype=torch.long).pin_memory()
        res.zero_()
    eb = host.shape[0]
    e_steps = max(3, min(args.steps, 20))
    op(host.to(dev, non_blocking=True)).cpu()
    barrier()
    # Each step copies its batch from pinned host memory, solves it and reads
    # the mapping back.  The upload of step k+1 runs on a copy stream while
    # step k solves (double-buffered), as a user of the op would pipeline it;
    # every copy still lies inside the timed region.
    copy_stream = torch.cuda.Stream(dev)

    def upload(dst):
        # four pieces: on this host link one 64 MiB pinned copy ran at
        # 37.5 GB/s, the same bytes in 2-16 pieces at 53-55 GB/s
        flat_d, flat_h = dst.view(-1), host.view(-1)
        step_n = -(-flat_h.numel() // 4)
        for p0 in range(0, flat_h.numel(), step_n):
            flat_d[p0:p0 + step_n].copy_(flat_h[p0:p0 + step_n], non_blocking=True)

    dbuf = [torch.empty(host.shape, dtype=host.dtype, device=dev) for _ in range(2)]
    ready = [torch.cuda.Event() for _ in range(2)]
    free = [torch.cuda.Event() for _ in range(2)]
    compute = torch.cuda.current_stream(dev)
    e0 = torch.cuda.Event(enable_timing=True)
    e1 = torch.cuda.Event(enable_timing=True)
    e0.record(compute)
    copy_stream.wait_event(e0)
    with torch.cuda.stream(copy_stream):
        upload(dbuf[0])
        ready[0].record(copy_stream)
    for k in range(e_steps):
        cur, nxt = k % 2, (k + 1) % 2
        if k + 1 < e_steps:
            with torch.cuda.stream(copy_stream):
                if k >= 1:
                    copy_stream.wait_event(free[nxt])
                upload(dbuf[nxt])
                ready[nxt].record(copy_stream)
        compute.wait_event(ready[cur])
        out_d = step(dbuf[cur])
        free[cur].record(compute)
        res.copy_(out_d, non_blocking=True)  # complete at the next step's sync and at e1
    e1.record(compute)
    barrier()
    assert int(res.min()) >= -1  # the last mapping arrived on the host
    e_ms = e0.elapsed_time(e1)
    if world > 1:
        t = torch.tensor([e_ms], device=dev)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        e_ms = float(t.item())
    e2e = {"value": eb * world * e_steps / (e_ms / 1e3), "unit": UNIT,
           "h2d_bytes_per_step": host.numel() * 4 * world,
           "d2h_bytes_per_step": res.numel() * 8 * world,
           "problems_per_step": eb * world}

    base = cpu_baseline(args.config) if (rank == 0 and world == 1) else None
    per_config = None
    if world == 1 and not args.no_per_config:
        per_config = {c: per_config_record(c, dev, lib, args, peak)
                      for c in ("c1", "c3", "c4", "c5")}
        per_config["c5_fused"] = fused_c5_record(dev, lib, peak)
    strong = strong_c5_record(dev, world, rank, args) if not args.no_per_config else None
    if rank == 0:
        line = {
            "metric": METRIC, "value": value, "unit": UNIT, "n_gpus": world,
            "steps": args.steps, "warmup": args.warmup, "ms_per_step": ms / args.steps,
            "higher_is_better": True, "scaling": "weak", "vs_baseline": None,
            "dtype": "f32", "data": "synthetic",
            "config": {"workload": spec["desc"], "global_batch": b * world, "per_gpu_batch": b,
                       "parallelism": f"batch-sharded x{world}" if world > 1 else "single GPU",
                       "l2": f"{nbuf} rotating input copies of {per_bytes / 2**20:.0f} MiB "
                             f"(> 2x L2) so each step reads HBM"},
            "roofline": {"bound": "hbm", "achieved": achieved, "peak": peak, "unit": "GB/s",
                         "frac": achieved / peak, "traffic": traffic_for(args.config),
                         "kernel": "jv_batch_kernel (check mode)", "avg_launch_us": solve_ms * 1e3,
                         "alg_bytes_per_launch": alg_bytes, "peak_source": peak_src,
                         "op_roofline_frac": (alg_bytes / (ms / args.steps / 1e3) / 1e9) / peak},
            "cpu_baseline": base,
            "e2e": e2e,
            "pipelined": pipelined,
            "per_config": per_config,
            "strong_c5": strong,
            "gpu_launches": args.steps,  # one check-mode solve per step (no +inf)
            "clocks": clk if clocks else None,
        }
        print(json.dumps(line), flush=True)
    if world > 1:
        dist.barrier()
        dist.destroy_process_group()


def run_fused(args):
    """Fused cost construction (jonker_sqeuclidean_batch) on the config-5
    problem set: x, y ~ N(0, I16) point sets of 256 points, B problems.
    Reported beside the dense op on the same problems with the (B, 256, 256)
    cost tensor already built (cost construction not timed there), and
    beside the unfused pipeline torch.cdist(x, y) ** 2 -> dense op.  One GPU."""
    import torch

    import torchmatch_b200  # noqa: F401
    from torchmatch_b200 import _loader

    if int(os.environ.get("WORLD_SIZE", "1")) > 1:
        if int(os.environ.get("RANK", "0")) == 0:
            print(json.dumps({"impl": "ours", "unavailable": "--fused runs on one GPU"}))
        return
    dev = torch.device("cuda", 0)
    torch.cuda.set_device(dev)
    b, n, d = args.batch or 65536, 256, 16
    g = torch.Generator(device=dev).manual_seed(1)
    x = torch.randn(b, n, d, device=dev, generator=g)
    y = torch.randn(b, n, d, device=dev, generator=g)
    ops = torch.ops.assignment

    def timed(fn, steps):
        for _ in range(args.warmup):
            fn()
        torch.cuda.synchronize()
        t0 = torch.cuda.Event(enable_timing=True)
        t1 = torch.cuda.Event(enable_timing=True)
        t0.record()
        for _ in range(steps):
            fn()
        t1.record()
        torch.cuda.synchronize()
        return t0.elapsed_time(t1) / steps

    steps = max(3, min(args.steps, 10))
    vis = (os.environ.get("CUDA_VISIBLE_DEVICES") or "0").split(",")[0]
    clocks = ClockSampler(int(vis) if vis.isdigit() else 0)
    clocks.start()
    fused_ms = timed(lambda: ops.jonker_sqeuclidean_batch(x, y), steps)
    clk = clocks.stop()
    # kernel-only: the check-mode launch through the C ABI
    lib = _loader.core()
    nbytes = lib.tm_jv_points_workspace_bytes(b, n, n)
    ws = torch.empty(nbytes, dtype=torch.uint8, device=dev)
    out = torch.empty(b, n, dtype=torch.long, device=dev)
    stream = torch.cuda.current_stream().cuda_stream

    def fused_abi():
        rc = lib.tm_jonker_sqeuclidean_batch_f32(x.data_ptr(), y.data_ptr(), b, n, n, d,
                                                 out.data_ptr(), ws.data_ptr(), nbytes, stream)
        assert rc == 0, lib.tm_status_string(rc)
    abi_ms = timed(fused_abi, steps)
    # the same problems through the dense op, cost tensor pre-built
    costs = torch.empty(b, n, n, device=dev)
    for s0 in range(0, b, 1024):
        s1 = min(b, s0 + 1024)
        costs[s0:s1] = ((x[s0:s1, :, None] - y[s0:s1, None]) ** 2).sum(-1)
    dense_ms = timed(lambda: ops.jonker_dense_batch(costs), steps)
    del costs
    # the unfused pipeline a user would run: torch builds the cost tensor
    # (cdist, squared; rounds differently, so timing only), then the dense op
    unfused_ms = timed(lambda: ops.jonker_dense_batch(torch.cdist(x, y).pow_(2)), steps)
    # end to end: pinned host points in (four pieces each, double-buffered on
    # a copy stream), mapping out to pinned memory, every step
    hb = min(b, 16384)
    hx, hy = x[:hb].cpu().pin_memory(), y[:hb].cpu().pin_memory()
    res = torch.empty(hb, n, dtype=torch.long).pin_memory()
    cs = torch.cuda.Stream(dev)
    comp = torch.cuda.current_stream(dev)
    dx = [torch.empty_like(hx, device=dev) for _ in range(2)]
    dy = [torch.empty_like(hy, device=dev) for _ in range(2)]
    ready = [torch.cuda.Event() for _ in range(2)]
    free = [torch.cuda.Event() for _ in range(2)]

    def upload(k):
        with torch.cuda.stream(cs):
            if k >= 2:
                cs.wait_event(free[k % 2])
            for src, dst in ((hx, dx[k % 2]), (hy, dy[k % 2])):
                fs, fd = src.view(-1), dst.view(-1)
                q = -(-fs.numel() // 4)
                for p0 in range(0, fs.numel(), q):
                    fd[p0:p0 + q].copy_(fs[p0:p0 + q], non_blocking=True)
            ready[k % 2].record(cs)

    def e2e_run(nsteps):
        cs.wait_stream(comp)
        upload(0)
        for k in range(nsteps):
            if k + 1 < nsteps:
                upload(k + 1)
            comp.wait_event(ready[k % 2])
            out_k = ops.jonker_sqeuclidean_batch(dx[k % 2], dy[k % 2])
            free[k % 2].record(comp)
            res.copy_(out_k, non_blocking=True)

    e2e_run(2)
    torch.cuda.synchronize()
    e_steps = max(3, steps // 2)
    q0 = torch.cuda.Event(enable_timing=True)
    q1 = torch.cuda.Event(enable_timing=True)
    q0.record(comp)
    e2e_run(e_steps)
    q1.record(comp)
    torch.cuda.synchronize()
    e2e_ms = q0.elapsed_time(q1) / e_steps
    peak, peak_src = peak_hbm()
    alg = b * (2 * n * d * 4 + n * 8)
    achieved = alg / (abi_ms / 1e3) / 1e9
    line = {
        "metric": METRIC, "value": b / (fused_ms / 1e3), "unit": UNIT, "n_gpus": 1,
        "steps": steps, "warmup": args.warmup, "ms_per_step": fused_ms,
        "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "f32",
        "data": "synthetic",
        "config": {"workload": f"config5 problems from points: fused sqeuclidean costs, "
                               f"B={b} N=M={n} D={d}, x,y~N(0,I16)",
                   "global_batch": b, "parallelism": "single GPU",
                   "l2": f"points {2 * b * n * d * 4 / 2**20:.0f} MiB, slabs "
                         f"{nbytes / 2**20:.0f} MiB (> L2)"},
        "roofline": {"bound": "hbm", "achieved": achieved, "peak": peak, "unit": "GB/s",
                     "frac": achieved / peak,
                     "traffic": int(traffic_for("c5_fused") * b / 65536)
                     if traffic_for("c5_fused") else None,
                     "kernel": "jv_batch_kernel (points, check mode)",
                     "avg_launch_us": abi_ms * 1e3, "alg_bytes_per_launch": alg,
                     "peak_source": peak_src},
        "dense_op_prebuilt_costs": {"value": b / (dense_ms / 1e3), "unit": UNIT,
                                    "ms_per_step": dense_ms,
                                    "cost_tensor_bytes": b * n * n * 4},
        "unfused_cdist_then_dense_op": {"value": b / (unfused_ms / 1e3), "unit": UNIT,
                                        "ms_per_step": unfused_ms},
        "e2e": {"value": hb / (e2e_ms / 1e3), "unit": UNIT,
                "h2d_bytes_per_step": 2 * hb * n * d * 4, "d2h_bytes_per_step": hb * n * 8,
                "problems_per_step": hb},
        "gpu_launches": steps,
        "clocks": clk,
    }
    print(json.dumps(line), flush=True)


def run_scatter(args):
    """One process, every visible GPU: the batch starts on cuda:0 and
    sharded.solve_multi_gpu peer-copies contiguous slices out over NVLink,
    solves them on their GPUs and copies the mappings back into one output on
    cuda:0, all inside the timed region (CUDA events on cuda:0's stream, which
    waits for every GPU's work).  Strong scaling: the whole batch is fixed."""
    import torch

    import torchmatch_b200  # noqa: F401
    from torchmatch_b200 import sharded

    spec = CONFIGS[args.config]
    b = args.batch or spec["B"]
    dev0 = torch.device("cuda", 0)
    torch.cuda.set_device(dev0)
    x = make_batch_device(args.config, b, 0, dev0)
    ngpu = torch.cuda.device_count()
    for _ in range(max(3, args.warmup)):
        sharded.solve_multi_gpu(x)
    for d in range(ngpu):
        torch.cuda.synchronize(d)
    steps = max(3, min(args.steps, 10))
    t0 = torch.cuda.Event(enable_timing=True)
    t1 = torch.cuda.Event(enable_timing=True)
    t0.record()
    for _ in range(steps):
        out = sharded.solve_multi_gpu(x)
    t1.record()
    for d in range(ngpu):
        torch.cuda.synchronize(d)
    ms = t0.elapsed_time(t1) / steps
    assert int(out.min()) >= -1
    print(json.dumps({
        "metric": METRIC, "value": b / (ms / 1e3), "unit": UNIT, "n_gpus": ngpu,
        "steps": steps, "warmup": max(3, args.warmup), "ms_per_step": ms,
        "higher_is_better": True, "scaling": "strong", "vs_baseline": None, "dtype": "f32",
        "data": "synthetic",
        "config": {"workload": spec["desc"], "global_batch": b,
                   "parallelism": f"single process, {ngpu} GPUs, input and output on cuda:0 "
                                  "(peer copies inside the timed region)"},
    }), flush=True)


def run_once(args):
    """Two calls of one entry point on one resident batch, nothing timed: the
    cases the committed ncu summaries under profiles/ were captured on.
    --op dense: jonker_dense_batch; async: jonker_dense_batch_async (check
    launch + gated launch); stats: the standalone statistics kernel through
    the C ABI; fused: jonker_sqeuclidean_batch on config-5 point sets."""
    import torch

    import torchmatch_b200  # noqa: F401
    from torchmatch_b200 import _loader

    dev = torch.device("cuda")
    spec = CONFIGS[args.config]
    b = args.batch or spec["B"]
    if args.op == "fused":
        g = torch.Generator(device=dev).manual_seed(1)
        px = torch.randn(b, 256, 16, device=dev, generator=g)
        py = torch.randn(b, 256, 16, device=dev, generator=g)
        for _ in range(2):
            out = torch.ops.assignment.jonker_sqeuclidean_batch(px, py)
        torch.cuda.synchronize()
        print("once fused", tuple(px.shape), tuple(out.shape))
        return
    x = make_batch_device(args.config, b, 0, dev)
    if args.op == "stats":
        lib = _loader.core()
        st = torch.zeros(lib.tm_jv_workspace_bytes() // 4, dtype=torch.int32, device=dev)
        for _ in range(2):
            rc = lib.tm_jv_stats_f32(x.data_ptr(), x.numel(), st.data_ptr(),
                                     torch.cuda.current_stream().cuda_stream)
            assert rc == 0, lib.tm_status_string(rc)
        torch.cuda.synchronize()
        print("once stats", args.config, tuple(x.shape))
        return
    for _ in range(2):
        if args.op == "async":
            out = torch.ops.assignment.jonker_dense_batch_async(x)[0]
        else:
            out = torch.ops.assignment.jonker_dense_batch(x)
    torch.cuda.synchronize()
    print("once", args.op, args.config, tuple(x.shape), tuple(out.shape))


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=50)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--config", default="c2", choices=sorted(CONFIGS))
    ap.add_argument("--impl", default="ours", choices=["ours", "reference"])
    ap.add_argument("--once", action="store_true",
                    help="solve the workload twice and exit (a small case for ncu captures)")
    ap.add_argument("--batch", type=int, default=0, help="override B (with --once / --fused)")
    ap.add_argument("--op", default="dense", choices=["dense", "async", "stats", "fused"],
                    help="entry point of --once")
    ap.add_argument("--streams", type=int, default=3,
                    help="streams of the pipelined (async op) measurement")
    ap.add_argument("--scatter", action="store_true",
                    help="one process over every visible GPU, batch scattered from cuda:0")
    ap.add_argument("--no-per-config", action="store_true",
                    help="skip the per-config records and the config-5 strong-scaling leg")
    ap.add_argument("--no-cpu", action="store_true",
                    help="skip the CPU baselines of the per-config records")
    ap.add_argument("--fused", action="store_true",
                    help="fused squared-Euclidean cost construction on config-5 point sets")
    args = ap.parse_args()
    if args.once:
        run_once(args)
    elif args.fused:
        run_fused(args)
    elif args.scatter:
        run_scatter(args)
    elif args.impl == "reference":
        run_reference(args)
    else:
        run_ours(args)


if __name__ == "__main__":
    main()
