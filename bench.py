"""Benchmark: CIM-simulation inferences/s on B200s, headline ResNet-18 at batch 1024.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--workload resnet18]
    python bench.py --impl reference ...      # the CPU reference arm

One step is one inference pass of the whole CIM-simulated network over one
batch (default: CIFAR ResNet-18, 1024 images of 3x32x32 ~ N(0,1), He-normal
weights; every Conv/Linear runs as BF16 sign-split crossbar tiles, bit-exact
with the reference simulator, the batch norms, ReLUs, residual adds and the
average pool as f32 glue). With N GPUs (torchrun, one process per GPU) each
rank runs its own batch: the work shards by batch with no collective (weak
scaling); ``value`` is the whole-job rate, timed on the device with CUDA
events and taken as the maximum over ranks.

Prints one JSON line (rank 0):
  value / ms_per_step   CUDA-graph replays of the whole network, L2 flushed
                        between steps outside the timed span.
  e2e                   the same metric through the public API (the
                        torch.compile backend, runtime="cuda") with the batch in
                        pinned host memory and the logits + status word read
                        back every step.
  roofline              the kernel with the largest share of device time, timed
                        per launch with CUDA events on its stream.
  kernels               every kernel of the step with its device time and share.
  clocks                nvidia-smi samples over a loaded window of >= 1 s (untimed
                        replays just before the timed loop, then the loop).
  configs               (N=1) the other four workloads at their own batches:
                        value, e2e, dominant kernel and its roof fraction.
  int8_sweep            (N=1) INT8 CIM MVM layers over an M x K=N grid: best TOPS
                        and the fraction of the int8 tensor peak at 8192^3.
  cpu_baseline          (N=1) the reference's CPU simulation on this host's
                        cores over a bounded sample (one core and all cores).
"""

from __future__ import annotations

import argparse
import json
import os
import platform
import statistics
import subprocess
import sys
import threading
import time
from pathlib import Path

REPO = Path(__file__).resolve().parent
sys.path[:0] = [str(REPO / "mlir-cim22_b200"), str(REPO / "oracle")]

METRIC = "CIM-sim inferences/sec"
UNIT = "inferences/s"
L2_FLUSH_BYTES = 256 << 20
L2_NOTE = "flushed between steps (256 MiB write, outside the timed span)"
REFERENCE_SECONDS = 90.0
CLOCK_WINDOW_S = 1.5
EXTRA_WORKLOADS = ("mlp", "lenet", "bf16_4x4096", "event_cnn")


def parse():
    p = argparse.ArgumentParser()
    p.add_argument("--gpus", type=int, default=1)
    p.add_argument("--steps", type=int, default=50)
    p.add_argument("--warmup", type=int, default=5)
    p.add_argument("--impl", default="ours", choices=["ours", "reference"])
    p.add_argument("--workload", default="resnet18")
    p.add_argument("--batch", type=int, default=None)
    p.add_argument("--no-cpu-baseline", action="store_true")
    p.add_argument("--no-extras", action="store_true",
                   help="skip the other workloads and the INT8 sweep (N=1 adds them by default)")
    p.add_argument("--int8-sweep", action="store_true",
                   help="only the INT8 CIM MVM sweep (M x K=N grid), one JSON row per point")
    p.add_argument("--sweep-m", default="1,16,128,1024,8192")
    p.add_argument("--sweep-kn", default="256,1024,4096,8192")
    p.add_argument("--parallel", default="batch", choices=["batch", "columns"],
                   help="batch: every rank runs its own batch (weak scaling); columns: every "
                        "Linear layer's output lanes are split over the ranks, outputs "
                        "all-gathered (strong scaling; Linear stacks such as bf16_4x4096)")
    p.add_argument("--profile", action="store_true",
                   help="only launch the program's kernels eagerly (warmup + steps passes); "
                        "for capturing single kernels under a profiler")
    return p.parse_args()


def peaks():
    path = REPO / "MEASURED_PEAKS.json"
    if path.exists():
        data = json.loads(path.read_text())
        return data["hbm_gbs"], data["bf16_tflops"], "measured"
    return 6650.0, 1590.0, "fallback"


def cpu_model() -> str:
    try:
        for line in Path("/proc/cpuinfo").read_text().splitlines():
            if line.startswith("model name"):
                return line.split(":", 1)[1].strip()
    except OSError:
        pass
    return platform.processor() or "unknown"


def bench_config(workload: str, batch: int, world: int) -> dict:
    """The workload a line measures; identical in both arms."""
    from cim22_b200 import workloads

    w = workloads.WORKLOADS[workload]
    return {"workload": f"{workload}: {w.description}", "batch_per_gpu": batch,
            "global_batch": batch * world, "parallelism": f"batch-sharded x{world}",
            "l2": L2_NOTE,
            "arithmetic": "BF16 sign-split: int8 mantissa crossbar dots, BF16 tiles, "
                          "f32 K sums; f32 glue"}


class ClockSampler:
    """nvidia-smi clocks and throttle reasons sampled every 100 ms."""

    QUERY = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
             "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
             "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, indices):
        self.indices = set(indices)
        self.rows = []
        self.proc = None

    def __enter__(self):
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", f"--query-gpu={self.QUERY}", "--format=csv,noheader,nounits",
                 "-lms", "100"], stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
            self.thread = threading.Thread(target=self._read, daemon=True)
            self.thread.start()
        except OSError:
            self.proc = None
        return self

    def _read(self):
        for line in self.proc.stdout:
            parts = [s.strip() for s in line.split(",")]
            if len(parts) >= 9:
                self.rows.append((time.perf_counter(), parts))

    def __exit__(self, *exc):
        if self.proc:
            self.proc.terminate()
            try:
                self.proc.wait(timeout=5)
            except subprocess.TimeoutExpired:
                self.proc.kill()

    def summary(self, since: float | None = None):
        rows = [r for t, r in self.rows
                if (since is None or t >= since) and r[0].isdigit() and int(r[0]) in self.indices]
        if not rows:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["unsampled"], "samples": 0}
        sm = [float(r[1]) for r in rows if r[1].replace(".", "").isdigit()]
        mx = [float(r[2]) for r in rows if r[2].replace(".", "").isdigit()]
        pw = [float(r[3]) for r in rows if r[3].replace(".", "").isdigit()]
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        reasons = sorted({n for r in rows for n, v in zip(names, r[5:9]) if v == "Active"})
        return {"sm_mhz": statistics.median(sm) if sm else None,
                "sm_max_mhz": max(mx) if mx else None, "reasons": reasons,
                "samples": len(rows), "power_w_max": max(pw) if pw else None}


def ncu_traffic(workload: str, batch: int, step: str):
    """DRAM bytes per launch (read + write) of a step's kernel from a committed
    ncu summary (profiles/traffic.json), or (None, None)."""
    try:
        table = json.loads((REPO / "profiles" / "traffic.json").read_text())
        entry = table[f"{workload}_b{batch}"]
        return entry["kernels"][step], entry["source"]
    except (OSError, KeyError, ValueError):
        return None, None


# ----------------------------------------------------------------- CPU legs


def cpu_sample_rate(workload: str, images: int, threads: int, seed: int = 0):
    """Images per second of the reference's CPU simulation of a workload over
    a sample of `images` inputs (oracle/: the tile runner driven with 40-Work
    transactions, plan reuse and weight residency; PyTorch CPU glue)."""
    import oracle
    from cim22_b200 import workloads

    model, x = workloads.build(workload, images, seed=seed)
    xs = x.numpy()
    oracle.cim_forward(model, xs[:1], threads=threads, via_runner="auto",
                       branches="reference")  # warm
    t0 = time.perf_counter()
    oracle.cim_forward(model, xs, threads=threads, via_runner="auto", branches="reference")
    dt = time.perf_counter() - t0
    return images / dt, dt


def runner_kind() -> tuple[str, str]:
    import oracle

    if oracle.reference_runner_available():
        return "reference", ("the reference's own CIMSoftwareRunner + BF16Compensation, "
                             "compiled unmodified into oracle/_ref")
    return "port", "the oracle's restated CIMSoftwareRunner"


def cpu_baseline(workload: str) -> dict:
    """One-core and all-core CPU simulation rates over bounded samples."""
    threads = os.cpu_count() or 1
    kind, what = runner_kind()
    # Size the samples from a short probe so each leg runs for about 10 s.
    probe, _ = cpu_sample_rate(workload, max(1, min(threads, 4)), threads)
    n_all = max(threads, min(4096, int(10.0 * probe)))
    rate, dt = cpu_sample_rate(workload, n_all, threads)
    n_one = max(1, min(1024, int(6.0 * probe / threads)))
    rate1, dt1 = cpu_sample_rate(workload, n_one, 1)
    return {"value": rate, "unit": UNIT, "cores": threads, "kind": kind,
            "sample": f"{n_all} {workload} images on {threads} host threads through {what} "
                      f"(40-Work transactions, plan reuse, weight residency; branch counts "
                      f"as the reference's lowering) + PyTorch CPU glue, {dt:.1f} s",
            "single_core": {"value": rate1, "unit": UNIT, "cores": 1,
                            "sample": f"{n_one} images, {dt1:.1f} s"},
            "cpu_model": cpu_model()}


def reference_arm(args) -> None:
    """The reference's CPU simulation on this host's cores, in the GPU arm's
    metric, unit and config; each step is a bounded sample of the workload."""
    rank = int(os.environ.get("RANK", "0"))
    world = int(os.environ.get("WORLD_SIZE", "1"))
    if rank != 0:
        return
    import oracle
    from cim22_b200 import workloads as wl

    threads = os.cpu_count() or 1
    kind, what = runner_kind()
    batch = args.batch or wl.WORKLOADS[args.workload].batch
    rate, _ = cpu_sample_rate(args.workload, max(1, min(threads, 4)), threads)
    per_step = int(REFERENCE_SECONDS * rate / max(1, args.steps + args.warmup))
    per_step = max(1, min(batch, per_step))
    model, x = wl.build(args.workload, per_step, seed=0)
    xs = x.numpy()
    for _ in range(args.warmup):
        oracle.cim_forward(model, xs, threads=threads, via_runner="auto", branches="reference")
    times = []
    for _ in range(args.steps):
        t0 = time.perf_counter()
        oracle.cim_forward(model, xs, threads=threads, via_runner="auto", branches="reference")
        times.append(time.perf_counter() - t0)
    total = sum(times)
    value = per_step * args.steps / total
    line = {
        "impl": "reference", "metric": METRIC, "value": value, "unit": UNIT,
        "n_gpus": world, "steps": args.steps, "warmup": args.warmup,
        "ms_per_step": 1000 * total / args.steps, "higher_is_better": True,
        "scaling": "weak", "vs_baseline": None, "dtype": "bf16", "data": "synthetic",
        "config": bench_config(args.workload, batch, world),
        "cpu_baseline": {"value": value, "unit": UNIT, "cores": threads, "kind": kind,
                         "sample": f"{per_step} images per step (of the {batch}-image batch) "
                                   f"on {threads} host threads through {what} (40-Work "
                                   "transactions, plan reuse, weight residency) + PyTorch "
                                   "CPU glue; rate per inference",
                         "cpu_model": cpu_model()},
        "e2e": {"value": value, "unit": UNIT, "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }
    print(json.dumps(line), flush=True)


# ----------------------------------------------------------------- INT8 sweep


def layer_launch(layer, x, out, m, ws, status):
    import ctypes

    import torch

    from cim22_b200.native import check, lib

    buf = ws.get(layer.workspace_bytes(m))
    check(lib().cim22_cuda_layer_forward_int8(
        layer._handle, ctypes.c_void_p(x.data_ptr()), m, ctypes.c_void_p(out.data_ptr()),
        ctypes.c_void_p(buf.data_ptr()), buf.numel(), ctypes.c_void_p(status.tensor.data_ptr()),
        ctypes.c_void_p(torch.cuda.current_stream().cuda_stream)), "forward_int8")


def int8_sweep(ms, kns, iters: int, dev, flush, emit=None) -> dict:
    """INT8 CIM MVM layers y = x W^T (int8 x int8 -> int32, exact), each point
    timed per launch with CUDA events on the current stream (median), L2
    flushed in between."""
    import numpy as np
    import torch

    from cim22_b200.cim_ops import CimLayer, StatusWord, Workspace
    from cim22_b200.native import lib

    _, bf16_peak, peak_kind = peaks()
    int8_peak = 2 * bf16_peak
    ws, status = Workspace(dev), StatusWord(dev)
    stream = torch.cuda.current_stream(dev)
    rng = np.random.default_rng(1)
    rows = []
    for kn in kns:
        w = rng.integers(-127, 128, (kn, kn)).astype(np.int8)
        layer = CimLayer(w, kind="int8", device=dev)
        for m in ms:
            x = torch.from_numpy(np.random.default_rng(0).integers(-128, 128, (m, kn))
                                 .astype(np.int8)).to(dev)
            out = torch.empty(m, kn, dtype=torch.int32, device=dev)
            tc0 = lib().cim22_cuda_tensor_core_launches()
            for _ in range(3):
                layer_launch(layer, x, out, m, ws, status)
            times = []
            for _ in range(iters):
                flush.zero_()
                a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
                a.record(stream)
                layer_launch(layer, x, out, m, ws, status)
                b.record(stream)
                b.synchronize()
                times.append(a.elapsed_time(b))
            status.raise_if_set()
            tc = lib().cim22_cuda_tensor_core_launches() - tc0
            ms_ = sorted(times)[len(times) // 2]
            tops = 2.0 * m * kn * kn / (ms_ / 1e3) / 1e12
            row = {"m": m, "k": kn, "n": kn, "ms": round(ms_, 5), "tops": round(tops, 2),
                   "frac_int8_peak": round(tops / int8_peak, 4), "tensor_core": tc > 0}
            rows.append(row)
            if emit:
                emit(row)
        del layer
    best = max(rows, key=lambda r: r["tops"])
    top = next((r for r in rows if r["m"] == 8192 and r["k"] == 8192), None)
    return {"grid": {"m": list(ms), "k=n": list(kns)}, "points": rows, "best": best,
            "frac_at_8192_cubed": top["frac_int8_peak"] if top else None,
            "int8_peak_tops": int8_peak,
            "peak_note": f"derived int8 peak = 2 x {peak_kind} bf16 cuBLAS burst ({bf16_peak} "
                         "TF/s); no int8 GEMM peak is measured on this pool",
            "method": f"median of {iters} launches per point, L2 flushed between launches"}


# ----------------------------------------------------------------- GPU arm


def step_names(prog) -> list[str]:
    names, seen = [], {}
    for s in prog.steps:
        seen[s.name] = seen.get(s.name, 0) + 1
        names.append(s.name if seen[s.name] == 1 else f"{s.name}#{seen[s.name]}")
    return names


def kernel_times(prog, dev, flush, iters: int) -> dict:
    """Per-step device time (eager launches, one CUDA event pair per step on
    the current stream, L2 flushed before each pass), averaged over iters."""
    import torch

    stream = torch.cuda.current_stream(dev)
    names = step_names(prog)
    per = {n: [] for n in names}
    for _ in range(iters):
        flush.zero_()
        prog.status.reset()
        evs = []
        for n, step in zip(names, prog.steps):
            a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            a.record(stream)
            step.fn()
            b.record(stream)
            evs.append((n, a, b))
        torch.cuda.synchronize(dev)
        for n, a, b in evs:
            per[n].append(a.elapsed_time(b))
    prog.check_status()
    return {n: sum(v) / len(v) for n, v in per.items()}


def roofline(prog, workload: str, batch: int, avg: dict) -> dict:
    """Both roofs of the dominant step: int8 MMA work on the (derived) int8
    tensor peak and its algorithmic bytes on the measured HBM copy bandwidth;
    `bound` names the one with the larger fraction."""
    names = step_names(prog)
    dominant = max(avg, key=avg.get)
    step = prog.steps[names.index(dominant)]
    info = next((l for l in prog.layers if dominant.split("#")[0] == l.name
                 or dominant.startswith(l.name + ".")), None)
    hbm_peak, bf16_peak, peak_kind = peaks()
    int8_peak = 2 * bf16_peak
    dur_s = avg[dominant] / 1000
    tensor = hbm = None
    if step.cim and step.meta and step.meta.get("kind") == "chain":
        ops = 2 * prog.macs
        nbytes = (4 * step.meta["x"].numel() + 4 * step.meta["out"].numel()
                  + sum(2 * l.n * l.k for l in prog.layers))
        what = ("whole-network chain: ops = 2 x MACs of every layer; bytes = input batch "
                "+ logits + int8 weights of both signs")
        tensor, hbm = ops, nbytes
    elif step.cim and info is not None:
        ops = 2 * info.macs
        ab = 1 if info.branches == 2 else 2
        t_tiles = -(-info.k // 64)
        m_pad = -(-info.m // 128) * 128
        eb = info.operand_bytes
        kind = "BF16 operand" if eb == 2 else "int8"
        if step.meta.get("x") is not None and dominant.split("#")[0] + ".prepare" in names:
            # The contraction of a two-kernel layer reads the prepared columns
            # and their group exponents, not the source image.
            src = ab * m_pad * t_tiles * (64 * eb + 4)
            what = ("CIM contraction: ops = 2 x branches x M x K x N (unpadded); bytes = "
                    f"prepared {kind} columns + group exponents + {kind} weights of both signs "
                    "+ f32 output (+ f32 residual addend)")
        else:
            src = info.in_bytes
            what = ("CIM layer: ops = 2 x branches x M x K x N (unpadded); bytes = source read "
                    f"once + {kind} weights of both signs + f32 output (+ f32 residual addend)")
        nbytes = src + 2 * eb * info.n * info.k + 4 * info.m * info.n
        if step.meta.get("residual") is not None:
            nbytes += 4 * info.m * info.n
        tensor, hbm = ops, nbytes
    elif info is not None and dominant.endswith(".prepare"):
        ab = 1 if info.branches == 2 else 2
        t_tiles = -(-info.k // 64)
        m_pad = -(-info.m // 128) * 128
        hbm = info.in_bytes + ab * m_pad * t_tiles * (64 * info.operand_bytes + 4)
        what = ("prepare: bytes = source read once + prepared "
                f"{'BF16 operand' if info.operand_bytes == 2 else 'int8'} columns and group "
                "exponents written")
    else:
        what = "glue kernel (bytes not modelled)"
    roofs = []
    if tensor is not None:
        a = tensor / dur_s / 1e12
        roofs.append({"bound": "tensor", "achieved": a, "peak": int8_peak, "unit": "TFLOP/s",
                      "frac": a / int8_peak, "ops_per_launch": tensor,
                      "peak_note": f"derived int8 dense peak = 2 x {peak_kind} bf16 cuBLAS "
                                   f"burst ({bf16_peak} TF/s), of measured"})
    if hbm is not None:
        a = hbm / dur_s / 1e9
        roofs.append({"bound": "hbm", "achieved": a, "peak": hbm_peak, "unit": "GB/s",
                      "frac": a / hbm_peak, "bytes_per_launch": hbm,
                      "peak_note": f"{peak_kind} HBM copy bandwidth"})
    if not roofs:
        roofs.append({"bound": "hbm", "achieved": None, "peak": hbm_peak, "unit": "GB/s",
                      "frac": None, "peak_note": f"{peak_kind} HBM copy bandwidth"})
    roofs.sort(key=lambda r: -(r["frac"] or 0))
    roof = dict(roofs[0], kernel=dominant, launch_ms=avg[dominant], work=what)
    if len(roofs) > 1:
        roof["other_roof"] = {k: roofs[1][k] for k in ("bound", "achieved", "peak", "unit",
                                                       "frac")}
    roof["traffic"], roof["traffic_source"] = ncu_traffic(workload, batch, dominant)
    return roof


def run_workload(name: str, batch: int, *, world: int, rank: int, local: int, dev, flush,
                 steps: int, warmup: int, clock_window: bool, barrier, reduce_max):
    """Build, time and e2e-time one workload. Returns a dict of results."""
    import torch

    from cim22_b200 import backend, program, workloads

    model, _ = workloads.build(name, batch, seed=0)
    _, x = workloads.build(name, batch, seed=1000 + rank)  # per-rank batch
    prog = program.from_module(model, x, device=local, name=name)
    prog.inputs[0].tensor.copy_(x.to(dev))
    prog.capture()
    stream = torch.cuda.current_stream(dev)

    for _ in range(warmup):
        flush.zero_()
        prog.replay()
    prog.check_status()
    barrier()

    starts = [torch.cuda.Event(enable_timing=True) for _ in range(steps)]
    ends = [torch.cuda.Event(enable_timing=True) for _ in range(steps)]
    clocks = None
    with ClockSampler([local] if world == 1 else range(world)) as sampler:
        if clock_window:
            # Untimed replays so the clock record covers a loaded window of at
            # least CLOCK_WINDOW_S before and through the timed loop.
            t_load = time.perf_counter()
            while time.perf_counter() - t_load < CLOCK_WINDOW_S:
                for _ in range(8):
                    flush.zero_()
                    prog.replay()
                torch.cuda.synchronize(dev)
        barrier()
        for i in range(steps):
            flush.zero_()  # L2 flush between steps, outside the timed span
            starts[i].record(stream)
            prog.replay()
            ends[i].record(stream)
        barrier()
        time.sleep(0.25 if clock_window else 0.0)
        if clock_window:
            clocks = sampler.summary(since=t_load)
    prog.check_status()
    elapsed_ms = reduce_max(sum(s.elapsed_time(e) for s, e in zip(starts, ends)))
    value = world * batch * steps / (elapsed_ms / 1000)

    avg = kernel_times(prog, dev, flush, max(3, min(steps, 10)))
    total_kernel = sum(avg.values())
    roof = roofline(prog, name, batch, avg)

    # End to end through the public API (torch.compile, runtime="cuda").
    bname = backend.register()
    torch._dynamo.reset()
    compiled = torch.compile(model, backend=bname, fullgraph=True, dynamic=False,
                             options={"runtime": "cuda", "device": local,
                                      "chain": prog.chained})
    host = x.pin_memory()
    with torch.inference_mode():
        out = compiled(host)
        for _ in range(warmup):
            out = compiled(host)
        barrier()
        e_ms = 0.0
        for _ in range(steps):
            flush.zero_()
            a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            a.record(stream)
            out = compiled(host)
            b.record(stream)
            b.synchronize()
            e_ms += a.elapsed_time(b)
        barrier()
    e_ms = reduce_max(e_ms)
    e2e_value = world * batch * steps / (e_ms / 1000)
    h2d = host.numel() * host.element_size()
    d2h = out.numel() * out.element_size() + 4  # outputs + status word
    return {
        "value": value, "ms_per_step": elapsed_ms / steps, "macs_per_batch": prog.macs,
        "gpu_launches": len(prog.steps) * steps,
        "lowering": "fused layer chain (one persistent kernel)" if prog.chained
                    else f"{len(prog.steps)} kernels per step (CUDA graph)",
        "e2e": {"value": e2e_value, "unit": UNIT, "h2d_bytes_per_step": h2d,
                "d2h_bytes_per_step": d2h},
        "roofline": roof,
        "kernels": {n: {"ms": round(v, 5), "share": round(v / total_kernel, 4)}
                    for n, v in avg.items()},
        "clocks": clocks,
    }


def column_bench(args, world: int, rank: int, local: int, dev) -> None:
    """Column-sharded Linear stack: every rank computes 1/world of each layer's
    lanes for all rows; outputs are all-gathered over NCCL. One step = one
    forward of the whole batch; value = rows per second for the whole job."""
    import torch
    import torch.distributed as dist

    from cim22_b200 import workloads
    from cim22_b200.sharding import ColumnShardedStack

    w = workloads.WORKLOADS[args.workload]
    rows = args.batch or w.batch
    model, x = workloads.build(args.workload, rows, seed=0)
    if args.workload != "bf16_4x4096":
        raise SystemExit("--parallel columns is defined for the bf16_4x4096 Linear stack")
    linears = [m for m in model.modules() if isinstance(m, torch.nn.Linear)]
    acts = ["gelu"] * (len(linears) - 1) + [None]  # GELU between the layers
    weights = [l.weight.detach() for l in linears]
    biases = [None if l.bias is None else l.bias.detach() for l in linears]
    try:
        # Peer stores in the contraction epilogue + a device barrier per layer
        # (every rank's lane block takes BF16 operands).
        stack = ColumnShardedStack(weights, biases, acts, rows, device=local, fused=True)
        exchange = "each rank's lanes stored into every rank's output by the contraction " \
                   "epilogue over NVLink (CUDA IPC), device barrier per layer"
    except ValueError:
        stack = ColumnShardedStack(weights, biases, acts, rows, device=local)
        exchange = "NCCL all-gather per layer"
    xd = x.to(dev)
    stream = torch.cuda.current_stream(dev)

    def barrier():
        torch.cuda.synchronize(dev)
        if world > 1:
            dist.barrier()

    for _ in range(args.warmup):
        stack(xd)
    stack.check_status()
    barrier()
    flush = torch.empty(L2_FLUSH_BYTES, dtype=torch.uint8, device=dev)
    starts = [torch.cuda.Event(enable_timing=True) for _ in range(args.steps)]
    ends = [torch.cuda.Event(enable_timing=True) for _ in range(args.steps)]
    with ClockSampler([local] if world == 1 else range(world)) as clocks:
        t_load = time.perf_counter()
        while time.perf_counter() - t_load < CLOCK_WINDOW_S:
            for _ in range(8):
                flush.zero_()
                stack(xd)
            torch.cuda.synchronize(dev)
        barrier()
        for i in range(args.steps):
            flush.zero_()
            starts[i].record(stream)
            stack(xd)
            ends[i].record(stream)
        barrier()
        time.sleep(0.25)
    stack.check_status()
    t = torch.tensor([sum(a.elapsed_time(b) for a, b in zip(starts, ends))], device=dev,
                     dtype=torch.float64)
    if world > 1:
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
    elapsed_ms = float(t.item())
    value = rows * args.steps / (elapsed_ms / 1000)

    # End to end: rows from pinned host memory, the output read back each step.
    host = x.pin_memory()
    out = torch.empty(stack(xd).shape, dtype=torch.float32, pin_memory=True)
    e_ms = 0.0
    barrier()
    for _ in range(args.steps):
        flush.zero_()
        a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        a.record(stream)
        out.copy_(stack(host.to(dev, non_blocking=True)), non_blocking=True)
        b.record(stream)
        b.synchronize()
        e_ms += a.elapsed_time(b)
    stack.check_status()
    et = torch.tensor([e_ms], device=dev, dtype=torch.float64)
    if world > 1:
        dist.all_reduce(et, op=dist.ReduceOp.MAX)
    e2e_value = rows * args.steps / (float(et.item()) / 1000)

    # Per-rank contraction of the first layer, timed alone (tensor roofline).
    layer = stack.layers[0]
    per = []
    for _ in range(5):
        a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        layer.prepare_bf16(xd, rows, branches=4, workspace=stack.workspace, status=stack.status)
        a.record(stream)
        layer.contract_bf16(stack.local[0], rows, activation="gelu", branches=4,
                            workspace=stack.workspace, status=stack.status)
        b.record(stream)
        torch.cuda.synchronize(dev)
        per.append(a.elapsed_time(b))
    stack.check_status()
    launch_ms = sorted(per)[len(per) // 2]
    ops = 2 * 4 * rows * layer.k * stack.plans[0].block
    hbm_peak, bf16_peak, peak_kind = peaks()
    achieved = ops / (launch_ms / 1000) / 1e12
    if rank == 0:
        line = {
            "metric": METRIC, "value": value, "unit": UNIT, "n_gpus": world,
            "steps": args.steps, "warmup": args.warmup,
            "ms_per_step": elapsed_ms / args.steps, "higher_is_better": True,
            "scaling": "strong", "vs_baseline": None, "dtype": "bf16", "data": "synthetic",
            "config": {"workload": f"{args.workload}: {w.description}", "global_batch": rows,
                       "parallelism": f"column-sharded x{world} (lanes split; {exchange})",
                       "l2": L2_NOTE},
            "gpu_launches": 3 * len(stack.layers) * args.steps,
            "e2e": {"value": e2e_value, "unit": UNIT,
                    "h2d_bytes_per_step": host.numel() * host.element_size(),
                    "d2h_bytes_per_step": out.numel() * out.element_size()},
            "roofline": {"bound": "tensor", "achieved": achieved, "peak": 2 * bf16_peak,
                         "unit": "TFLOP/s", "frac": achieved / (2 * bf16_peak), "traffic": None,
                         "kernel": "linear0 (local lanes)", "launch_ms": launch_ms,
                         "peak_note": f"derived int8 dense peak = 2 x {peak_kind} bf16 "
                                      "cuBLAS burst"},
            "cpu_baseline": None,
            "clocks": clocks.summary(since=t_load),
        }
        print(json.dumps(line), flush=True)
    stack.close()
    if world > 1:
        dist.barrier()
        dist.destroy_process_group()


def main() -> None:
    args = parse()
    if args.impl == "reference":
        reference_arm(args)
        return

    import torch
    import torch.distributed as dist

    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    flush = torch.empty(L2_FLUSH_BYTES, dtype=torch.uint8, device=dev)

    if args.int8_sweep:
        int8_sweep([int(v) for v in args.sweep_m.split(",")],
                   [int(v) for v in args.sweep_kn.split(",")], max(3, min(args.steps, 20)),
                   dev, flush, emit=lambda r: print(json.dumps(r), flush=True))
        return
    if world > 1:
        from datetime import timedelta

        dist.init_process_group("nccl", timeout=timedelta(seconds=120), device_id=dev)

    if args.parallel == "columns":
        column_bench(args, world, rank, local, dev)
        return

    from cim22_b200 import program, workloads

    batch = args.batch or workloads.WORKLOADS[args.workload].batch
    if args.profile:
        model, x = workloads.build(args.workload, batch, seed=0)
        prog = program.from_module(model, x, device=local, name=args.workload)
        prog.inputs[0].tensor.copy_(x.to(dev))
        for _ in range(args.warmup + args.steps):
            prog.status.reset()
            prog.launch()
        torch.cuda.synchronize(dev)
        prog.check_status()
        print(json.dumps({"profile": args.workload, "passes": args.warmup + args.steps,
                          "kernels": [s.name for s in prog.steps]}))
        return

    def barrier():
        torch.cuda.synchronize(dev)
        if world > 1:
            dist.barrier()

    def reduce_max(v: float) -> float:
        t = torch.tensor([v], device=dev, dtype=torch.float64)
        if world > 1:
            dist.all_reduce(t, op=dist.ReduceOp.MAX)
        return float(t.item())

    head = run_workload(args.workload, batch, world=world, rank=rank, local=local, dev=dev,
                        flush=flush, steps=args.steps, warmup=args.warmup, clock_window=True,
                        barrier=barrier, reduce_max=reduce_max)

    extras = sweep = cpu = None
    if world == 1 and not args.no_extras:
        extras = {}
        for name in EXTRA_WORKLOADS:
            if name == args.workload:
                continue
            b = workloads.WORKLOADS[name].batch
            r = run_workload(name, b, world=1, rank=0, local=local, dev=dev, flush=flush,
                             steps=max(args.steps, 20), warmup=args.warmup, clock_window=False,
                             barrier=barrier, reduce_max=reduce_max)
            roof = r["roofline"]
            extras[name] = {
                "config": bench_config(name, b, 1), "value": r["value"], "unit": UNIT,
                "ms_per_step": r["ms_per_step"], "e2e": r["e2e"], "lowering": r["lowering"],
                "dominant_kernel": roof["kernel"], "dominant_ms": roof["launch_ms"],
                "dominant_share": r["kernels"][roof["kernel"]]["share"],
                "roofline": {k: roof.get(k) for k in ("bound", "achieved", "unit", "frac",
                                                       "peak", "other_roof")},
                "macs_per_batch": r["macs_per_batch"],
            }
        sweep = int8_sweep([1, 16, 128, 1024, 8192], [256, 1024, 4096, 8192], 10, dev, flush)
        sweep.pop("points")
    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        cpu = cpu_baseline(args.workload)

    if rank == 0:
        line = {
            "metric": METRIC, "value": head["value"], "unit": UNIT, "n_gpus": world,
            "steps": args.steps, "warmup": args.warmup, "ms_per_step": head["ms_per_step"],
            "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "bf16",
            "data": "synthetic", "config": bench_config(args.workload, batch, world),
            "graph": "CUDA graph replay of the whole network per step",
            "lowering": head["lowering"], "cim_macs_per_batch": head["macs_per_batch"],
            "gpu_launches": head["gpu_launches"], "e2e": head["e2e"],
            "roofline": head["roofline"], "kernels": head["kernels"],
            "cpu_baseline": cpu, "clocks": head["clocks"],
        }
        if extras is not None:
            line["configs"] = extras
        if sweep is not None:
            line["int8_sweep"] = sweep
        print(json.dumps(line), flush=True)
    if world > 1:
        dist.barrier()
        dist.destroy_process_group()


if __name__ == "__main__":
    main()
