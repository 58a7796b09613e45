"""Benchmark: CIM-simulation inferences/s of the LeNet workload on B200s.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--workload lenet]
    python bench.py --impl reference ...      # the CPU reference arm

One step is one inference pass of the whole CIM-simulated network over one
batch (LeNet: 256 images of 1x32x32, U[0,1], He-normal weights; every
Linear/Conv runs as BF16 sign-split crossbar tiles, bit-exact with the
reference simulator). With N GPUs (torchrun, one process per GPU) each rank
runs its own batch: the work shards by batch with no collective (weak
scaling); ``value`` is the whole-job rate, timed on the device with CUDA
events and taken as the maximum over ranks.

Prints one JSON line (rank 0). ``e2e`` is the same metric through the public
API (the torch.compile backend, runtime="cuda") with the batch in pinned host
memory and the logits read back every step. ``roofline`` covers the kernel
with the largest share of device time, timed per launch with CUDA events on
its stream. ``cpu_baseline`` is the oracle port of the reference's software
runner (oracle/), run on this host's cores over a bounded sample.
"""

from __future__ import annotations

import argparse
import json
import os
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
REFERENCE_SECONDS = 90.0


def parse():
    p = argparse.ArgumentParser()
    p.add_argument("--gpus", type=int, default=1)
    p.add_argument("--steps", type=int, default=3000)
    p.add_argument("--warmup", type=int, default=20)
    p.add_argument("--impl", default="ours", choices=["ours", "reference"])
    p.add_argument("--workload", default="lenet")
    p.add_argument("--batch", type=int, default=None)
    p.add_argument("--cpu-sample", type=int, default=2048,
                   help="images in the CPU baseline sample")
    p.add_argument("--no-cpu-baseline", action="store_true")
    p.add_argument("--int8-sweep", action="store_true",
                   help="INT8 CIM MVM sweep (M x K=N grid): TOPS vs the int8 tensor peak")
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


class ClockSampler:
    """nvidia-smi clocks and throttle reasons sampled during the timed region."""

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
                 "-lms", "200"], stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
            self.thread = threading.Thread(target=self._read, daemon=True)
            self.thread.start()
        except OSError:
            self.proc = None
        return self

    def _read(self):
        for line in self.proc.stdout:
            parts = [s.strip() for s in line.split(",")]
            if len(parts) >= 9:
                self.rows.append(parts)

    def __exit__(self, *exc):
        if self.proc:
            self.proc.terminate()
            try:
                self.proc.wait(timeout=5)
            except subprocess.TimeoutExpired:
                self.proc.kill()

    def summary(self):
        rows = [r for r in self.rows if r[0].isdigit() and int(r[0]) in self.indices]
        if not rows:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["unsampled"]}
        sm = [float(r[1]) for r in rows if r[1].replace(".", "").isdigit()]
        mx = [float(r[2]) for r in rows if r[2].replace(".", "").isdigit()]
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        reasons = sorted({n for r in rows for n, v in zip(names, r[5:9]) if v == "Active"})
        return {"sm_mhz": statistics.median(sm) if sm else None,
                "sm_max_mhz": max(mx) if mx else None, "reasons": reasons,
                "samples": len(rows)}


def ncu_traffic(workload: str, batch: int, step: str):
    """DRAM bytes per launch (read + write) of a step's kernel from a committed
    ncu launch-list summary (profiles/traffic.json), or (None, None)."""
    try:
        table = json.loads((REPO / "profiles" / "traffic.json").read_text())
        entry = table[f"{workload}_b{batch}"]
        return entry["kernels"][step], entry["source"]
    except (OSError, KeyError, ValueError):
        return None, None


def cpu_baseline(workload: str, sample: int, threads: int, batch_seed: int = 0):
    """Oracle port of the reference's software runner on host cores."""
    import oracle
    from cim22_b200 import workloads

    model, x = workloads.build(workload, sample, seed=batch_seed)
    oracle.cim_forward(model, x[:2].numpy(), threads=threads, via_runner=True)  # warm
    t0 = time.perf_counter()
    oracle.cim_forward(model, x.numpy(), threads=threads, via_runner=True)
    dt = time.perf_counter() - t0
    return sample / dt, dt


def reference_arm(args) -> None:
    rank = int(os.environ.get("RANK", "0"))
    if rank != 0:
        return
    import oracle
    from cim22_b200 import workloads as wl

    threads = os.cpu_count() or 1
    # Size each step's sample so the whole run takes about REFERENCE_SECONDS.
    rate, _ = cpu_baseline(args.workload, 2 * threads, threads)
    per_step = int(REFERENCE_SECONDS * rate / max(1, args.steps + args.warmup))
    per_step = max(1, min(args.cpu_sample, 256, per_step))
    model, x = wl.build(args.workload, per_step, seed=0)
    xs = x.numpy()
    for _ in range(args.warmup):
        oracle.cim_forward(model, xs, threads=threads, via_runner=True)
    times = []
    for _ in range(args.steps):
        t0 = time.perf_counter()
        oracle.cim_forward(model, xs, threads=threads, via_runner=True)
        times.append(time.perf_counter() - t0)
    total = sum(times)
    value = per_step * args.steps / total
    from cim22_b200 import workloads

    w = workloads.WORKLOADS[args.workload]
    line = {
        "impl": "reference", "metric": METRIC, "value": value, "unit": UNIT,
        "n_gpus": args.gpus, "steps": args.steps, "warmup": args.warmup,
        "ms_per_step": 1000 * total / args.steps, "higher_is_better": True,
        "scaling": "weak", "vs_baseline": None, "dtype": "bf16", "data": "synthetic",
        "config": {"workload": f"{args.workload}: {w.description}",
                   "batch_per_step": per_step, "parallelism": "host threads over columns"},
        "cpu_baseline": {"value": value, "unit": UNIT, "cores": threads, "kind": "port",
                         "sample": f"{per_step} images per step through the oracle's "
                                   "restated CIMSoftwareRunner (40-Work transactions, plan "
                                   "reuse, weight residency) + PyTorch CPU glue"},
        "e2e": {"value": value, "unit": UNIT, "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }
    print(json.dumps(line), flush=True)


def int8_sweep(args) -> None:
    """INT8 CIM MVM layers y = x W^T (int8 x int8 -> int32, exact), timed per
    launch with CUDA events on the current stream, L2 flushed in between."""
    import numpy as np
    import torch

    from cim22_b200.cim_ops import CimLayer, StatusWord, Workspace
    from cim22_b200.native import lib

    dev = torch.device("cuda", 0)
    torch.cuda.set_device(dev)
    _, bf16_peak, peak_kind = peaks()
    int8_peak = 2 * bf16_peak
    flush = torch.empty(L2_FLUSH_BYTES, dtype=torch.uint8, device=dev)
    ws, status = Workspace(dev), StatusWord(dev)
    stream = torch.cuda.current_stream(dev)
    rng = np.random.default_rng(1)
    rows = []
    for kn in [int(v) for v in args.sweep_kn.split(",")]:
        w = rng.integers(-127, 128, (kn, kn)).astype(np.int8)
        layer = CimLayer(w, kind="int8", device=dev)
        for m in [int(v) for v in args.sweep_m.split(",")]:
            x = torch.from_numpy(np.random.default_rng(0).integers(-128, 128, (m, kn))
                                 .astype(np.int8)).to(dev)
            out = torch.empty(m, kn, dtype=torch.int32, device=dev)
            tc0 = lib().cim22_cuda_tensor_core_launches()
            for _ in range(3):
                layer_launch(layer, x, out, m, ws, status)
            times = []
            for _ in range(max(3, min(args.steps, 20))):
                flush.zero_()
                a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
                a.record(stream)
                layer_launch(layer, x, out, m, ws, status)
                b.record(stream)
                b.synchronize()
                times.append(a.elapsed_time(b))
            status.raise_if_set()
            tc = lib().cim22_cuda_tensor_core_launches() - tc0
            ms = sorted(times)[len(times) // 2]
            tops = 2.0 * m * kn * kn / (ms / 1e3) / 1e12
            row = {"m": m, "k": kn, "n": kn, "ms": ms, "tops": tops,
                   "frac_int8_peak": tops / int8_peak, "tensor_core": tc > 0}
            rows.append(row)
            print(json.dumps(row), flush=True)
    best = max(rows, key=lambda r: r["tops"])
    print(json.dumps({"metric": "int8 CIM MVM TOPS", "best": best,
                      "int8_peak_tops": int8_peak,
                      "peak_note": f"2 x {peak_kind} bf16 cuBLAS ({bf16_peak} TF/s)"}), flush=True)


def layer_launch(layer, x, out, m, ws, status):
    import ctypes

    import torch

    from cim22_b200.native import check, lib

    buf = ws.get(layer.workspace_bytes(m))
    check(lib().cim22_cuda_layer_forward_int8(
        layer._handle, ctypes.c_void_p(x.data_ptr()), m, ctypes.c_void_p(out.data_ptr()),
        ctypes.c_void_p(buf.data_ptr()), buf.numel(), ctypes.c_void_p(status.tensor.data_ptr()),
        ctypes.c_void_p(torch.cuda.current_stream().cuda_stream)), "forward_int8")


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
    stack = ColumnShardedStack([l.weight.detach() for l in linears],
                               [None if l.bias is None else l.bias.detach() for l in linears],
                               acts, rows, device=local)
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
        barrier()
        for i in range(args.steps):
            flush.zero_()
            starts[i].record(stream)
            stack(xd)
            ends[i].record(stream)
        barrier()
    stack.check_status()
    t = torch.tensor([sum(a.elapsed_time(b) for a, b in zip(starts, ends))], device=dev,
                     dtype=torch.float64)
    if world > 1:
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
    elapsed_ms = float(t.item())
    value = rows * args.steps / (elapsed_ms / 1000)

    # End to end: rows from pinned host memory, the output read back each step.
    host = x.pin_memory()
    e_ms = 0.0
    out = None
    barrier()
    for _ in range(args.steps):
        flush.zero_()
        a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        a.record(stream)
        out = stack(host.to(dev, non_blocking=True)).cpu()
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
                       "parallelism": f"column-sharded x{world} (lanes split, NCCL all-gather "
                                      f"per layer)",
                       "l2": "flushed between steps (256 MiB write, outside the timed span)",
                       "graph": "eager launches"},
            "gpu_launches": 3 * len(stack.layers) * args.steps,
            "e2e": {"value": e2e_value, "unit": UNIT,
                    "h2d_bytes_per_step": host.numel() * host.element_size(),
                    "d2h_bytes_per_step": out.numel() * out.element_size()},
            "roofline": {"bound": "tensor", "achieved": achieved, "peak": 2 * bf16_peak,
                         "unit": "TFLOP/s", "frac": achieved / (2 * bf16_peak), "traffic": None,
                         "kernel": "linear0 (local lanes)", "launch_ms": launch_ms,
                         "peak_note": f"int8 dense = 2 x {peak_kind} bf16 cuBLAS"},
            "cpu_baseline": None,
            "clocks": clocks.summary(),
        }
        print(json.dumps(line), flush=True)
    if world > 1:
        dist.barrier()
        dist.destroy_process_group()


def main() -> None:
    args = parse()
    if args.impl == "reference":
        reference_arm(args)
        return
    if args.int8_sweep:
        int8_sweep(args)
        return

    import torch
    import torch.distributed as dist

    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    if world > 1:
        from datetime import timedelta

        dist.init_process_group("nccl", timeout=timedelta(seconds=120), device_id=dev)

    from cim22_b200 import backend, program, workloads

    if args.parallel == "columns":
        column_bench(args, world, rank, local, dev)
        return

    w = workloads.WORKLOADS[args.workload]
    batch = args.batch or w.batch
    model, x = workloads.build(args.workload, batch, seed=0)
    _, x = workloads.build(args.workload, batch, seed=1000 + rank)  # per-rank batch

    prog = program.from_module(model, x, device=local, name=args.workload)
    prog.inputs[0].tensor.copy_(x.to(dev))
    if args.profile:
        for _ in range(args.warmup + args.steps):
            prog.status.reset()
            prog.launch()
        torch.cuda.synchronize(dev)
        prog.check_status()
        print(json.dumps({"profile": args.workload, "passes": args.warmup + args.steps,
                          "kernels": [s.name for s in prog.steps]}))
        return
    prog.capture()
    flush = torch.empty(L2_FLUSH_BYTES, dtype=torch.uint8, device=dev)

    def barrier():
        torch.cuda.synchronize(dev)
        if world > 1:
            dist.barrier()

    # Warm-up.
    for _ in range(args.warmup):
        flush.zero_()
        prog.replay()
    prog.check_status()
    barrier()

    stream = torch.cuda.current_stream(dev)
    starts = [torch.cuda.Event(enable_timing=True) for _ in range(args.steps)]
    ends = [torch.cuda.Event(enable_timing=True) for _ in range(args.steps)]
    with ClockSampler([local] if world == 1 else range(world)) as clocks:
        barrier()
        for i in range(args.steps):
            flush.zero_()  # L2 flush between steps, outside the timed span
            starts[i].record(stream)
            prog.replay()
            ends[i].record(stream)
        barrier()
    prog.check_status()
    elapsed_ms = sum(s.elapsed_time(e) for s, e in zip(starts, ends))
    t = torch.tensor([elapsed_ms], device=dev, dtype=torch.float64)
    if world > 1:
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
    elapsed_ms = float(t.item())
    value = world * batch * args.steps / (elapsed_ms / 1000)

    # Per-kernel device time (eager launches, one event pair per kernel);
    # repeated glue names get an ordinal ("add", "add#2", ...).
    names, seen = [], {}
    for s in prog.steps:
        seen[s.name] = seen.get(s.name, 0) + 1
        names.append(s.name if seen[s.name] == 1 else f"{s.name}#{seen[s.name]}")
    per = {n: [] for n in names}
    kernel_iters = max(3, min(args.steps, 20))
    for _ in range(kernel_iters):
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
    avg = {n: sum(v) / len(v) for n, v in per.items()}
    total_kernel = sum(avg.values())
    dominant = max(avg, key=avg.get)
    hbm_peak, bf16_peak, peak_kind = peaks()
    step = prog.steps[names.index(dominant)]
    info = next((l for l in prog.layers if dominant.startswith(l.name)), None)
    dur_s = avg[dominant] / 1000
    if step.cim and step.meta and step.meta.get("kind") == "chain":
        # The whole network in one kernel: the MMA-equivalent work of every
        # layer on the int8 tensor peak (the chain computes it with dp4a on
        # CUDA cores), and on HBM the input images, the logits and each
        # layer's int8 weights of both signs.
        ops = 2 * prog.macs
        achieved = ops / dur_s / 1e12
        int8_peak = 2 * bf16_peak
        chain_bytes = (4 * step.meta["x"].numel() + 4 * step.meta["out"].numel()
                       + sum(2 * l.n * l.k for l in prog.layers))
        gbs = chain_bytes / dur_s / 1e9
        tensor = {"bound": "tensor", "achieved": achieved, "peak": int8_peak, "unit": "TFLOP/s",
                  "frac": achieved / int8_peak, "ops_per_launch": ops,
                  "peak_note": f"int8 dense = 2 x {peak_kind} bf16 cuBLAS ({bf16_peak} TF/s); "
                               "ops = 2 x branches x M x K x N of every layer (unpadded)"}
        hbm = {"bound": "hbm", "achieved": gbs, "peak": hbm_peak, "unit": "GB/s",
               "frac": gbs / hbm_peak, "bytes_per_launch": chain_bytes,
               "peak_note": f"{peak_kind} HBM copy bandwidth"}
        first, other = (tensor, hbm) if tensor["frac"] >= hbm["frac"] else (hbm, tensor)
        roof = dict(first, traffic=None, kernel=dominant, launch_ms=avg[dominant],
                    other_roof={k: other[k] for k in ("bound", "achieved", "peak", "unit",
                                                       "frac")})
    elif step.cim and info is not None:
        # Both roofs of a CIM layer step: the MMA work on the int8 tensor
        # peak, and the bytes it must move (its source read once, int8
        # weights of both signs, the f32 output) on HBM; the binding one is
        # the one with the larger fraction.
        ops = 2 * info.macs
        achieved = ops / dur_s / 1e12
        int8_peak = 2 * bf16_peak
        layer_bytes = info.in_bytes + 2 * info.n * info.k + 4 * info.m * info.n
        gbs = layer_bytes / dur_s / 1e9
        tensor = {"bound": "tensor", "achieved": achieved, "peak": int8_peak, "unit": "TFLOP/s",
                  "frac": achieved / int8_peak, "ops_per_launch": ops,
                  "peak_note": f"int8 dense = 2 x {peak_kind} bf16 cuBLAS ({bf16_peak} TF/s); "
                               "ops = 2 x branches x M x K x N (unpadded) as TOPS"}
        hbm = {"bound": "hbm", "achieved": gbs, "peak": hbm_peak, "unit": "GB/s",
               "frac": gbs / hbm_peak, "bytes_per_launch": layer_bytes,
               "peak_note": f"{peak_kind} HBM copy bandwidth"}
        first, other = (tensor, hbm) if tensor["frac"] >= hbm["frac"] else (hbm, tensor)
        roof = dict(first, traffic=None, kernel=dominant, launch_ms=avg[dominant],
                    other_roof={k: other[k] for k in ("bound", "achieved", "peak", "unit",
                                                       "frac")})
    else:
        algo = None
        if info is not None and dominant.endswith(".prepare"):
            # Read the source tensor once; write the prepared int8 columns and
            # their group exponents (m_pad x (k_pad + 4 T) per activation branch).
            ab = 1 if info.branches == 2 else 2
            t_tiles = -(-info.k // 64)
            m_pad = -(-info.m // 128) * 128
            algo = info.in_bytes + ab * m_pad * t_tiles * (64 + 4)
        gbs = (algo / dur_s / 1e9) if algo else None
        roof = {"bound": "hbm", "achieved": gbs, "peak": hbm_peak, "unit": "GB/s",
                "frac": (gbs / hbm_peak) if gbs else None, "traffic": None, "kernel": dominant,
                "bytes_per_launch": algo, "launch_ms": avg[dominant],
                "peak_note": f"{peak_kind} HBM copy bandwidth"}
    roof["traffic"], roof["traffic_source"] = ncu_traffic(args.workload, batch, dominant)
    kernel_table = {n: {"ms": round(avg[n], 5), "share": round(avg[n] / total_kernel, 4)}
                    for n in names}

    # End to end through the public API (torch.compile, runtime="cuda").
    name = backend.register()
    compiled = torch.compile(model, backend=name, fullgraph=True, dynamic=False,
                             options={"runtime": "cuda", "device": local,
                                      "chain": prog.chained})
    host = x.pin_memory()
    with torch.inference_mode():
        out = compiled(host)
        for _ in range(args.warmup):
            out = compiled(host)
        barrier()
        e_ms = 0.0
        for _ in range(args.steps):
            flush.zero_()
            a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            a.record(stream)
            out = compiled(host)
            b.record(stream)
            b.synchronize()
            e_ms += a.elapsed_time(b)
        barrier()
    et = torch.tensor([e_ms], device=dev, dtype=torch.float64)
    if world > 1:
        dist.all_reduce(et, op=dist.ReduceOp.MAX)
    e2e_value = world * batch * args.steps / (float(et.item()) / 1000)
    h2d = host.numel() * host.element_size()
    d2h = out.numel() * out.element_size() + 4  # logits + status word

    cpu = None
    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        threads = os.cpu_count() or 1
        rate, dt = cpu_baseline(args.workload, args.cpu_sample, threads)
        cpu = {"value": rate, "unit": UNIT, "cores": threads, "kind": "port",
               "sample": f"{args.cpu_sample} {args.workload} images through the oracle's "
                         f"restated CIMSoftwareRunner (40-Work transactions, plan reuse, "
                         f"residency) + PyTorch CPU glue, {dt:.1f} s wall"}

    if rank == 0:
        line = {
            "metric": METRIC, "value": value, "unit": UNIT, "n_gpus": world,
            "steps": args.steps, "warmup": args.warmup,
            "ms_per_step": elapsed_ms / args.steps, "higher_is_better": True,
            "scaling": "weak", "vs_baseline": None, "dtype": "bf16", "data": "synthetic",
            "config": {"workload": f"{args.workload}: {w.description}", "batch_per_gpu": batch,
                       "global_batch": batch * world, "parallelism": f"batch-sharded x{world}",
                       "l2": "flushed between steps (256 MiB write, outside the timed span)",
                       "graph": "CUDA graph replay", "cim_macs_per_batch": prog.macs,
                       "lowering": "fused layer chain (one persistent kernel)" if prog.chained
                                   else "per-layer kernels",
                       "arithmetic": "BF16 sign-split: int8 mantissa crossbar dots, BF16 "
                                     "tiles, f32 K sums"},
            "gpu_launches": len(prog.steps) * args.steps,
            "e2e": {"value": e2e_value, "unit": UNIT, "h2d_bytes_per_step": h2d,
                    "d2h_bytes_per_step": d2h},
            "roofline": roof,
            "kernels": kernel_table,
            "cpu_baseline": cpu,
            "clocks": clocks.summary(),
        }
        print(json.dumps(line), flush=True)
    if world > 1:
        dist.barrier()
        dist.destroy_process_group()


if __name__ == "__main__":
    main()
