#!/usr/bin/env python
"""Benchmark of the fused-kernel path on B200s: one JSON line on rank 0.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--workload NAME]
                    [--impl molten|reference]

A step is one launch of the fused kernel over one batch of the workload's
synthetic inputs, already resident in HBM.  Default workload: RMSNorm*SiLU
(gate), bf16, hidden 3584, 8192 rows (176 MB per call, larger than L2).
With N GPUs (torchrun, one process per GPU, NCCL only for the barrier and
the max-over-ranks time) every rank runs the same workload on its own rows
(global row offset = rank * rows): weak scaling, no data-path collective.
The GEMM workload is instead split by output columns (strong scaling).

``--impl reference`` times the reference's CPU path (benchmarks/ops.py,
restated in oracle/torch_cpu.py) on the host cores, rank 0 only.
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

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, ROOT)

L2_BYTES = 126 * 1024 * 1024
FALLBACK_PEAKS = {"hbm_gbs": 6650.0, "bf16_tflops": 1590.0, "bf16_tflops_sustained": 1400.0}


def parse_args():
    p = argparse.ArgumentParser()
    p.add_argument("--gpus", type=int, default=1)
    p.add_argument("--steps", type=int, default=50)
    p.add_argument("--warmup", type=int, default=5)
    p.add_argument("--impl", choices=["molten", "reference"], default="molten")
    p.add_argument("--workload", default=None)
    p.add_argument("--tune", default=None, help="JSON tile overrides, e.g. '{\"row\": {\"tpc\": 128}}'")
    p.add_argument("--no-e2e", action="store_true")
    p.add_argument("--e2e-chunks", type=int, default=5,
                   help="row blocks whose host<->device copies overlap in the end-to-end step")
    p.add_argument("--no-cpu-baseline", action="store_true")
    p.add_argument("--cpu-seconds", type=float, default=12.0)
    p.add_argument("--soak", type=float, default=1.0, help="untimed seconds under load before timing")
    p.add_argument("--no-graph", action="store_true", help="time eager launches, not a CUDA graph")
    return p.parse_args()


def load_peaks():
    path = os.path.join(ROOT, "MEASURED_PEAKS.json")
    try:
        with open(path) as f:
            d = json.load(f)
        return d, "measured"
    except (OSError, ValueError):
        return dict(FALLBACK_PEAKS), "fallback"


# ------------------------------------------------------------------ clocks
class ClockSampler:
    """nvidia-smi samples (every 200 ms) of this GPU during the timed region."""
    FIELDS = ("pci.bus_id,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, bus_id: str):
        self.bus_id = str(bus_id).lower()
        self.proc = None
        self.lines = []
        self.t = None

    def start(self):
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", f"--query-gpu={self.FIELDS}", "--format=csv,noheader,nounits",
                 "-lms", "200"], stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
        except OSError:
            self.proc = None
            return
        self.t = threading.Thread(target=self._read, daemon=True)
        self.t.start()

    def _read(self):
        for line in self.proc.stdout:
            self.lines.append(line.strip())

    def stop(self):
        if self.proc is None:
            return None
        self.proc.terminate()
        try:
            self.proc.wait(timeout=5)
        except subprocess.TimeoutExpired:
            self.proc.kill()
        if self.t:
            self.t.join(timeout=2)
        sms, mx, reasons = [], None, set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for ln in self.lines:
            parts = [p.strip() for p in ln.split(",")]
            if len(parts) < 9:
                continue
            bus = parts[0].lower()
            if self.bus_id and bus[-7:] != self.bus_id[-7:]:      # "bb:dd.f"
                continue
            try:
                sms.append(float(parts[1]))
                mx = float(parts[2])
            except ValueError:
                continue
            for n, v in zip(names, parts[5:9]):
                if v.lower() == "active":
                    reasons.add(n)
        if not sms:
            return None
        return {"sm_mhz": statistics.median(sms), "sm_max_mhz": mx, "samples": len(sms),
                "reasons": sorted(reasons)}


# ---------------------------------------------------------------- helpers
def dist_info():
    return (int(os.environ.get("RANK", 0)), int(os.environ.get("WORLD_SIZE", 1)),
            int(os.environ.get("LOCAL_RANK", 0)))


def emit(obj):
    print(json.dumps(obj), flush=True)


def cpu_sample(w, fraction_rows=None):
    """A bounded sample of the workload for the CPU path: same kind, dtype
    and row width, fewer rows (GEMM: fewer output rows)."""
    from molten_b200 import workloads
    p = dict(w.params)
    if w.kind in ("rmsnorm", "rmsnorm_silu_gate", "chain"):
        p["rows"] = max(1, min(p["rows"], fraction_rows or 1024))
    elif w.kind == "softmax":
        shape = list(p["shape"])
        cols = shape[-1]
        rows = max(1, min(int(__import__("numpy").prod(shape[:-1])), (fraction_rows or 1024)))
        p["shape"] = (rows, cols)
    elif w.kind in workloads.GEMM_KINDS:
        p["m"] = min(p["m"], fraction_rows or 256)
    elif w.kind == "attention_score":
        p["heads"] = 1
        p["m"] = min(p["m"], fraction_rows or 256)
    elif w.kind == "rope":
        p["batch"] = 1
        p["seq"] = max(1, min(p["seq"], (fraction_rows or 1024) // max(1, p["heads"] // 8)))
    return workloads.scaled(w, **p)


def time_cpu(w, budget_s: float, threads: int):
    """Run the reference's CPU path (oracle/torch_cpu.py) on a bounded sample
    until ~budget_s seconds are spent; returns (bytes or flops per second,
    sample description, per-call seconds)."""
    import torch
    from molten_b200 import workloads
    from oracle import torch_cpu
    torch.set_num_threads(threads)
    sw = cpu_sample(w)
    xs = workloads.make_inputs(sw, seed=0, device="cpu")
    params = dict(sw.params)
    # memory-bound kinds: rotate over distinct copies of the sample, ~1 GB in
    # all, so that calls stream from host DRAM as the full workload would
    # instead of re-reading a sample that sits in the last-level cache
    sets = [xs]
    if w.kind not in workloads.GEMM_KINDS:
        nbytes = max(1, sum(t.numel() * t.element_size() for t in xs))
        sets += [[t.clone() for t in xs] for _ in range(min(47, -(-(1 << 30) // nbytes)) - 1)]
    torch_cpu.run_workload(sw.kind, xs, params)          # warm-up
    times = []
    t_end = time.perf_counter() + budget_s
    while time.perf_counter() < t_end or len(times) < 3:
        t0 = time.perf_counter()
        torch_cpu.run_workload(sw.kind, sets[len(times) % len(sets)], params)
        times.append(time.perf_counter() - t0)
        if len(times) >= 200:
            break
    t = statistics.median(times)
    work = sw.flops_per_call if w.kind in workloads.GEMM_KINDS else sw.bytes_per_call
    desc = (f"{sw.kind} {sw.params} {sw.dtype}, median of {len(times)} calls"
            + (f" over {len(sets)} rotating input copies" if len(sets) > 1 else ""))
    return work / t, desc, t


def metric_of(w):
    from molten_b200 import workloads
    if w.kind in workloads.GEMM_KINDS:
        return "epilogue GEMM TFLOP/s", "TFLOP/s", 1e12
    return "fused-kernel HBM GB/s", "GB/s", 1e9


# ------------------------------------------------------------ reference arm
def run_reference(args, w):
    rank, world, _ = dist_info()
    if rank != 0:
        return
    threads = os.cpu_count() or 1
    metric, unit, scale = metric_of(w)
    vals = []
    for _ in range(args.warmup):
        time_cpu(w, 0.0, threads)
    t_start = time.perf_counter()
    desc = ""
    for _ in range(args.steps):
        v, desc, _ = time_cpu(w, max(0.5, args.cpu_seconds / max(args.steps, 1)), threads)
        vals.append(v / scale)
    elapsed = time.perf_counter() - t_start
    value = statistics.median(vals)
    emit({"impl": "reference", "metric": metric, "value": value, "unit": unit,
          "n_gpus": args.gpus, "steps": args.steps, "warmup": args.warmup,
          "ms_per_step": 1000.0 * elapsed / max(args.steps, 1),
          "higher_is_better": True, "scaling": "weak", "vs_baseline": None,
          "dtype": {"float32": "f32", "bfloat16": "bf16", "float16": "f16"}[w.dtype],
          "data": "synthetic",
          "config": {"workload": w.name, **{k: (list(v) if isinstance(v, tuple) else v)
                                            for k, v in w.params.items()}},
          "cpu_baseline": {"value": value, "unit": unit, "cores": threads, "kind": "port",
                           "sample": desc},
          "e2e": {"value": value, "unit": unit, "h2d_bytes_per_step": 0,
                  "d2h_bytes_per_step": 0}})


# --------------------------------------------------------------- molten arm
def run_molten(args, w):
    import torch
    import torch.distributed as dist

    from molten_b200 import workloads
    from molten_b200.codegen import CodeGenerator
    from molten_b200.fusion import FusionEngine
    from molten_b200.runtime import MoltenRuntime
    from molten_b200.shard import col_shards

    rank, world, local = dist_info()
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    if world > 1:
        import datetime
        dist.init_process_group("nccl", device_id=dev, timeout=datetime.timedelta(seconds=180))
    tune = json.loads(args.tune) if args.tune else None
    rt = MoltenRuntime(tune=tune)
    metric, unit, scale = metric_of(w)
    is_gemm = w.kind in workloads.GEMM_KINDS

    # ---- inputs (this rank's rows, or its column block for the GEMM)
    xs = workloads.make_inputs(w, seed=rank if not is_gemm else 0, device=dev)
    row_offset = 0
    if is_gemm:
        n = w.params["n"]
        n0, n1 = col_shards(n, world)[rank]
        *lead, B, bias = xs             # [A, B, bias] or [x, w, B, bias]
        xs = [*lead, B[:, n0:n1].contiguous(), bias[n0:n1].contiguous()]
        w_local = workloads.scaled(w, n=n1 - n0)
        scaling = "strong" if world > 1 else "weak"
    else:
        w_local = w
        row_offset = rank * (xs[0].numel() // xs[0].shape[-1])
        scaling = "weak"
    g = w_local.graph()
    grp = FusionEngine().fuse(g)[0]
    gen = CodeGenerator(tune=tune)
    shapes = {i: tuple(t.shape) for i, t in zip(sorted(i for i, o in g.ops.items()
                                                      if o.op_type.name == "INPUT"), xs)}
    dtypes = {i: str(t.dtype).replace("torch.", "") for i, t in zip(sorted(shapes), xs)}
    gk = gen.generate(g, grp, shapes, dtypes)
    ck = rt.compile(gk)
    work = w_local.flops_per_call if is_gemm else w_local.bytes_per_call
    launches_per_step = len(gk.plan.kernels)

    # ---- L2 policy: rotate (inputs, output) sets so that the bytes one pass
    # over the sets reads and writes exceed 2x L2.  Each set has its own
    # output: a single output buffer rewritten every step could stay dirty
    # in L2 and never be written back to HBM.
    in_bytes = sum(t.numel() * t.element_size() for t in xs)
    out0 = ck(*xs)
    out_bytes = out0.numel() * out0.element_size()
    io_bytes = in_bytes + out_bytes
    sets = 1 if io_bytes >= 2 * L2_BYTES else min(64, -(-2 * L2_BYTES // max(io_bytes, 1)))
    flush = None
    if io_bytes * sets < 2 * L2_BYTES:
        flush = torch.empty(2 * L2_BYTES // 4, dtype=torch.float32, device=dev)
    bufs = [xs] + [[t.clone() for t in xs] for _ in range(sets - 1)]
    outs = [out0] + [torch.empty_like(out0) for _ in range(sets - 1)]
    out = outs[0]
    stream = torch.cuda.current_stream(dev)

    def step(i):
        ck(*bufs[i % sets], out=outs[i % sets], row_offset=row_offset)

    for i in range(args.warmup):
        step(i)
    torch.cuda.synchronize(dev)

    # The K timed steps are one CUDA graph holding exactly K launches, so the
    # host's per-call Python cost is not inside the device timing.
    graph = None
    if flush is None and not args.no_graph:
        graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(graph):
            for i in range(args.steps):
                step(i)
        torch.cuda.synchronize(dev)

    # ---- timed region (device time, max over ranks)
    bus = ""
    try:
        pr = torch.cuda.get_device_properties(dev)
        bus = f"{pr.pci_domain_id:08x}:{pr.pci_bus_id:02x}:{pr.pci_device_id:02x}.0"
    except Exception:
        pass
    clocks = ClockSampler(bus)
    clocks.start()
    # untimed soak (extra warm-up) so the clocks are sampled under load
    soak_end = time.perf_counter() + args.soak
    while time.perf_counter() < soak_end:
        if graph is not None:
            graph.replay()
        else:
            for i in range(min(args.steps, 20)):
                if flush is not None:
                    flush.zero_()
                step(i)
        torch.cuda.synchronize(dev)
    if world > 1:
        dist.barrier()
    torch.cuda.synchronize(dev)
    if flush is None:
        e0 = torch.cuda.Event(enable_timing=True)
        e1 = torch.cuda.Event(enable_timing=True)
        e0.record(stream)
        if graph is not None:
            graph.replay()
        else:
            for i in range(args.steps):
                step(i)
        e1.record(stream)
        torch.cuda.synchronize(dev)
        total_ms = e0.elapsed_time(e1)
    else:
        evs = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True))
               for _ in range(args.steps)]
        for i, (a, b) in enumerate(evs):
            flush.zero_()
            a.record(stream)
            step(i)
            b.record(stream)
        torch.cuda.synchronize(dev)
        total_ms = sum(a.elapsed_time(b) for a, b in evs)
    if world > 1:
        dist.barrier()
    torch.cuda.synchronize(dev)
    clk = clocks.stop()
    ms = total_ms / args.steps
    if world > 1:
        t = torch.tensor([ms], device=dev, dtype=torch.float64)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        ms = float(t.item())
    status = MoltenRuntime.read_status(local) if is_gemm else 0

    # ---- end to end: host buffers -> H2D -> kernel -> D2H, same metric
    e2e = None
    if not args.no_e2e:
        host_in = [t.cpu().pin_memory() for t in xs]
        host_out = torch.empty(out.shape, dtype=out.dtype, pin_memory=True)
        n_e2e = max(3, min(args.steps, 20))
        chunks = args.e2e_chunks if ck.row_chunkable(host_in) else 1

        def e2e_step():
            # the public host-buffer call: uploads, kernels and downloads of
            # row blocks overlap on three streams (one block when the graph
            # does not split by rows)
            ck.run_host(*host_in, out=host_out, chunks=chunks, row_offset=row_offset, device=local)

        for _ in range(2):
            e2e_step()
        torch.cuda.synchronize(dev)
        if world > 1:
            dist.barrier()
        a = torch.cuda.Event(enable_timing=True)
        b = torch.cuda.Event(enable_timing=True)
        a.record(stream)
        for _ in range(n_e2e):
            e2e_step()
        b.record(stream)
        torch.cuda.synchronize(dev)
        e_ms = a.elapsed_time(b) / n_e2e
        if world > 1:
            t = torch.tensor([e_ms], device=dev, dtype=torch.float64)
            dist.all_reduce(t, op=dist.ReduceOp.MAX)
            e_ms = float(t.item())
        h2d = sum(t.numel() * t.element_size() for t in xs)
        d2h = out.numel() * out.element_size()
        e2e = {"value": world * work / (e_ms * 1e-3) / scale, "unit": unit,
               "h2d_bytes_per_step": h2d, "d2h_bytes_per_step": d2h, "ms_per_step": e_ms,
               "path": "CompiledKernel.run_host", "row_blocks": chunks}

    if world > 1:
        dist.barrier()
    if rank != 0:
        if world > 1:
            dist.destroy_process_group()
        return

    peaks, peaks_kind = load_peaks()
    achieved = work / (ms * 1e-3) / scale                  # this rank's kernel, per launch
    burst = None
    if is_gemm:
        # the K timed launches follow a >= 1 s soak under the power cap: the
        # sustained cuBLAS figure is the like-for-like denominator; the burst
        # figure's fraction is reported beside it
        burst = peaks.get("bf16_tflops", FALLBACK_PEAKS["bf16_tflops"])
        sustained = peaks.get("bf16_tflops_sustained", FALLBACK_PEAKS["bf16_tflops_sustained"])
        peak = sustained if args.soak >= 1.0 else burst
        roof = {"bound": "tensor", "unit": "TFLOP/s"}
    else:
        peak = peaks.get("hbm_gbs", FALLBACK_PEAKS["hbm_gbs"])
        roof = {"bound": "hbm", "unit": "GB/s"}
    traffic = None
    tpath = os.path.join(ROOT, "profiles", "ncu_traffic.json")
    try:
        # captured on the whole single-GPU workload: a column shard's launch
        # moves a different byte count, so N > 1 GEMM lines carry none
        if not (is_gemm and world > 1):
            with open(tpath) as f:
                traffic = json.load(f).get(w_local.name if not is_gemm else w.name)
    except (OSError, ValueError):
        traffic = None
    src = f"{peaks_kind} (MEASURED_PEAKS.json)" if peaks_kind == "measured" else "fallback"
    if is_gemm:
        src += (" cuBLAS bf16 sustained, after a %.1f s soak" % args.soak if peak != burst
                else " cuBLAS bf16 burst")
    roof.update({"achieved": achieved, "peak": peak, "frac": achieved / peak,
                 "traffic": traffic, "peak_source": src})
    if burst is not None:
        roof["frac_of_burst"] = achieved / burst
    cpu = None
    if world == 1 and not args.no_cpu_baseline:
        threads = os.cpu_count() or 1
        v, desc, _ = time_cpu(w, args.cpu_seconds, threads)
        cpu = {"value": v / scale, "unit": unit, "cores": threads, "kind": "port", "sample": desc}
    cfg = {"workload": w.name, **{k: (list(v) if isinstance(v, tuple) else v)
                                  for k, v in w_local.params.items()},
           "l2": ("inputs + output larger than 2x L2" if sets == 1 else
                  f"{sets} rotating input+output sets ({io_bytes * sets / 2**20:.0f} MiB > 2x L2)")
           if flush is None else "L2 flushed (256 MiB write) before every timed launch",
           "parallelism": f"dp{world}" if not is_gemm else f"n-shard{world}",
           "timing": ("one CUDA graph replay of exactly K launches" if graph is not None
                      else "eager launches") + f", CUDA events; {args.soak:.1f} s untimed soak",
           "kernel": gk.name, "tiles": {k: v for k, v in gk.plan.kernels[0].config.items()
                                        if k not in ("needed", "prefetch", "materialize")}}
    res = {"metric": metric, "value": world * work / (ms * 1e-3) / scale, "unit": unit,
           "n_gpus": world, "steps": args.steps, "warmup": args.warmup, "ms_per_step": ms,
           "us_per_call": ms * 1e3, "higher_is_better": True, "scaling": scaling,
           "vs_baseline": None,
           "dtype": {"float32": "f32", "bfloat16": "bf16", "float16": "f16"}[w.dtype],
           "data": "synthetic", "config": cfg, "e2e": e2e,
           "gpu_launches": args.steps * launches_per_step,
           "roofline": roof, "cpu_baseline": cpu, "clocks": clk}
    if is_gemm:
        res["status_word"] = status
    emit(res)
    if world > 1:
        dist.destroy_process_group()


def main():
    args = parse_args()
    from molten_b200 import workloads
    name = args.workload or workloads.HEADLINE
    if name not in workloads.WORKLOADS:
        sys.exit(f"unknown workload {name}; one of {sorted(workloads.WORKLOADS)}")
    w = workloads.WORKLOADS[name]
    if args.impl == "reference":
        run_reference(args, w)
    else:
        run_molten(args, w)


if __name__ == "__main__":
    main()
