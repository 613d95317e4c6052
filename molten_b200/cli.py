"""Molten command line: ``molten compile | benchmark | info``.

Mirrors the reference's ``molten/cli.py:19-120`` (same commands, options and
graph-JSON schema) on the sm_100a backend:

* ``compile graph.json -o DIR [--fp16] [--dtype D] [--build]`` reads a graph
  in the reference's JSON form -- ``{"name": ..., "ops": [{"type": "<OpType
  name>", "inputs": [op ids], "name": ...}, ...]}`` (``cli.py:27-35``) -- and
  writes one ``.cu`` per fusion group plus ``molten_generated.h`` and the
  engine headers (``ZeroCompiler.save``).  Ops may also carry ``"shape"``
  (ints or symbolic names), ``"dtype"`` and ``"attrs"`` (``eps``, ``value``,
  ``min``/``max``, ``period``/``offset``, ``dim`` ...); without shapes the
  kernels are emitted for stand-in sizes and the runtime re-specialises them
  per call.  ``--fp16`` (a TypeError in the reference, ``cli.py:37``) selects
  fp16 I/O; ``--build`` also compiles each kernel to an sm_100a cubin.
* ``benchmark --dim D --seq S [-o DIR] [--dtype D] [--run]`` builds the
  RMSNorm graph of ``cli.py:47-72`` and generates its kernel; ``--run`` also
  launches it on cuda:0 against seeded inputs and reports us/call and GB/s.
* ``info`` prints the version and what the backend generates.
"""

from __future__ import annotations

import argparse
import json
import sys
from pathlib import Path

from . import __version__
from .compiler import ZeroCompiler
from .ir import DataflowGraph, OpType, TensorShape

_ATTR_KEYS = ("eps", "value", "min", "max", "period", "offset", "kind", "dim")


def graph_from_json(data: dict) -> DataflowGraph:
    """DataflowGraph from the reference's graph JSON (``cli.py:27-35``).

    Op ids are positions in ``ops`` (``add_op`` numbers ops from 0 in
    order).  OUTPUT ops are registered as graph outputs."""
    g = DataflowGraph(data.get("name", "unnamed"))
    for pos, spec in enumerate(data.get("ops", [])):
        try:
            op_type = OpType[spec["type"]]
        except KeyError as exc:
            raise ValueError(f"op {pos}: unknown op type {spec.get('type')!r}") from exc
        inputs = [int(i) for i in spec.get("inputs", [])]
        for i in inputs:
            if not 0 <= i < pos:
                raise ValueError(f"op {pos} ({spec['type']}): input {i} is not an earlier op")
        name = spec.get("name", "")
        if op_type == OpType.OUTPUT:
            if len(inputs) != 1:
                raise ValueError(f"op {pos}: OUTPUT takes exactly one input")
            g.add_output(inputs[0], name or "output")
            continue
        shape = spec.get("shape")
        attrs = dict(spec.get("attrs", {}))
        for k in _ATTR_KEYS:
            if k in spec and k not in attrs:
                attrs[k] = spec[k]
        g.add_op(op_type, inputs=inputs, name=name,
                 shape=TensorShape(list(shape)) if shape is not None else None,
                 dtype=spec.get("dtype", "float16"), **attrs)
    return g


def graph_to_json(g: DataflowGraph) -> dict:
    """The inverse of ``graph_from_json`` (op ids must be 0..n-1)."""
    ops = []
    for pos, oid in enumerate(sorted(g.ops)):
        if oid != pos:
            raise ValueError("graph op ids are not contiguous from 0")
        op = g.ops[oid]
        spec = {"type": op.op_type.name, "inputs": list(op.inputs), "name": op.name}
        if op.shape is not None and op.op_type != OpType.OUTPUT:
            spec["shape"] = list(op.shape.dims)
        if op.op_type == OpType.INPUT:
            spec["dtype"] = op.dtype
        if op.attrs:
            spec["attrs"] = dict(op.attrs)
        ops.append(spec)
    return {"name": g.name, "ops": ops}


def cmd_compile(args) -> int:
    path = Path(args.graph)
    if not path.exists():
        print(f"Error: {path} not found")
        return 1
    g = graph_from_json(json.loads(path.read_text()))
    compiler = ZeroCompiler(verbose=True, fp16=args.fp16, dtype=args.dtype)
    kernels = compiler.compile(g)
    out = Path(args.output)
    compiler.save(kernels, str(out))
    print(f"Generated {len(kernels)} kernel(s) in {out}")
    if args.build:
        from .build import build_cubin
        for k in kernels:
            cubin = build_cubin(k.source, k.name, cache_dir=out)
            print(f"  built {cubin.name}")
    return 0


def _rmsnorm_graph(seq: int, dim: int, dtype: str) -> DataflowGraph:
    g = DataflowGraph("rmsnorm_bench")
    x = g.add_input("x", TensorShape([seq, dim]), dtype=dtype)
    w = g.add_input("w", TensorShape([dim]), dtype=dtype)
    g.add_output(g.rms_norm(x, w, "norm"))
    return g


def cmd_benchmark(args) -> int:
    print("Molten Benchmark")
    print(f"  Dimensions: seq={args.seq}, dim={args.dim}, dtype={args.dtype}")
    g = _rmsnorm_graph(args.seq, args.dim, args.dtype)
    compiler = ZeroCompiler(verbose=True, dtype=args.dtype)
    kernels = compiler.compile(g)
    print(f"\n  Generated {len(kernels)} kernel(s):")
    for k in kernels:
        print(f"    {k.name} ({k.source.count(chr(10))} lines)")
    if args.output:
        compiler.save(kernels, args.output)
        print(f"  Saved to {args.output}")
    if args.run:
        res = run_rmsnorm_benchmark(args.seq, args.dim, args.dtype, kernels[0])
        print(f"  {res['us_per_call']:.2f} us/call, {res['gbs']:.1f} GB/s "
              f"({res['bytes'] / 1e6:.1f} MB per call, cuda:0)")
    return 0


def run_rmsnorm_benchmark(seq: int, dim: int, dtype: str, kernel, iters: int = 50) -> dict:
    """Launch the generated RMSNorm kernel on cuda:0 (seeded inputs) and
    time ``iters`` back-to-back calls with CUDA events."""
    import torch
    from .runtime import MoltenRuntime
    tdt = {"float32": torch.float32, "bfloat16": torch.bfloat16, "float16": torch.float16}[dtype]
    gen = torch.Generator().manual_seed(0)
    x = torch.randn(seq, dim, generator=gen).to(tdt).cuda()
    w = (1 + 0.1 * torch.randn(dim, generator=gen)).to(tdt).cuda()
    fn = MoltenRuntime().compile(kernel)
    out = fn(x, w)
    for _ in range(3):
        fn(x, w, out=out)
    torch.cuda.synchronize()
    a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    a.record()
    for _ in range(iters):
        fn(x, w, out=out)
    b.record()
    torch.cuda.synchronize()
    us = a.elapsed_time(b) * 1e3 / iters
    nbytes = 2 * x.numel() * x.element_size() + w.numel() * w.element_size()
    return {"us_per_call": us, "gbs": nbytes / (us * 1e-6) / 1e9, "bytes": nbytes}


def cmd_info() -> int:
    print(f"Molten v{__version__} (sm_100a backend)")
    print("  Fused GPU kernel generation from mathematical specifications")
    print("")
    print("  Row patterns:  RMSNorm, RMSNorm*SiLU(gate), softmax (+causal mask),")
    print("                 reductions + elementwise DAGs (register engine,")
    print("                 TMA-staged ring, persistent stream form)")
    print("  Elementwise:   N-op chains with per-column / per-row broadcasting")
    print("  MatMul:        tcgen05/TMEM GEMM with a fused elementwise epilogue")
    print("  Output:        .cu + nvcc-built sm_100a cubins, loaded through the")
    print("                 libmolten_rt.so C ABI (include/molten_rt.h)")
    print("  Precision:     fp32 compute; fp32, bf16 or fp16 I/O")
    return 0


def build_parser() -> argparse.ArgumentParser:
    parser = argparse.ArgumentParser(prog="molten",
                                     description="Molten: math to fused CUDA kernels (sm_100a)")
    sub = parser.add_subparsers(dest="command")
    p = sub.add_parser("compile", help="Compile a graph JSON to .cu")
    p.add_argument("graph", help="Path to graph JSON")
    p.add_argument("--output", "-o", default="output/", help="Output directory")
    p.add_argument("--fp16", action="store_true", help="Generate fp16 I/O kernels")
    p.add_argument("--dtype", default=None, choices=["float32", "bfloat16", "float16"],
                   help="I/O dtype of the graph inputs (overrides --fp16)")
    p.add_argument("--build", action="store_true", help="Also build sm_100a cubins")
    p = sub.add_parser("benchmark", help="Generate (and optionally run) an RMSNorm kernel")
    p.add_argument("--dim", type=int, default=3584, help="Hidden dimension")
    p.add_argument("--seq", type=int, default=2048, help="Sequence length")
    p.add_argument("--output", "-o", default=None, help="Save kernels to dir")
    p.add_argument("--dtype", default="float32", choices=["float32", "bfloat16", "float16"])
    p.add_argument("--run", action="store_true", help="Launch and time it on cuda:0")
    sub.add_parser("info", help="Show version and capabilities")
    return parser


def main(argv=None) -> int:
    parser = build_parser()
    args = parser.parse_args(argv)
    if args.command == "compile":
        return cmd_compile(args)
    if args.command == "benchmark":
        return cmd_benchmark(args)
    if args.command == "info":
        return cmd_info()
    parser.print_help()
    return 0


if __name__ == "__main__":
    sys.exit(main() or 0)
