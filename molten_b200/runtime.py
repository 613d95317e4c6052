"""Runtime: generated source -> nvcc cubin -> launches through libmolten_rt.so.

Drop-in for the reference's ``molten/runtime.py``: ``MoltenRuntime(cache_dir,
verbose).compile(kernel) -> CompiledKernel`` (``runtime.py:47-94``) and
``CompiledKernel(*tensors)`` returning a new output tensor
(``runtime.py:31-36``), with ``clear_cache`` (``runtime.py:201-207``).

Differences that follow from the design:

* the kernel is built with nvcc into an sm_100a cubin (cached on disk by
  content hash) and launched through the C ABI of ``libmolten_rt.so``
  (``include/molten_rt.h``) on the caller's current torch stream; there is no
  pybind module and no torch.utils.cpp_extension build;
* a call takes every graph input in graph-input order (x, w[, g] ...), not
  only ``x``; outputs are allocated with ``torch.empty`` (no zero fill), or
  passed in with ``out=``;
* the first call with a new (shape, dtype) signature re-specialises the
  group for it (shapes and dtypes are baked into the kernel);
* there is no CPU or eager fallback: a missing library, a failed build or a
  failed launch raises.
"""

from __future__ import annotations

import ctypes
import hashlib
import os
import threading
from collections import OrderedDict
from dataclasses import dataclass, field
from pathlib import Path
from typing import Optional

from . import _capi
from .build import build_cubin, default_cache_dir
from .codegen import CodeGenerator, GeneratedKernel, KernelConfig, kernel_entry
from .lowering import DTYPE_SIZE, LoweringError, canon_dtype

_TORCH_DTYPES = None


def _torch():
    import torch
    return torch


def _dtype_name(t) -> str:
    return canon_dtype(str(t.dtype))


def _torch_dtype(name: str):
    torch = _torch()
    return {"float32": torch.float32, "bfloat16": torch.bfloat16, "float16": torch.float16}[name]


_TMA_CODE = {"bfloat16": _capi.DT_BF16, "float16": _capi.DT_F16, "float32": _capi.DT_F32}

# Programmatic dependent launch for every kernel (MOLTEN_PDL=0 turns it off):
# consecutive launches overlap launch processing and CTA scheduling; each
# kernel still waits for its predecessor before touching global memory.
PDL = os.environ.get("MOLTEN_PDL", "1") != "0"

# MOLTEN_DEBUG=1: every call waits for its kernels and reads (and clears)
# the device's status word, so a bounded wait that ran out, or an
# asynchronous CUDA error, is raised by the call that caused it instead of
# surfacing at a later read.  Costs a synchronisation per call.
DEBUG = os.environ.get("MOLTEN_DEBUG", "0") not in ("", "0")


class _Spec:
    """One shape/dtype specialisation of a group, ready to launch."""

    def __init__(self, gk: GeneratedKernel, cubin: Path):
        self.gk = gk
        self.plan = gk.plan
        self.cubin = cubin
        self.modules: dict = {}
        self.lock = threading.Lock()
        self.entries = [kernel_entry(gk.name, i, len(self.plan.kernels)).encode()
                        for i in range(len(self.plan.kernels))]
        self.out_dtypes = [_torch_dtype(d) for d in self.plan.output_dtypes]
        self.temp_specs = {k: (tuple(s), _torch_dtype(d)) for k, (s, d) in self.plan.temps.items()}
        self._cfgs: dict = {}
        self._tmaps: OrderedDict = OrderedDict()
        self.align = [_alignment_rules(sk) for sk in self.plan.kernels]

    def module(self, device: int) -> _capi.Module:
        m = self.modules.get(device)
        if m is None:
            with self.lock:
                m = self.modules.get(device)
                if m is None:
                    m = _capi.Module(str(self.cubin), device)
                    self.modules[device] = m
        return m

    def launch_cfg(self, i: int, device: int) -> _capi.LaunchCfg:
        key = (i, device)
        cfg = self._cfgs.get(key)
        if cfg is not None:
            return cfg
        sk = self.plan.kernels[i]
        c = sk.config
        cfg = _capi.LaunchCfg()
        if sk.family == "row" and c.get("engine") == "tma":
            torch = _torch()
            sms = torch.cuda.get_device_properties(device).multi_processor_count
            cfg.grid[:] = [max(1, min(sk.rows, sms)), 1, 1]
            cfg.block[:] = [32 * (c["nc"] * c.get("tw", 1) + 1), 1, 1]
            cfg.cluster[:] = [1, 1, 1]
            cfg.smem_bytes = c["smem"]
        elif sk.family == "row":
            teams = -(-sk.rows // c["rpc"])
            cfg.block[:] = [c["block"], 1, 1]
            cfg.cluster[:] = [c["cl"], 1, 1] if c["cl"] > 1 else [1, 1, 1]
            cfg.smem_bytes = c.get("smem", 0) if c.get("stream") else 0
            if c.get("stream"):
                # persistent: as many teams (clusters) as are resident at once,
                # never more -- a late wave would walk as many rows again
                _, resident = self.module(device).max_resident(self.entries[i], cfg)
                if resident < 1:
                    raise _capi.MoltenError(f"kernel {self.entries[i].decode()} cannot be "
                                            f"resident with {cfg.smem_bytes} bytes of shared memory")
                teams = min(teams, resident)
            cfg.grid[:] = [max(1, teams * c["cl"]), 1, 1]
        elif sk.family == "rope":
            total = sk.rows * c["spr"]
            per_cta = c["block"] * c.get("upt", 1)
            cfg.grid[:] = [max(1, min(-(-total // per_cta), 2 ** 31 - 1)), 1, 1]
            cfg.block[:] = [c["block"], 1, 1]
            cfg.cluster[:] = [1, 1, 1]
            cfg.smem_bytes = 0
        elif sk.family == "ew":
            rb = -(-sk.rows // (c["rpc"] * c["upt"]))
            cfg.grid[:] = [c["tiles"], max(1, min(rb, 65535)), 1]
            cfg.block[:] = [c["block"], 1, 1]
            cfg.cluster[:] = [1, 1, 1]
            cfg.smem_bytes = 0
        elif sk.family == "causal":
            # one CTA per row (visible logits) + a CTA per zero tile, or
            # persistent zero CTAs
            zp = c.get("zpersist", 0)
            cfg.grid[:] = [sk.rows + (zp if zp else sk.rows * c["zt"]), 1, 1]
            cfg.block[:] = [c["threads"], 1, 1]
            cfg.cluster[:] = [1, 1, 1]
            cfg.smem_bytes = 0
        elif sk.family == "split3":
            # grid-stride over the operand's VEC-element slots, 8 CTAs per SM
            torch = _torch()
            sms = torch.cuda.get_device_properties(device).multi_processor_count
            slots = -(-c["total"] // c["vec"])
            cfg.grid[:] = [max(1, min(-(-slots // c["block"]), 8 * sms)), 1, 1]
            cfg.block[:] = [c["block"], 1, 1]
            cfg.cluster[:] = [1, 1, 1]
            cfg.smem_bytes = 0
        elif sk.family == "attn":
            # persistent: one CTA per SM (the tile's shared memory allows one)
            torch = _torch()
            sms = torch.cuda.get_device_properties(device).multi_processor_count
            items = c["batch"] * (-(-sk.m // 128))
            cfg.grid[:] = [max(1, min(items, sms)), 1, 1]
            cfg.block[:] = [c["threads"], 1, 1]
            cfg.cluster[:] = [1, 1, 1]
            cfg.smem_bytes = c["smem_bytes"]
        else:
            torch = _torch()
            sms = torch.cuda.get_device_properties(device).multi_processor_count
            tiles = c.get("batch", 1) * (-(-sk.m // c["bm"])) * (-(-sk.n // c["bn"]))
            cfg.block[:] = [128, c["threads"] // 128, 1]
            cfg.smem_bytes = c["smem_bytes"]
            if c.get("streamk"):
                # stream-K: one range of the tiles x k-blocks per CTA over a
                # fixed CTA count (the kernel's workspace slots assume it)
                cfg.grid[:] = [c["sk_ctas"], 1, 1]
                cfg.cluster[:] = [1, 1, 1]
            elif c.get("pair"):
                # clusters of 2 CTAs (an SM pair per 256-row tile), persistent
                cfg.cluster[:] = [2, 1, 1]
                cfg.grid[:] = [2 * max(1, min(tiles, sms // 2)), 1, 1]
                _, clusters = self.module(device).max_resident(self.entries[i], cfg)
                if clusters < 1:
                    raise _capi.MoltenError(f"kernel {self.entries[i].decode()} cannot be resident "
                                            f"as a 2-CTA cluster")
                cfg.grid[:] = [2 * max(1, min(tiles, clusters)), 1, 1]
            else:
                cfg.grid[:] = [max(1, min(tiles, sms)), 1, 1]
                cfg.cluster[:] = [1, 1, 1]
        cfg.flags = _capi.LAUNCH_PDL if PDL else 0
        self._cfgs[key] = cfg
        return cfg

    def stream_k_workspace(self, i: int, device: int):
        """(fp32 partial tiles, int32 per-tile counters) of stream-K kernel i
        on ``device``, allocated once; the kernel leaves the counters at 0.
        Calls of one specialisation must not overlap on the GPU (they share
        this workspace)."""
        key = ("sk", i, device)
        ws = self._cfgs.get(key)
        if ws is None:
            torch = _torch()
            c = self.plan.kernels[i].config
            n = c["sk_tiles"] * c["sk_maxseg"] * c["bm"] * c["bn"]
            ws = (torch.empty(n, dtype=torch.float32, device=f"cuda:{device}"),
                  torch.zeros(c["sk_tiles"], dtype=torch.int32, device=f"cuda:{device}"))
            self._cfgs[key] = ws
        return ws

    def tmap(self, t, dtype: str, rows: int, cols: int, box_inner: int, box_outer: int,
             swizzle: int = 128) -> bytes:
        key = (t.data_ptr(), rows, cols, t.stride(0), box_inner, box_outer, swizzle)
        v = self._tmaps.get(key)
        if v is None:
            esz = DTYPE_SIZE[dtype]
            v = _capi.encode_tma_2d(_TMA_CODE[dtype], t.data_ptr(), cols, rows,
                                    t.stride(0) * esz, box_inner, box_outer, swizzle)
            self._tmaps[key] = v
            if len(self._tmaps) > 64:
                self._tmaps.popitem(last=False)
        else:
            self._tmaps.move_to_end(key)
        return v

    def _attn_args(self, sk, env, device: int):
        """molten_attn_args for the fused attention-score kernel."""
        c = sk.config
        a = _capi.AttnArgs()
        dt = sk.operands[0].dtype
        nb = c["batch"]
        Q = _attn_tensor_2d(env[sk.operands[0].op_id])
        K = _attn_tensor_2d(env[sk.operands[1].op_id])
        P = _attn_tensor_2d(env[sk.outputs[0].op_id])
        ctypes.memmove(a.tmap_q, self.tmap(Q, dt, nb * sk.m, sk.k, 64, 128), 128)
        ctypes.memmove(a.tmap_k, self.tmap(K, dt, nb * sk.n, sk.k, 64, c["bn"]), 128)
        if c["tma_store"]:
            sc = c["store_cols"]          # 32 or 64 columns: a 64- or 128-byte swizzled row
            ctypes.memmove(a.tmap_p, self.tmap(P, sk.outputs[0].dtype, nb * sk.m, sk.n, sc, 32,
                                               2 * sc), 128)
        a.out = P.data_ptr()
        a.m, a.n, a.d = sk.m, sk.n, sk.k
        a.batch = nb
        a.status = _capi.status_word(device)
        return a

    def _row_template(self, i: int, device: int) -> bytes:
        """molten_row_args of row-type kernel i with its per-shape fields set
        (rows, cols, the status word where the kernel has bounded waits),
        as bytes that each call copies and fills with pointers."""
        key = ("row_args", i, device)
        tpl = self._cfgs.get(key)
        if tpl is None:
            sk = self.plan.kernels[i]
            a = _capi.RowArgs()
            a.rows, a.cols = sk.rows, sk.cols
            if (sk.config.get("engine") == "tma" or sk.config.get("stream")
                    or sk.config.get("cl", 1) > 1):
                a.status = _capi.status_word(device)
            tpl = bytes(a)
            self._cfgs[key] = tpl
        return tpl

    def run(self, tensors, outs, stream: Optional[int], row_offset: int):
        torch = _torch()
        plan = self.plan
        dev = tensors[0].device
        di = dev.index if dev.index is not None else torch.cuda.current_device()
        if stream is None:
            # the caller's current stream on that device (the raw handle:
            # torch.cuda.current_stream() costs several microseconds a call)
            stream = torch._C._cuda_getCurrentRawStream(di)
        env = dict(zip(plan.inputs, tensors))
        if outs is None:
            outs = [torch.empty(s, dtype=d, device=dev)
                    for s, d in zip(plan.output_shapes, self.out_dtypes)]
        env.update(zip(plan.outputs, outs))
        if all(o.numel() == 0 for o in outs):
            return outs                      # empty outputs (no rows or no columns): no launch
        for op_id, (s, d) in self.temp_specs.items():
            env[op_id] = torch.empty(s, dtype=d, device=dev)
        mod = self.module(di)
        for i, sk in enumerate(plan.kernels):
            cfg = self.launch_cfg(i, di)
            if sk.family == "attn":
                a = self._attn_args(sk, env, di)
            elif sk.family == "gemm":
                a = _capi.GemmArgs()
                dt = sk.operands[sk.a_operand].dtype
                nb = sk.config.get("batch", 1)
                planes = 1
                if sk.config.get("split3"):
                    # fp32 operands: the three stacked bf16 planes the split
                    # kernels before this one wrote
                    A, B = (env[key] for key in sk.config["planes"])
                    dt, planes = "bfloat16", 3
                else:
                    A = env[sk.operands[sk.a_operand].op_id]
                    B = env[sk.operands[sk.b_operand].op_id]
                A2 = A.reshape(-1, A.shape[-1])
                ctypes.memmove(a.tmap_a, self.tmap(A2, dt, planes * nb * sk.m, sk.k, 64, 128), 128)
                if sk.config.get("b_kmajor"):
                    # B is the transpose of Bt [(batch x) N, K]: its rows, K-major
                    # (an SM pair's CTA stages BN/2 of them)
                    B2 = B.reshape(-1, B.shape[-1])
                    rows_b = sk.config["bn"] // (2 if sk.config.get("pair") else 1)
                    ctypes.memmove(a.tmap_b, self.tmap(B2, dt, planes * nb * sk.n, sk.k, 64, rows_b),
                                   128)
                else:
                    B2 = B.reshape(-1, B.shape[-1])
                    ctypes.memmove(a.tmap_b, self.tmap(B2, dt, planes * nb * sk.k, sk.n, 64, 64), 128)
                a.m, a.n, a.k = sk.m, sk.n, sk.k
                a.batch = nb
                a.status = _capi.status_word(di)
                if sk.config.get("streamk"):
                    work, count = self.stream_k_workspace(i, di)
                    a.work, a.tile_count = work.data_ptr(), count.data_ptr()
            else:
                a = _capi.RowArgs.from_buffer_copy(self._row_template(i, di))
            a.row_offset = row_offset
            ins_al, outs_al = self.align[i]
            if sk.family == "attn":
                # pointers travel inside the tensor maps; check their alignment
                for opd, al in zip(sk.operands, ins_al):
                    if env[opd.op_id].data_ptr() % al:
                        raise _capi.MoltenError(f"input {opd.name!r} is not {al}-byte aligned as "
                                                f"kernel {self.entries[i].decode()} requires")
                if a.out % outs_al[0]:
                    raise _capi.MoltenError(f"output is not {outs_al[0]}-byte aligned as kernel "
                                            f"{self.entries[i].decode()} requires")
                mod.launch(self.entries[i], cfg, a, stream)
                continue
            inp, outp = a.inp, a.out        # (one array view each, not one per access)
            for opd, al in zip(sk.operands, ins_al):
                p = env[opd.op_id].data_ptr()
                if p % al:
                    raise _capi.MoltenError(f"input {opd.name!r} at {p:#x} is not {al}-byte aligned "
                                            f"as kernel {self.entries[i].decode()} requires")
                inp[opd.index] = p
            for o, al in zip(sk.outputs, outs_al):
                p = env[o.op_id].data_ptr()
                if p % al:
                    raise _capi.MoltenError(f"output at {p:#x} is not {al}-byte aligned "
                                            f"as kernel {self.entries[i].decode()} requires")
                outp[o.index] = p
            mod.launch(self.entries[i], cfg, a, stream)
        if DEBUG:
            torch.cuda.synchronize(di)
            bits = _capi.read_status(di, True)
            if bits:
                raise _capi.MoltenError(f"{self.gk.name}: a bounded wait ran out on device {di} "
                                        f"(status word {bits:#x})")
        return outs


def _empty_outputs(gk: GeneratedKernel) -> bool:
    """Every output of this specialisation has no elements (no rows or no
    columns): calls return empty tensors without a launch."""
    shapes = gk.plan.output_shapes if gk.plan is not None else []
    return bool(shapes) and all(any(int(d) == 0 for d in s) for s in shapes)


def _attn_tensor_2d(t):
    """[.., rows, cols] contiguous-row tensor as a 2-D [rows, cols] view."""
    return t.reshape(-1, t.shape[-1])


def _alignment_rules(sk):
    """Byte alignment each input / output pointer of a sub-kernel needs:
    16 for TMA sources and for 16-byte vector slots, the slot size for
    narrower slots, the element size for per-row scalars."""
    c = sk.config
    if sk.family == "attn":
        # TMA sources; P is written by TMA (16) or element by element (2)
        return [16, 16], [16 if c["rows_aligned"] else 2]
    if sk.family == "gemm":
        ins = [16 if o.last == "vec" else DTYPE_SIZE[o.dtype] for o in sk.operands]
        return ins, [16 for _ in sk.outputs]
    if sk.family == "causal":
        # 16-byte slots in and out; 32-byte zero stores need 32-byte rows
        return [16], [32 if c.get("w32") else 16]
    if sk.family == "split3":
        # VEC-element slots of the operand; plane stores of VEC bf16
        return ([min(16, c["vec"] * DTYPE_SIZE[sk.operands[0].dtype])],
                [min(16, 2 * c["vec"])])
    if sk.family == "rope":
        if c["scalar"]:
            return ([DTYPE_SIZE[o.dtype] for o in sk.operands],
                    [DTYPE_SIZE[o.dtype] for o in sk.outputs])
        from .emit_rope import rope_table_slot
        vec, tab = c["vec"], rope_table_slot(c)
        x = sk.operands[0]
        ins = [min(16, vec * DTYPE_SIZE[x.dtype])]
        ins += [min(16, tab * DTYPE_SIZE[o.dtype]) for o in sk.operands[1:]]
        return ins, [min(16, vec * DTYPE_SIZE[o.dtype]) for o in sk.outputs]
    vec = c.get("vec", 1)
    staged = set(c.get("staged", ())) if c.get("engine") == "tma" else set()
    ins = []
    for o in sk.operands:
        esz = DTYPE_SIZE[o.dtype]
        if o.index in staged:
            ins.append(16)
        elif o.last == "vec":
            ins.append(min(16, vec * esz))
        else:
            ins.append(esz)
    outs = [min(16, vec * DTYPE_SIZE[o.dtype]) if o.kind == "full" else DTYPE_SIZE[o.dtype]
            for o in sk.outputs]
    return ins, outs


class _HostPlan:
    """State ``CompiledKernel.run_host`` keeps per device and shapes."""


def host_row_blocks(rows: int, chunks: int) -> list:
    """[(r0, r1), ...] row blocks of a host-buffer call: equal blocks, but
    the last two 3/4 and 1/4 of one, so that the call's tail (the last
    block's kernel and download, after the last upload) is short (measured,
    RMSNorm*SiLU bf16 8192 x 3584 from host buffers: 8 equal blocks
    2.58-2.66 ms, 4 equal 2.59, 2048/2048/2048/1536/512 rows 2.51 ms).
    Empty blocks are dropped; the blocks tile [0, rows) in order."""
    chunks = max(1, int(chunks))
    wts = [4] * (chunks - 2) + [3, 1] if chunks >= 3 else [1] * chunks
    tot, acc, bounds = sum(wts), 0, []
    for wt in wts:
        r0 = rows * acc // tot
        acc += wt
        bounds.append((r0, rows * acc // tot))
    return [b for b in bounds if b[1] > b[0]]


@dataclass
class CompiledKernel:
    """A generated kernel bound to its cubin; call it with CUDA tensors."""
    name: str
    source: str
    config: KernelConfig
    _module: object = None
    kernel: Optional[GeneratedKernel] = None
    runtime: Optional["MoltenRuntime"] = None
    _specs: dict = field(default_factory=dict)
    _hosts: dict = field(default_factory=dict)

    def __call__(self, *tensors, out=None, stream=None, row_offset: int = 0):
        if self.kernel is None or self.runtime is None:
            raise RuntimeError(f"Kernel '{self.name}' not compiled. Call compile() first.")
        plan = self.kernel.plan
        if len(tensors) != len(plan.inputs):
            g = self.kernel.graph
            names = [g.ops[i].name or f"op{i}" for i in plan.inputs] if g else plan.inputs
            raise RuntimeError(f"{self.name} takes {len(plan.inputs)} tensors {names}, "
                               f"got {len(tensors)}")
        prepared = []
        for t in tensors:
            if not getattr(t, "is_cuda", False):
                raise RuntimeError(f"{self.name}: inputs must be CUDA tensors (got {type(t).__name__} "
                                   f"on {getattr(t, 'device', '?')})")
            prepared.append(t)
        dev = prepared[0].device
        for t in prepared[1:]:
            if t.device != dev:
                raise RuntimeError(f"{self.name}: all inputs must be on {dev}, got {t.device}")
        spec = self._spec_for(prepared)
        if not all(t.is_contiguous() for t in prepared):
            prepared = self._conform(spec, prepared)
        if out is not None:
            outs = list(out) if isinstance(out, (list, tuple)) else [out]
            self._check_outs(spec, outs, dev)
        else:
            outs = None
        res = spec.run(prepared, outs, stream, row_offset)
        return res[0] if len(res) == 1 else tuple(res)

    # -- specialisation -------------------------------------------------
    @staticmethod
    def _signature(tensors):
        # (torch.Size hashes and compares as the tuple of its dims)
        aligned = all(t.data_ptr() % 16 == 0 for t in tensors)
        return tuple([(t.dtype, t.shape) for t in tensors]) + (aligned,)

    def _spec_for(self, tensors) -> _Spec:
        sig = self._signature(tensors)
        spec = self._specs.get(sig)
        if spec is not None:
            return spec
        plan = self.kernel.plan
        shapes = {i: tuple(t.shape) for i, t in zip(plan.inputs, tensors)}
        dtypes = {i: _dtype_name(t) for i, t in zip(plan.inputs, tensors)}
        same = (all(tuple(plan.input_shapes[k]) == shapes[i] for k, i in enumerate(plan.inputs))
                and all(plan.input_dtypes[k] == dtypes[i] for k, i in enumerate(plan.inputs))
                and sig[-1])
        if same:
            gk = self.kernel
        else:
            if self.kernel.graph is None or self.kernel.group is None:
                raise RuntimeError(f"{self.name} was generated for {plan.input_shapes} "
                                   f"{plan.input_dtypes} and cannot be re-specialised")
            tune = dict(self.runtime.tune)
            if not sig[-1]:
                for fam in ("row", "ew", "rope"):
                    tune[fam] = dict(tune.get(fam) or {}, vec=1)
            gen = CodeGenerator(dtype=None, tune=tune)
            gk = gen.generate(self.kernel.graph, self.kernel.group, shapes, dtypes)
        cubin = None if _empty_outputs(gk) else \
            build_cubin(gk.source, gk.name, self.runtime.cache_dir, self.runtime.verbose)
        spec = _Spec(gk, cubin)
        self._specs[sig] = spec
        return spec

    @staticmethod
    def _conform(spec: _Spec, tensors):
        plan = spec.plan
        gemm_b = set()
        for sk in plan.kernels:
            if sk.family == "gemm" and not sk.config.get("split3"):
                # (an fp32 B is read whole by its split kernel: contiguous)
                gemm_b.add(sk.operands[sk.b_operand].op_id)
        out = []
        for op_id, t in zip(plan.inputs, tensors):
            if op_id in gemm_b and t.dim() == 2 and t.stride(1) == 1 \
                    and (t.stride(0) * t.element_size()) % 16 == 0:
                out.append(t)              # a column slice of B is fine for TMA
            else:
                out.append(t.contiguous())
        return out

    @staticmethod
    def _check_outs(spec: _Spec, outs, dev):
        plan = spec.plan
        if len(outs) != len(plan.outputs):
            raise RuntimeError(f"expected {len(plan.outputs)} output tensors, got {len(outs)}")
        for t, s, d in zip(outs, plan.output_shapes, spec.out_dtypes):
            if t.shape != tuple(s) or t.dtype != d or t.device != dev or not t.is_contiguous():
                raise RuntimeError(f"output must be a contiguous {d} tensor of shape {tuple(s)} "
                                   f"on {dev}")

    def specialization(self, *tensors) -> GeneratedKernel:
        """The GeneratedKernel that a call with these tensors runs."""
        return self._spec_for(list(tensors)).gk

    # -- host buffers ---------------------------------------------------
    def row_chunkable(self, tensors) -> Optional[list]:
        """Which of these (host) inputs are split by rows in ``run_host``:
        a list of flags when every output is 2-D [R, C] and every input is
        either 2-D [R, C'] (one row per output row) or has no row dimension
        (1-D, or all leading dims 1), and every sub-kernel is a row,
        elementwise or GEMM kernel (rows of the GEMM = rows of A); else None."""
        plan = self.kernel.plan
        if any(sk.family not in ("row", "ew", "gemm", "causal") for sk in plan.kernels):
            return None
        if any(len(s) != 2 for s in plan.output_shapes):
            return None
        rows = plan.output_shapes[0][0]
        # a GEMM's B goes up whole (its rows are K, not the output's rows)
        gemm_b = {sk.operands[sk.b_operand].op_id for sk in plan.kernels if sk.family == "gemm"}
        flags = []
        for op_id, t in zip(plan.inputs, tensors):
            s = tuple(t.shape)
            if op_id in gemm_b:
                flags.append(False)
            elif len(s) == 2 and s[0] == rows and rows > 1:
                flags.append(True)
            elif all(d == 1 for d in s[:-1]) or len(s) <= 1:
                flags.append(False)
            else:
                return None
        return flags if any(flags) else None

    def _host_plan(self, dev, tensors, flags, outs, chunks):
        """Streams, device slots and events of ``run_host`` for one device and
        one set of shapes, kept across calls (each call's work waits for the
        previous call's downloads before reusing the slots)."""
        torch = _torch()
        key = (dev.index, tuple((tuple(t.shape), t.dtype) for t in tensors),
               tuple((tuple(o.shape), o.dtype) for o in outs), chunks)
        hp = self._hosts.get(key)
        if hp is not None:
            return hp
        rows = outs[0].shape[0]
        bounds = host_row_blocks(rows, chunks)
        rmax = max(b1 - b0 for b0, b1 in bounds)
        nslot = 1 if len(bounds) == 1 else 2
        hp = _HostPlan()
        hp.bounds, hp.nslot, hp.last = bounds, nslot, None
        hp.dev_whole = [None if f else torch.empty(tuple(t.shape), dtype=t.dtype, device=dev)
                        for t, f in zip(tensors, flags)]
        hp.dev_split = [[torch.empty((rmax, t.shape[1]), dtype=t.dtype, device=dev)
                         for _ in range(nslot)] if f else None for t, f in zip(tensors, flags)]
        hp.dev_out = [[torch.empty((rmax, o.shape[1]), dtype=o.dtype, device=dev)
                       for _ in range(nslot)] for o in outs]
        hp.streams = tuple(torch.cuda.Stream(dev) for _ in range(3))
        hp.ev_up = [torch.cuda.Event() for _ in bounds]
        hp.ev_run = [torch.cuda.Event() for _ in bounds]
        hp.ev_down = [torch.cuda.Event() for _ in bounds]
        if len(self._hosts) > 8:
            self._hosts.clear()
        self._hosts[key] = hp
        return hp

    def run_host(self, *tensors, out=None, chunks: int = 5, row_offset: int = 0, device=None):
        """Host tensors in, host outputs back.  Row-indexed inputs are split
        into ``chunks`` blocks of rows (equal, except that the last two are
        3/4 and 1/4 of one); each block's upload, kernel and
        download run on three streams of ``device`` so that block i+1's
        upload, block i's kernel and block i-1's download overlap (PCIe is
        full duplex), through two device slots per tensor.  Inputs without a
        row dimension go up once per call.  Pinned host memory makes the
        copies asynchronous.  Returns the host output(s); the current stream
        of ``device`` waits for all of it, so events recorded on it around
        the call time the whole transfer.  Graphs that do not split by rows
        (see ``row_chunkable``) run as one block."""
        torch = _torch()
        dev = torch.device("cuda", torch.cuda.current_device() if device is None else device)
        plan = self.kernel.plan
        flags = self.row_chunkable(tensors) if chunks > 1 else None
        if flags is None:
            # one block: upload everything, run, download (any output shape)
            cur = torch.cuda.current_stream(dev)
            dev_in = [t.to(dev, non_blocking=True) for t in tensors]
            res = self(*dev_in, stream=cur.cuda_stream, row_offset=row_offset)
            res = list(res) if isinstance(res, tuple) else [res]
            if out is None:
                out = [torch.empty(tuple(r.shape), dtype=r.dtype, pin_memory=True) for r in res]
            outs = list(out) if isinstance(out, (list, tuple)) else [out]
            for o, r in zip(outs, res):
                o.copy_(r, non_blocking=True)
            return outs[0] if len(outs) == 1 else tuple(outs)
        rows = plan.output_shapes[0][0]
        chunks = max(1, min(int(chunks), rows))
        if out is None:
            out = [torch.empty(tuple(s), dtype=d, pin_memory=True)
                   for s, d in zip(plan.output_shapes, [_torch_dtype(x) for x in plan.output_dtypes])]
        outs = list(out) if isinstance(out, (list, tuple)) else [out]
        hp = self._host_plan(dev, tensors, flags, outs, chunks)
        cur = torch.cuda.current_stream(dev)
        # this call's work follows the caller's stream and the previous call
        # (whose slots it reuses)
        for s in hp.streams:
            s.wait_stream(cur)
            if hp.last is not None:
                s.wait_event(hp.last)
        s_up, s_run, s_down = hp.streams
        with torch.cuda.stream(s_up):
            for t, d in zip(tensors, hp.dev_whole):
                if d is not None:
                    d.copy_(t, non_blocking=True)
        nslot = hp.nslot
        for i, (r0, r1) in enumerate(hp.bounds):
            slot, n = i % nslot, r1 - r0
            with torch.cuda.stream(s_up):
                if i >= nslot:
                    s_up.wait_event(hp.ev_run[i - nslot])      # the slot's inputs were consumed
                for t, d in zip(tensors, hp.dev_split):
                    if d is not None:
                        d[slot][:n].copy_(t[r0:r1], non_blocking=True)
                hp.ev_up[i].record(s_up)
            with torch.cuda.stream(s_run):
                s_run.wait_event(hp.ev_up[i])
                if i >= nslot:
                    s_run.wait_event(hp.ev_down[i - nslot])    # the slot's outputs were read back
                args = [w if w is not None else d[slot][:n] for w, d in zip(hp.dev_whole, hp.dev_split)]
                self(*args, out=[o[slot][:n] for o in hp.dev_out], stream=s_run.cuda_stream,
                     row_offset=row_offset + r0)
                hp.ev_run[i].record(s_run)
            with torch.cuda.stream(s_down):
                s_down.wait_event(hp.ev_run[i])
                for o, d in zip(outs, hp.dev_out):
                    o[r0:r1].copy_(d[slot][:n], non_blocking=True)
                hp.ev_down[i].record(s_down)
        hp.last = hp.ev_down[len(hp.bounds) - 1]
        cur.wait_stream(s_down)
        return outs[0] if len(outs) == 1 else tuple(outs)


class MoltenRuntime:
    """Builds generated kernels into cubins and hands out callables."""

    def __init__(self, cache_dir: Optional[str] = None, verbose: bool = False,
                 tune: Optional[dict] = None):
        self.verbose = verbose
        self.cache_dir = Path(cache_dir) if cache_dir else default_cache_dir()
        self.cache_dir.mkdir(parents=True, exist_ok=True)
        self.tune = tune or {}
        self._compiled: dict = {}
        _capi.load_library()           # fail loudly when the runtime is missing

    def compile(self, kernel: GeneratedKernel) -> CompiledKernel:
        key = hashlib.sha256(kernel.source.encode()).hexdigest()[:16]
        ck = self._compiled.get(key)
        if ck is not None:
            return ck
        # a specialisation whose outputs are empty launches nothing: no cubin
        cubin = None if _empty_outputs(kernel) else \
            build_cubin(kernel.source, kernel.name, self.cache_dir, self.verbose)
        ck = CompiledKernel(name=kernel.name, source=kernel.source, config=kernel.config,
                            _module=str(cubin), kernel=kernel, runtime=self)
        sig = None
        if kernel.plan is not None:
            sig = tuple((_torch_dtype(d), tuple(s))
                        for d, s in zip(kernel.plan.input_dtypes, kernel.plan.input_shapes)) + (True,)
            ck._specs[sig] = _Spec(kernel, cubin)
        self._compiled[key] = ck
        if self.verbose and cubin is not None:
            print(f"molten: built {cubin.name}")
        return ck

    def clear_cache(self) -> None:
        if self.cache_dir.exists():
            for f in self.cache_dir.iterdir():
                if f.suffix in (".cubin", ".cu"):
                    f.unlink()
        self._compiled.clear()

    @staticmethod
    def read_status(device: int = 0, reset: bool = True) -> int:
        """Error bits set by kernels with bounded waits on ``device``."""
        return _capi.read_status(device, reset)
