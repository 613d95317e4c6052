"""Named workloads of the benchmark set: graph + seeded synthetic inputs.

Shapes and value distributions are the benchmark set's (no dataset is
involved):

=========================  ==============================================
rmsnorm                    x fp32 [2048, 5120] ~ N(0,1); w = 1 + 0.1 N(0,1)
rmsnorm_silu_gate          x, g bf16 [rows, 3584] ~ N(0,1); w = 1 + 0.1 N(0,1);
                           rows 1 (decode), 2048 (prefill), 8192 (long)
softmax                    logits ~ N(0, 3^2), [32*2048, 2048] (as
                           [32, 2048, 2048]) or [4096, 32768]; fp32 / bf16;
                           optional causal mask
chain                      x, r bf16 [16384, 8192] ~ N(0,1); a, b, s ~ U(-1,1)
attention_score            q, k bf16 [32 heads, 2048, 128] ~ N(0,1); scale 1/sqrt(128)
rmsnorm_gemm               x bf16 [8192, 4096] ~ N(0,1), w = 1 + 0.1 N(0,1), then
                           B and bias as gemm_bias_gelu (GELU(rmsnorm(x, w) @ B + bias))
gemm_bias_gelu             A bf16 [8192, 4096] ~ N(0,1); B [4096, 14336] ~
                           N(0, 1/4096); bias [14336] ~ N(0, 0.02^2)
=========================  ==============================================

Values are drawn in fp32 from ``torch.Generator().manual_seed(seed)`` and
then cast, so a given (workload, seed, device type) always yields the same
tensors.
"""

from __future__ import annotations

from dataclasses import dataclass, field

from . import graphs


@dataclass
class Workload:
    name: str
    kind: str
    params: dict
    dtype: str
    # algorithmic work per call
    bytes_per_call: int = 0
    flops_per_call: int = 0
    input_names: list = field(default_factory=list)

    def graph(self, **over):
        p = dict(self.params)
        p.update(over)
        return graphs.BUILDERS[self.kind](dtype=self.dtype, **p)


def _esz(dtype):
    return 4 if dtype == "float32" else 2


def _rms(name, rows, cols, dtype, silu):
    kind = "rmsnorm_silu_gate" if silu else "rmsnorm"
    e = _esz(dtype)
    nbytes = rows * cols * e * (3 if silu else 2) + cols * e
    names = ["x", "w", "gate"] if silu else ["x", "w"]
    return Workload(name, kind, {"rows": rows, "cols": cols}, dtype, nbytes, 0, names)


def _visible_fraction(rows: int, cols: int) -> float:
    """Share of a causal mask's entries that are visible (col <= row mod
    cols), i.e. the logits a causal softmax has to read."""
    full, rem = divmod(rows, cols)
    per_period = cols * (cols + 1) // 2
    tail = rem * (rem + 1) // 2
    return (full * per_period + tail) / (rows * cols)


def _softmax(name, shape, dtype, causal):
    n = 1
    for d in shape:
        n *= d
    cols = shape[-1]
    reads = n if not causal else round(n * _visible_fraction(n // cols, cols))
    return Workload(name, "softmax", {"shape": tuple(shape), "causal": causal}, dtype,
                    (reads + n) * _esz(dtype), 0, ["logits"])


def _rope(name, batch, seq, heads, head_dim, dtype):
    """RoPE (ops.py:24-35): x [batch, seq, heads, head_dim] in dtype, fp32
    cos/sin tables [seq, head_dim/2]; bytes = x in + out + both tables."""
    n = batch * seq * heads * head_dim
    nbytes = 2 * n * _esz(dtype) + 2 * seq * (head_dim // 2) * 4
    return Workload(name, "rope", {"batch": batch, "seq": seq, "heads": heads,
                                   "head_dim": head_dim}, dtype, nbytes, 0, ["x", "cos", "sin"])


WORKLOADS = {w.name: w for w in [
    _rms("rmsnorm_f32_2048x5120", 2048, 5120, "float32", False),
    _rms("rmsnorm_silu_bf16_1x3584", 1, 3584, "bfloat16", True),
    _rms("rmsnorm_silu_bf16_2048x3584", 2048, 3584, "bfloat16", True),
    _rms("rmsnorm_silu_bf16_8192x3584", 8192, 3584, "bfloat16", True),
    _softmax("softmax_f32_65536x2048", (32, 2048, 2048), "float32", False),
    _softmax("softmax_f32_65536x2048_causal", (32, 2048, 2048), "float32", True),
    _softmax("softmax_bf16_65536x2048", (32, 2048, 2048), "bfloat16", False),
    _softmax("softmax_bf16_65536x2048_causal", (32, 2048, 2048), "bfloat16", True),
    _softmax("softmax_f32_4096x32768", (4096, 32768), "float32", False),
    _softmax("softmax_f32_4096x32768_causal", (4096, 32768), "float32", True),
    _softmax("softmax_bf16_4096x32768", (4096, 32768), "bfloat16", False),
    _softmax("softmax_bf16_4096x32768_causal", (4096, 32768), "bfloat16", True),
    Workload("chain_bf16_16384x8192", "chain", {"rows": 16384, "cols": 8192}, "bfloat16",
             3 * 16384 * 8192 * 2 + 3 * 8192 * 2, 0, ["x", "r", "a", "b", "s"]),
    _rope("rope_bf16_4x4096x32x128", 4, 4096, 32, 128, "bfloat16"),
    Workload("attention_score_bf16_32x2048x2048x128", "attention_score",
             {"heads": 32, "m": 2048, "n": 2048, "d": 128}, "bfloat16",
             (2 * 32 * 2048 * 128 + 32 * 2048 * 2048) * 2, 2 * 32 * 2048 * 2048 * 128,
             ["q", "k"]),
    Workload("rmsnorm_gemm_bf16_64x4096x14336", "rmsnorm_gemm",
             {"m": 64, "k": 4096, "n": 14336}, "bfloat16",
             (64 * 4096 + 4096 + 4096 * 14336 + 14336 + 64 * 14336) * 2,
             2 * 64 * 4096 * 14336, ["x", "w", "B", "bias"]),
    Workload("rmsnorm_gemm_bf16_8192x4096x14336", "rmsnorm_gemm",
             {"m": 8192, "k": 4096, "n": 14336}, "bfloat16",
             (8192 * 4096 + 4096 + 4096 * 14336 + 14336 + 8192 * 14336) * 2,
             2 * 8192 * 4096 * 14336, ["x", "w", "B", "bias"]),
    Workload("gemm_bias_gelu_bf16_8192x4096x14336", "gemm_bias_gelu",
             {"m": 8192, "k": 4096, "n": 14336}, "bfloat16",
             (8192 * 4096 + 4096 * 14336 + 14336 + 8192 * 14336) * 2,
             2 * 8192 * 4096 * 14336, ["A", "B", "bias"]),
]}

HEADLINE = "rmsnorm_silu_bf16_8192x3584"


def scaled(w: Workload, **params) -> Workload:
    """The same workload kind at other sizes (for small parity cases)."""
    p = dict(w.params)
    p.update(params)
    if w.kind in ("rmsnorm", "rmsnorm_silu_gate"):
        return _rms(w.name + "_scaled", p["rows"], p["cols"], w.dtype, w.kind != "rmsnorm")
    if w.kind == "softmax":
        return _softmax(w.name + "_scaled", p["shape"], w.dtype, p["causal"])
    if w.kind == "chain":
        r, c = p["rows"], p["cols"]
        return Workload(w.name + "_scaled", "chain", {"rows": r, "cols": c}, w.dtype,
                        3 * r * c * 2 + 3 * c * 2, 0, list(w.input_names))
    if w.kind == "rope":
        return _rope(w.name + "_scaled", p["batch"], p["seq"], p["heads"], p["head_dim"], w.dtype)
    if w.kind == "attention_score":
        h, m, n, d = p["heads"], p["m"], p["n"], p["d"]
        return Workload(w.name + "_scaled", "attention_score", dict(p), w.dtype,
                        (h * m * d + h * n * d + h * m * n) * 2, 2 * h * m * n * d, ["q", "k"])
    m, k, n = p["m"], p["k"], p["n"]
    if w.kind == "rmsnorm_gemm":
        return Workload(w.name + "_scaled", "rmsnorm_gemm", {"m": m, "k": k, "n": n}, w.dtype,
                        (m * k + k + k * n + n + m * n) * 2, 2 * m * k * n, list(w.input_names))
    return Workload(w.name + "_scaled", "gemm_bias_gelu", {"m": m, "k": k, "n": n}, w.dtype,
                    (m * k + k * n + n + m * n) * 2, 2 * m * k * n, list(w.input_names))


def make_inputs(w: Workload, seed: int = 0, device="cpu") -> list:
    """Seeded inputs of a workload, in graph-input order, as torch tensors."""
    import torch
    dev = torch.device(device)
    g = torch.Generator(device=dev)
    g.manual_seed(seed)
    dt = {"float32": torch.float32, "bfloat16": torch.bfloat16, "float16": torch.float16}[w.dtype]
    p = w.params

    def normal(shape, mean=0.0, std=1.0):
        t = torch.randn(*shape, generator=g, device=dev, dtype=torch.float32)
        if std != 1.0:
            t.mul_(std)
        if mean != 0.0:
            t.add_(mean)
        return t.to(dt)

    def uniform(shape, lo, hi):
        t = torch.rand(*shape, generator=g, device=dev, dtype=torch.float32)
        return t.mul_(hi - lo).add_(lo).to(dt)

    if w.kind in ("rmsnorm", "rmsnorm_silu_gate"):
        rows, cols = p["rows"], p["cols"]
        x = normal((rows, cols))
        wt = normal((cols,), 1.0, 0.1)
        if w.kind == "rmsnorm":
            return [x, wt]
        gate = normal((rows, cols))
        return [x, wt, gate]
    if w.kind == "softmax":
        return [normal(p["shape"], 0.0, 3.0)]
    if w.kind == "chain":
        rows, cols = p["rows"], p["cols"]
        x = normal((rows, cols))
        r = normal((rows, cols))
        a = uniform((cols,), -1.0, 1.0)
        b = uniform((cols,), -1.0, 1.0)
        s = uniform((cols,), -1.0, 1.0)
        return [x, r, a, b, s]
    if w.kind == "attention_score":
        return [normal((p["heads"], p["m"], p["d"])), normal((p["heads"], p["n"], p["d"]))]
    if w.kind == "rope":
        x = normal((p["batch"], p["seq"], p["heads"], p["head_dim"]))
        ang = torch.rand(p["seq"], p["head_dim"] // 2, generator=g, device=dev,
                         dtype=torch.float32) * 6.283185307179586
        return [x, torch.cos(ang), torch.sin(ang)]
    if w.kind == "rmsnorm_gemm":
        m, k, n = p["m"], p["k"], p["n"]
        x = normal((m, k))
        wt = normal((k,), 1.0, 0.1)
        B = normal((k, n), 0.0, (1.0 / k) ** 0.5)
        bias = normal((n,), 0.0, 0.02)
        return [x, wt, B, bias]
    if w.kind == "gemm_bias_gelu":
        m, k, n = p["m"], p["k"], p["n"]
        A = normal((m, k))
        B = normal((k, n), 0.0, (1.0 / k) ** 0.5)
        bias = normal((n,), 0.0, 0.02)
        return [A, B, bias]
    raise KeyError(w.kind)


def input_shapes(w: Workload) -> list:
    """Shapes of ``make_inputs(w)`` without allocating anything."""
    p = w.params
    if w.kind == "rmsnorm":
        return [(p["rows"], p["cols"]), (p["cols"],)]
    if w.kind == "rmsnorm_silu_gate":
        return [(p["rows"], p["cols"]), (p["cols"],), (p["rows"], p["cols"])]
    if w.kind == "softmax":
        return [tuple(p["shape"])]
    if w.kind == "chain":
        r, c = p["rows"], p["cols"]
        return [(r, c), (r, c), (c,), (c,), (c,)]
    if w.kind == "gemm_bias_gelu":
        return [(p["m"], p["k"]), (p["k"], p["n"]), (p["n"],)]
    if w.kind == "rmsnorm_gemm":
        return [(p["m"], p["k"]), (p["k"],), (p["k"], p["n"]), (p["n"],)]
    if w.kind == "attention_score":
        return [(p["heads"], p["m"], p["d"]), (p["heads"], p["n"], p["d"])]
    if w.kind == "rope":
        half = (p["seq"], p["head_dim"] // 2)
        return [(p["batch"], p["seq"], p["heads"], p["head_dim"]), half, half]
    raise KeyError(w.kind)


def input_dtypes(w: Workload) -> list:
    """Dtypes of ``make_inputs(w)`` (RoPE tables are fp32)."""
    n = len(input_shapes(w))
    if w.kind == "rope":
        return [w.dtype, "float32", "float32"]
    return [w.dtype] * n


GEMM_KINDS = ("gemm_bias_gelu", "rmsnorm_gemm")
