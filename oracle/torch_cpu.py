"""The reference's CPU path, restated in torch -- TEST/BASELINE INFRASTRUCTURE.

Used only by bench.py (the timed ``cpu_baseline`` and the ``--impl
reference`` arm) and by tests; never by the product path.  Each function
restates one function of the reference's ``benchmarks/ops.py`` (the CPU
semantics its paper benchmarks against), run as written: eager torch on the
caller's tensors, in their dtype, on the host's cores.

* rmsnorm            benchmarks/ops.py:13-16
* silu_gate          benchmarks/ops.py:19-21
* rmsnorm_silu_gate  benchmarks/ops.py:38-42
* softmax            benchmarks/ops.py:45-47 (plus an additive causal mask)
* gelu (tanh)        benchmarks/ops.py:50-52
* chain              the 8-op chain composed from the ops above
* gemm_bias_gelu     torch.matmul as benchmarks/ops.py:58, + bias, GELU
* rope               benchmarks/ops.py:24-35
* rmsnorm_gemm       rmsnorm, then gemm_bias_gelu
* attention_score    benchmarks/ops.py:55-59
"""

from __future__ import annotations

import torch
import torch.nn.functional as F


def rmsnorm(x, w, eps=1e-6):
    rms = torch.sqrt(x.pow(2).mean(-1, keepdim=True) + eps)
    return x / rms * w


def silu_gate(x, gate):
    return F.silu(gate) * x


def rmsnorm_silu_gate(x, w, gate, eps=1e-6):
    return silu_gate(rmsnorm(x, w, eps), gate)


def causal_mask(rows, cols, dtype, period=None, row_offset=0):
    p = period or cols
    r = (torch.arange(rows) + row_offset) % p
    c = torch.arange(cols)
    m = torch.zeros(rows, cols, dtype=dtype)
    return m.masked_fill(c[None, :] > r[:, None], float("-inf"))


def softmax(x, causal=False, row_offset=0):
    if causal:
        x2 = x.reshape(-1, x.shape[-1])
        x = (x2 + causal_mask(x2.shape[0], x2.shape[1], x.dtype, row_offset=row_offset)).reshape(x.shape)
    return F.softmax(x, dim=-1)


def gelu(x):
    return F.gelu(x, approximate="tanh")


def chain(x, r, a, b, s):
    y = gelu(x * a + b) * s + r
    y = torch.clamp(y, -6.0, 6.0)
    return y * 0.5 + r


def gemm_bias_gelu(A, B, bias):
    return gelu(torch.matmul(A, B) + bias)


def rope(x, cos, sin):
    """x (batch, seq, heads, head_dim), cos/sin (seq, head_dim/2)."""
    xr = x.float().reshape(*x.shape[:-1], -1, 2)
    x0, x1 = xr[..., 0], xr[..., 1]
    c = cos.unsqueeze(0).unsqueeze(2)
    s = sin.unsqueeze(0).unsqueeze(2)
    out = torch.stack([x0 * c - x1 * s, x0 * s + x1 * c], dim=-1).flatten(-2)
    return out.to(x.dtype)


def rmsnorm_gemm(x, w, B, bias, eps=1e-6):
    return gemm_bias_gelu(rmsnorm(x, w, eps), B, bias)


def attention_score(q, k, scale):
    """softmax(q @ k^T * scale) over the last dim (benchmarks/ops.py:55-59)."""
    return F.softmax(torch.matmul(q, k.transpose(-2, -1)) * scale, dim=-1)


def run_workload(kind: str, tensors, params: dict):
    """Evaluate a named workload kind on CPU tensors."""
    if kind == "rmsnorm":
        return rmsnorm(*tensors)
    if kind == "rmsnorm_silu_gate":
        return rmsnorm_silu_gate(*tensors)
    if kind == "softmax":
        return softmax(tensors[0], causal=params.get("causal", False))
    if kind == "chain":
        return chain(*tensors)
    if kind == "gemm_bias_gelu":
        return gemm_bias_gelu(*tensors)
    if kind == "rope":
        return rope(*tensors)
    if kind == "rmsnorm_gemm":
        return rmsnorm_gemm(*tensors)
    if kind == "attention_score":
        return attention_score(*tensors, params["d"] ** -0.5)
    raise KeyError(kind)
