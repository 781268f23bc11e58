"""Capability probes: tiny forward/backward runs of each model operator per dtype.

Results (and errors) are cached; the planner excludes workers whose probes
fail for an op a model needs (reference worker/capabilities.py:24-115).
"""

from __future__ import annotations

import torch
import torch.nn.functional as F

_DTYPES = {"float32": torch.float32, "float16": torch.float16, "bfloat16": torch.bfloat16, "float64": torch.float64}


def _grad_probe(fn):
    def run(dev, dt):
        x = torch.randn(4, 8, device=dev, dtype=dt, requires_grad=True)
        y = fn(x)
        y.float().sum().backward()
        return x.grad is not None
    return run


def _sdpa(dev, dt):
    q = torch.randn(1, 2, 4, 8, device=dev, dtype=dt, requires_grad=True)
    F.scaled_dot_product_attention(q, q, q, is_causal=True).float().sum().backward()
    return True


def _embedding(dev, dt):
    w = torch.randn(10, 8, device=dev, dtype=dt, requires_grad=True)
    F.embedding(torch.tensor([1, 2, 3], device=dev), w).float().sum().backward()
    return True


def _cross_entropy(dev, dt):
    x = torch.randn(4, 5, device=dev, dtype=dt, requires_grad=True)
    F.cross_entropy(x.float(), torch.tensor([0, 1, 2, 3], device=dev)).backward()
    return True


def _adamw(dev, dt):
    p = torch.nn.Parameter(torch.randn(8, device=dev, dtype=dt))
    p.grad = torch.ones_like(p)
    torch.optim.AdamW([p], lr=1e-3).step()
    return True


def _dtype(dev, dt):
    return torch.ones(2, device=dev, dtype=dt).sum().item() == 2


PROBES = {
    "matmul": _grad_probe(lambda x: x @ x.t()),
    "linear": _grad_probe(lambda x: F.linear(x, torch.ones(3, 8, device=x.device, dtype=x.dtype))),
    "gelu": _grad_probe(F.gelu),
    "silu": _grad_probe(F.silu),
    "layer_norm": _grad_probe(lambda x: F.layer_norm(x, (8,))),
    "rms_norm": _grad_probe(lambda x: x * torch.rsqrt(x.float().pow(2).mean(-1, keepdim=True) + 1e-5).to(x.dtype)),
    "softmax": _grad_probe(lambda x: torch.softmax(x, -1)),
    "sdpa": _sdpa,
    "embedding": _embedding,
    "cross_entropy": _cross_entropy,
    "adamw": _adamw,
    "dtype": _dtype,
}


class CapabilityProber:
    def __init__(self, device: torch.device, supports_dtype=None):
        self.device = device
        self.supports_dtype = supports_dtype or (lambda dt: True)
        self.results: dict[tuple[str, str], bool] = {}
        self.errors: dict[str, str] = {}

    def supports(self, op: str, dtype: str = "float32") -> bool:
        key = (op, dtype)
        if key in self.results:
            return self.results[key]
        dt = _DTYPES.get(dtype)
        ok = False
        if dt is not None and self.supports_dtype(dt):
            probe = PROBES.get(op)
            if probe is None:
                ok = True  # unknown ops are assumed supported: torch reports real failures
            else:
                try:
                    ok = bool(probe(self.device, dt))
                except Exception as exc:  # noqa: BLE001 - any failure means "unsupported"
                    self.errors[f"{op}:{dtype}"] = f"{type(exc).__name__}: {exc}"[:200]
        self.results[key] = ok
        return ok

    def report(self, ops=("matmul", "linear", "gelu", "layer_norm", "softmax", "sdpa", "embedding",
                          "cross_entropy", "adamw"), dtypes=("float32", "bfloat16", "float16")) -> dict:
        table = {op: [dt for dt in dtypes if self.supports(op, dt)] for op in ops}
        return {"ops": table, "dtypes": [dt for dt in dtypes if self.supports("dtype", dt)],
                "probe_errors": dict(self.errors)}
