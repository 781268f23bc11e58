"""Functional op layer over the hand-written sm_100a kernels.

Every hot op of the models is one function here with an explicit forward and
backward (no autograd inside).  Dispatch rule, per call:

* CUDA tensor, bf16, backend ``"custom"`` (default) -> the kernel in the
  in-tree extension ``meshtrain_b200.ops._C``.  If the extension is missing on
  a CUDA machine the call raises; there is no silent library fallback.
* anything else (CPU tensors, fp32, or backend ``"torch"``) -> a plain PyTorch
  restatement of the same math.  That path is the numerics oracle for the
  kernels, the fp32 parity path, and what runs on CPU-only hosts.

The reference runs all of these as stock PyTorch ops (reference
models/tiny_transformer.py:19-59, runtime/stage.py:28-36); here they are the
replacement kernels' entry points.
"""

from __future__ import annotations

import math
import os
import threading
from contextlib import contextmanager

import torch
import torch.nn.functional as F

_EXT = None
_EXT_ERR: str | None = None
_BACKEND = os.environ.get("MESHTRAIN_KERNELS", "custom")

EPI_BF16, EPI_GELU, EPI_RESID, EPI_DGELU, EPI_F32, EPI_SWIGLU = range(6)


# Kernel launches issued through this module since import (each binding call
# launches one kernel; the attention bindings report their own count).
LAUNCHES = 0
_MULTI_LAUNCH = {"attention_fwd": 1, "attention_bwd": 3}
_NO_LAUNCH = {"read_status"}


class _CountingExtension:
    """Proxy over the compiled module that counts kernel launches."""

    def __init__(self, ext):
        self._ext = ext

    def __getattr__(self, name):
        fn = getattr(self._ext, name)
        if name in _NO_LAUNCH or not callable(fn):
            return fn
        n = _MULTI_LAUNCH.get(name, 1)

        def call(*args, **kwargs):
            global LAUNCHES
            LAUNCHES += n
            return fn(*args, **kwargs)

        object.__setattr__(self, name, call)
        return call


def launches() -> int:
    return LAUNCHES


def _load():
    global _EXT, _EXT_ERR
    if _EXT is not None or _EXT_ERR is not None:
        return _EXT
    try:
        import importlib

        # MT_OPS_DEBUG=1: the debug-checks build (setup.py with MT_DEBUG_CHECKS=1)
        name = "meshtrain_b200.ops._C_debug" if os.environ.get("MT_OPS_DEBUG") == "1" else "meshtrain_b200.ops._C"
        _EXT = _CountingExtension(importlib.import_module(name))
    except Exception as exc:  # pragma: no cover - depends on the build
        _EXT_ERR = f"{type(exc).__name__}: {exc}"
    return _EXT


def extension():
    """The compiled kernel module; raises if it is not built."""
    ext = _load()
    if ext is None:
        raise RuntimeError(
            "meshtrain_b200 CUDA extension is not built (python setup.py build_ext --inplace): " + str(_EXT_ERR))
    return ext


def extension_available() -> bool:
    return _load() is not None


def backend() -> str:
    return _BACKEND


def set_backend(name: str) -> None:
    """``custom`` (hand-written kernels on CUDA) or ``torch`` (PyTorch ops everywhere)."""
    global _BACKEND
    if name not in ("custom", "torch"):
        raise ValueError(f"unknown kernel backend {name!r}")
    _BACKEND = name


@contextmanager
def use_backend(name: str):
    prev = _BACKEND
    set_backend(name)
    try:
        yield
    finally:
        set_backend(prev)


def _custom(*tensors: torch.Tensor) -> bool:
    """True when this call must go to the CUDA kernels."""
    t = tensors[0]
    if not (t.is_cuda and _BACKEND == "custom"):
        return False
    if any(x is not None and x.dtype not in (torch.bfloat16, torch.int64, torch.float32) for x in tensors):
        return False
    if t.dtype != torch.bfloat16:
        return False
    extension()  # raise loudly if the kernels are missing on a CUDA host
    return True


def _mat(x: torch.Tensor) -> torch.Tensor:
    """2-D row-major view suitable for TMA: unit column stride, row stride a
    multiple of 8 elements (16 bytes), 16-byte aligned base.  Rows whose width
    is not a multiple of 8 are copied into a padded buffer (the padding is
    never read: tensor maps carry the logical width)."""
    x2 = x.reshape(-1, x.shape[-1])
    if x2.stride(-1) == 1 and x2.stride(0) % 8 == 0 and x2.stride(0) >= x2.shape[1] and x2.data_ptr() % 16 == 0:
        return x2
    rows, cols = x2.shape
    ld = (cols + 7) // 8 * 8
    buf = torch.empty(rows, ld, dtype=x2.dtype, device=x2.device)
    buf[:, :cols] = x2
    return buf[:, :cols]


# ----------------------------------------------------------------------------- linear

def linear(x: torch.Tensor, w: torch.Tensor, b: torch.Tensor | None = None, *, gelu: bool = False,
           residual: torch.Tensor | None = None):
    """y = x W^T + b [+ residual]; with ``gelu`` returns (gelu(h), h)."""
    if _custom(x, w):
        ext = extension()
        x2, w2 = _mat(x), _mat(w)
        M, N = x2.shape[0], w2.shape[0]
        out = torch.empty(M, N, device=x.device, dtype=torch.bfloat16)
        if gelu:
            h = torch.empty_like(out)
            ext.gemm(x2, False, w2, False, out, EPI_GELU, b, None, h, 0.0)
            return out.view(*x.shape[:-1], N), h.view(*x.shape[:-1], N)
        if residual is not None:
            ext.gemm(x2, False, w2, False, out, EPI_RESID, b, _mat(residual), None, 0.0)
        else:
            ext.gemm(x2, False, w2, False, out, EPI_BF16, b, None, None, 0.0)
        return out.view(*x.shape[:-1], N)
    y = F.linear(x, w, b)
    if gelu:
        return F.gelu(y), y
    if residual is not None:
        y = y + residual
    return y


def linear_dgrad(dy: torch.Tensor, w: torch.Tensor, *, gelu_pre: torch.Tensor | None = None,
                 out: torch.Tensor | None = None) -> torch.Tensor:
    """dx = dy W  (times gelu'(gelu_pre) when given: the GELU backward fused in).

    ``out`` (a contiguous [M, N] bf16 tensor, e.g. a row block of a larger
    buffer) receives the result directly instead of a new tensor.
    """
    if _custom(dy, w):
        ext = extension()
        dy2, w2 = _mat(dy), _mat(w)
        M, N = dy2.shape[0], w2.shape[1]
        if out is None:
            out = torch.empty(M, N, device=dy.device, dtype=torch.bfloat16)
        elif tuple(out.shape) != (M, N) or out.dtype != torch.bfloat16 or not out.is_contiguous():
            raise ValueError("linear_dgrad: out must be a contiguous bf16 [M, N] tensor")
        if gelu_pre is not None:
            ext.gemm(dy2, False, w2, True, out, EPI_DGELU, None, _mat(gelu_pre), None, 0.0)
        else:
            ext.gemm(dy2, False, w2, True, out, EPI_BF16, None, None, None, 0.0)
        return out.view(*dy.shape[:-1], N)
    dx = dy @ w
    if gelu_pre is not None:
        dx = dx * gelu_grad(gelu_pre)
    if out is not None:
        out.copy_(dx)
        return out
    return dx


# Deferred weight gradients: inside ``deferred_wgrad()`` the weight-gradient GEMMs
# and bias column sums go to one side stream per device, so they fill the SMs that
# the critical-path kernels (input-gradient GEMMs, attention) leave idle in their
# last waves.  They only accumulate into gradient buffers that nothing reads until
# the block ends, and the block's exit makes the current stream wait for them.
_WGRAD = threading.local()
_WGRAD_STREAMS: dict[int, torch.cuda.Stream] = {}


def _wgrad_stream(device: torch.device) -> torch.cuda.Stream:
    idx = device.index if device.index is not None else torch.cuda.current_device()
    st = _WGRAD_STREAMS.get(idx)
    if st is None:
        st = _WGRAD_STREAMS[idx] = torch.cuda.Stream(device=idx)
    return st


@contextmanager
def deferred_wgrad(enabled: bool = True, timer=None):
    """Run ``linear_wgrad_`` calls of the block on a side stream; join on exit.

    ``timer.side_work(stream)``, when given, is called before each side-stream
    GEMM is enqueued, so the caller can bracket that work with CUDA events and
    count it as busy time of the device.
    """
    outer = getattr(_WGRAD, "used", None)
    if not enabled or outer is not None or not torch.cuda.is_available():
        yield
        return
    _WGRAD.used = set()
    _WGRAD.timer = timer
    try:
        yield
    finally:
        used, _WGRAD.used, _WGRAD.timer = _WGRAD.used, None, None
        for idx in used:
            torch.cuda.current_stream(idx).wait_stream(_WGRAD_STREAMS[idx])


def linear_wgrad_(dy: torch.Tensor, x: torch.Tensor, w_grad: torch.Tensor, b_grad: torch.Tensor | None = None) -> None:
    """w_grad += dy^T x (fp32 accumulate); b_grad += sum_t dy."""
    if _custom(dy, x) and w_grad.dtype == torch.float32:
        ext = extension()
        dy2, x2 = _mat(dy), _mat(x)
        used = getattr(_WGRAD, "used", None)
        if used is not None:
            side = _wgrad_stream(dy.device)
            side.wait_stream(torch.cuda.current_stream(dy.device))  # dy, x and the gradient buffers are ready
            timer = getattr(_WGRAD, "timer", None)
            if timer is not None:
                timer.side_work(side)
            with torch.cuda.stream(side):
                ext.gemm(dy2, True, x2, True, w_grad, EPI_F32, None, None, None, 1.0)
                if b_grad is not None:
                    ext.colsum_(dy2, b_grad)
            dy2.record_stream(side)  # the allocator keeps them until the side stream has read them
            x2.record_stream(side)
            used.add(side.device.index)
            return
        ext.gemm(dy2, True, x2, True, w_grad, EPI_F32, None, None, None, 1.0)
        if b_grad is not None:
            ext.colsum_(dy2, b_grad)
        return
    dy2, x2 = dy.reshape(-1, dy.shape[-1]), x.reshape(-1, x.shape[-1])
    if dy2.dtype == torch.bfloat16 and dy2.is_cuda:
        w_grad += (dy2.t() @ x2).to(w_grad.dtype)
    else:
        w_grad += (dy2.t().to(w_grad.dtype) @ x2.to(w_grad.dtype))
    if b_grad is not None:
        b_grad += dy2.to(b_grad.dtype).sum(0)


def gelu_grad(h: torch.Tensor) -> torch.Tensor:
    hf = h.float()
    cdf = 0.5 * (1.0 + torch.erf(hf / math.sqrt(2.0)))
    pdf = torch.exp(-0.5 * hf * hf) / math.sqrt(2.0 * math.pi)
    return (cdf + hf * pdf).to(h.dtype)


# SwiGLU: the fused gate/up weight stores rows in blocks of 32 = [16 gate | 16 up].

def interleave_gate_up(w_gate: torch.Tensor, w_up: torch.Tensor) -> torch.Tensor:
    F_, d = w_gate.shape
    g = w_gate.reshape(F_ // 16, 16, d)
    u = w_up.reshape(F_ // 16, 16, d)
    return torch.cat([g, u], dim=1).reshape(2 * F_, d)


def split_gate_up(raw: torch.Tensor):
    *lead, n2 = raw.shape
    r = raw.reshape(*lead, n2 // 32, 32)
    return r[..., :16].reshape(*lead, n2 // 2), r[..., 16:].reshape(*lead, n2 // 2)


def merge_gate_up(g: torch.Tensor, u: torch.Tensor) -> torch.Tensor:
    *lead, f = g.shape
    return torch.cat([g.reshape(*lead, f // 16, 16), u.reshape(*lead, f // 16, 16)], dim=-1).reshape(*lead, 2 * f)


def swiglu_linear(x: torch.Tensor, w_gu: torch.Tensor):
    """(silu(x Wg^T) * (x Wu^T), raw) with the interleaved fused weight."""
    if _custom(x, w_gu):
        ext = extension()
        x2, w2 = _mat(x), _mat(w_gu)
        M, N2 = x2.shape[0], w2.shape[0]
        out = torch.empty(M, N2 // 2, device=x.device, dtype=torch.bfloat16)
        raw = torch.empty(M, N2, device=x.device, dtype=torch.bfloat16)
        ext.gemm(x2, False, w2, False, out, EPI_SWIGLU, None, None, raw, 0.0)
        return out.view(*x.shape[:-1], N2 // 2), raw.view(*x.shape[:-1], N2)
    raw = F.linear(x, w_gu)
    g, u = split_gate_up(raw)
    return F.silu(g) * u, raw


def swiglu_bwd(dout: torch.Tensor, raw: torch.Tensor) -> torch.Tensor:
    if _custom(dout, raw):
        return extension().swiglu_bwd(dout.contiguous(), raw.contiguous())
    g, u = split_gate_up(raw.float())
    sg = torch.sigmoid(g)
    d = dout.float()
    dg = d * u * (sg * (1 + g * (1 - sg)))
    du = d * g * sg
    return merge_gate_up(dg, du).to(raw.dtype)


# ----------------------------------------------------------------------------- norms

def layernorm(x: torch.Tensor, g: torch.Tensor, b: torch.Tensor, eps: float = 1e-5):
    """(y, mean, rstd) with fp32 statistics."""
    if _custom(x, g, b):
        y, mean, rstd = extension().layernorm_fwd(x.contiguous(), g, b, eps)
        return y, mean, rstd
    xf = x.float()
    mean = xf.mean(-1)
    var = xf.var(-1, unbiased=False)
    rstd = torch.rsqrt(var + eps)
    y = F.layer_norm(x, (x.shape[-1],), g, b, eps)
    return y, mean.reshape(-1), rstd.reshape(-1)


def layernorm_bwd(dy, x, g, mean, rstd, dres, dg_acc, db_acc):
    if _custom(dy, x, g) and dg_acc.dtype == torch.float32:
        return extension().layernorm_bwd(dy.contiguous(), x.contiguous(), g, mean, rstd,
                                         None if dres is None else dres.contiguous(), dg_acc, db_acc)
    d = x.shape[-1]
    xf = x.reshape(-1, d).float()
    dyf = dy.reshape(-1, d).float()
    xh = (xf - mean[:, None]) * rstd[:, None]
    wdy = dyf * g.float()
    m1 = wdy.mean(-1, keepdim=True)
    m2 = (wdy * xh).mean(-1, keepdim=True)
    dx = rstd[:, None] * (wdy - m1 - xh * m2)
    dg_acc += (dyf * xh).sum(0).to(dg_acc.dtype)
    db_acc += dyf.sum(0).to(db_acc.dtype)
    if dres is not None:
        dx = dx + dres.reshape(-1, d).float()
    return dx.to(x.dtype).reshape(x.shape)


def rmsnorm(x: torch.Tensor, g: torch.Tensor, eps: float = 1e-5):
    if _custom(x, g):
        y, rstd = extension().rmsnorm_fwd(x.contiguous(), g, eps)
        return y, rstd
    xf = x.float()
    rstd = torch.rsqrt(xf.pow(2).mean(-1) + eps)
    y = (xf * rstd[..., None] * g.float()).to(x.dtype)
    return y, rstd.reshape(-1)


def rmsnorm_bwd(dy, x, g, rstd, dres, dg_acc):
    if _custom(dy, x, g) and dg_acc.dtype == torch.float32:
        return extension().rmsnorm_bwd(dy.contiguous(), x.contiguous(), g, rstd,
                                       None if dres is None else dres.contiguous(), dg_acc)
    d = x.shape[-1]
    xf = x.reshape(-1, d).float()
    dyf = dy.reshape(-1, d).float()
    xh = xf * rstd[:, None]
    wdy = dyf * g.float()
    m2 = (wdy * xh).mean(-1, keepdim=True)
    dx = rstd[:, None] * (wdy - xh * m2)
    dg_acc += (dyf * xh).sum(0).to(dg_acc.dtype)
    if dres is not None:
        dx = dx + dres.reshape(-1, d).float()
    return dx.to(x.dtype).reshape(x.shape)


# ----------------------------------------------------------------------------- embedding

def embedding(ids: torch.Tensor, tok: torch.Tensor, pos: torch.Tensor | None, seq_len: int) -> torch.Tensor:
    """tok[ids] (+ pos[t % seq_len]); returns [T, d]."""
    flat = ids.reshape(-1)
    if _custom(tok) and flat.is_cuda:
        return extension().embedding_fwd(flat, tok, pos, seq_len)
    out = F.embedding(flat, tok)
    if pos is not None:
        T = flat.shape[0]
        out = out + pos[torch.arange(T, device=flat.device) % seq_len]
    return out


def embedding_bwd_(ids, dy, tok_grad, pos_grad, seq_len: int) -> None:
    flat = ids.reshape(-1)
    dy2 = dy.reshape(-1, dy.shape[-1])
    if _custom(dy2) and tok_grad.dtype == torch.float32:
        extension().embedding_bwd(flat, dy2.contiguous(), tok_grad, pos_grad, seq_len)
        return
    tok_grad.index_add_(0, flat, dy2.to(tok_grad.dtype))
    if pos_grad is not None:
        T = flat.shape[0]
        pos_grad.index_add_(0, torch.arange(T, device=flat.device) % seq_len, dy2.to(pos_grad.dtype))


# ----------------------------------------------------------------------------- rope

def rope_(qk: torch.Tensor, seq_len: int, heads: int, head_dim: int, theta: float, inverse: bool = False) -> None:
    """Rotate-half RoPE in place on the first ``heads`` heads of each row of qk [T, >=heads*hd]."""
    if _custom(qk):
        extension().rope_(qk, seq_len, heads, head_dim, theta, inverse)
        return
    T = qk.shape[0]
    half = head_dim // 2
    pos = (torch.arange(T, device=qk.device) % seq_len).float()
    inv = theta ** (-2.0 * torch.arange(half, device=qk.device).float() / head_dim)
    ang = pos[:, None] * inv[None]
    cs, sn = torch.cos(ang), torch.sin(ang)
    if inverse:
        sn = -sn
    v = qk[:, : heads * head_dim].reshape(T, heads, head_dim).float()
    x1, x2 = v[..., :half], v[..., half:]
    o1 = x1 * cs[:, None] - x2 * sn[:, None]
    o2 = x2 * cs[:, None] + x1 * sn[:, None]
    qk[:, : heads * head_dim] = torch.cat([o1, o2], -1).reshape(T, heads * head_dim).to(qk.dtype)


# ----------------------------------------------------------------------------- attention

def attention(q, k, v, *, causal: bool = True, scale: float | None = None):
    """Flash attention over [B, S, H, hd] views (GQA when k/v have fewer heads).

    Returns (o [B,S,Hq,hd] contiguous, lse [B,Hq,S] fp32).
    """
    from meshtrain_b200.ops import attention_impl

    return attention_impl.forward(q, k, v, causal=causal, scale=scale)


def attention_bwd(dout, q, k, v, o, lse, *, causal: bool = True, scale: float | None = None, out=None):
    """Returns (dq, dk, dv) with the shapes of q, k, v (written into ``out`` views when given)."""
    from meshtrain_b200.ops import attention_impl

    return attention_impl.backward(dout, q, k, v, o, lse, causal=causal, scale=scale, out=out)


# ----------------------------------------------------------------------------- loss

def cross_entropy_chunk_(logits: torch.Tensor, vocab: int, targets: torch.Tensor, loss_sum: torch.Tensor,
                         loss_scale: float, grad_scale: float) -> None:
    """In place: logits[:, :vocab] -> (softmax - onehot) * grad_scale; loss_sum += sum ce * loss_scale."""
    if _custom(logits) and targets.is_cuda:
        extension().cross_entropy_(logits, vocab, targets.reshape(-1), loss_sum, loss_scale, grad_scale)
        return
    lg = logits[:, :vocab].float()
    tg = targets.reshape(-1)
    lse = torch.logsumexp(lg, -1)
    valid = (tg >= 0) & (tg < vocab)
    tgc = tg.clamp(0, vocab - 1)
    ce = (lse - lg.gather(1, tgc[:, None])[:, 0]) * valid
    loss_sum += ce.sum() * loss_scale
    grad = torch.softmax(lg, -1)
    grad[torch.arange(lg.shape[0], device=lg.device), tgc] -= 1.0
    grad *= (grad_scale * valid.float())[:, None]
    logits[:, :vocab] = grad.to(logits.dtype)


# ----------------------------------------------------------------------------- optimizer

def adam_(p, g, m, v, p_lowp, *, lr, beta1, beta2, eps, weight_decay, decoupled, step, grad_scale=1.0):
    """Fused Adam/AdamW on flat fp32 buffers (torch.optim semantics); optional bf16 copy-out."""
    bc1 = 1.0 - beta1 ** step
    bc2 = 1.0 - beta2 ** step
    if p.is_cuda and _BACKEND == "custom":
        extension().adam_(p, g, m, v, p_lowp, lr, beta1, beta2, eps, weight_decay, decoupled, bc1, bc2, grad_scale)
        return
    gg = g * grad_scale if grad_scale != 1.0 else g
    if decoupled:
        p.mul_(1 - lr * weight_decay)
    elif weight_decay:
        gg = gg + weight_decay * p
    m.mul_(beta1).add_(gg, alpha=1 - beta1)
    v.mul_(beta2).addcmul_(gg, gg, value=1 - beta2)
    denom = (v.sqrt() / math.sqrt(bc2)).add_(eps)
    p.addcdiv_(m, denom, value=-lr / bc1)
    if p_lowp is not None:
        p_lowp.copy_(p)


def read_status(device: int = 0) -> int:
    """Non-zero if a kernel on ``device`` gave up a bounded wait since the last call."""
    return int(extension().read_status(device))


def read_checks() -> int:
    """Failed-check codes (``kErrCheck*``) of the debug-checks build since the last call on the
    current device; always 0 with the release build."""
    return int(extension().read_checks())


def debug_checks_built() -> bool:
    return bool(extension().debug_checks_built())
