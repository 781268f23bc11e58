"""Causal (GQA) attention forward/backward dispatch.

Layouts: q [B, S, Hq, hd], k/v [B, S, Hk, hd] (strided views into a packed
QKV row are fine), o [B, S, Hq, hd], lse [B, Hq, S] fp32 natural-log
logsumexp of the scaled scores.

* CUDA + bf16 + backend ``custom``: the tcgen05 flash-attention kernels in the
  extension (``attention_fwd`` / ``attention_bwd``).
* backend ``torch`` on CUDA: PyTorch's fused SDPA flash kernels (the reference's
  own path, reference models/tiny_transformer.py:47) - kept for A/B timing.
* CPU / fp32: exact math in fp32 (the numerics oracle).
"""

from __future__ import annotations

import math

import torch

from meshtrain_b200 import ops as _ops


def _has_kernel() -> bool:
    ext = _ops._load()
    return ext is not None and hasattr(ext, "attention_fwd")


def _use_kernel(q: torch.Tensor) -> bool:
    if not (q.is_cuda and q.dtype == torch.bfloat16 and _ops.backend() == "custom"):
        return False
    if not _has_kernel():
        raise RuntimeError("meshtrain_b200: attention kernel missing from the CUDA extension")
    return True


def _rows(t: torch.Tensor) -> torch.Tensor:
    """Ensure [B,S,H,hd] with unit stride on hd and 16-byte aligned rows."""
    if t.stride(-1) != 1 or t.stride(-2) != t.shape[-1] or t.stride(1) % 8 or t.data_ptr() % 16:
        t = t.contiguous()
    return t


def _expand_kv(k: torch.Tensor, hq: int) -> torch.Tensor:
    hk = k.shape[2]
    return k if hk == hq else k.repeat_interleave(hq // hk, dim=2)


def _reference_fwd(q, k, v, causal, scale):
    B, S, Hq, hd = q.shape
    kf, vf = _expand_kv(k, Hq).float(), _expand_kv(v, Hq).float()
    qf = q.float()
    s = torch.einsum("bqhd,bkhd->bhqk", qf, kf) * scale
    if causal:
        mask = torch.ones(S, S, dtype=torch.bool, device=q.device).triu(1)
        s = s.masked_fill(mask, float("-inf"))
    lse = torch.logsumexp(s, -1)
    p = torch.exp(s - lse[..., None])
    o = torch.einsum("bhqk,bkhd->bqhd", p, vf)
    return o.to(q.dtype), lse


def _reference_bwd(dout, q, k, v, o, lse, causal, scale):
    B, S, Hq, hd = q.shape
    Hk = k.shape[2]
    kf, vf = _expand_kv(k, Hq).float(), _expand_kv(v, Hq).float()
    qf, of, dof = q.float(), o.float(), dout.float()
    s = torch.einsum("bqhd,bkhd->bhqk", qf, kf) * scale
    if causal:
        mask = torch.ones(S, S, dtype=torch.bool, device=q.device).triu(1)
        s = s.masked_fill(mask, float("-inf"))
    p = torch.exp(s - lse[..., None])
    dv = torch.einsum("bhqk,bqhd->bkhd", p, dof)
    dp = torch.einsum("bqhd,bkhd->bhqk", dof, vf)
    delta = (dof * of).sum(-1).permute(0, 2, 1)  # [B,H,S]
    ds = p * (dp - delta[..., None])
    dq = torch.einsum("bhqk,bkhd->bqhd", ds, kf) * scale
    dk = torch.einsum("bhqk,bqhd->bkhd", ds, qf) * scale
    if Hk != Hq:
        g = Hq // Hk
        dk = dk.reshape(B, S, Hk, g, hd).sum(3)
        dv = dv.reshape(B, S, Hk, g, hd).sum(3)
    return dq.to(q.dtype), dk.to(k.dtype), dv.to(v.dtype)


def forward(q, k, v, *, causal=True, scale=None):
    hd = q.shape[-1]
    scale = 1.0 / math.sqrt(hd) if scale is None else scale
    if _use_kernel(q):
        q, k, v = _rows(q), _rows(k), _rows(v)
        return _ops.extension().attention_fwd(q, k, v, causal, scale)
    if q.is_cuda and q.dtype in (torch.bfloat16, torch.float16):
        return _sdpa_forward(q, k, v, causal, scale)
    return _reference_fwd(q, k, v, causal, scale)


class _SdpaGraph:
    """Autograd graph of a library SDPA call, returned in place of ``lse``."""

    def __init__(self, leaves, out):
        self.leaves, self.out = leaves, out


def _sdpa_forward(q, k, v, causal, scale):
    Hq = q.shape[2]
    with torch.enable_grad():
        leaves = [t.detach().requires_grad_() for t in (q, k, v)]
        qt = leaves[0].transpose(1, 2)
        kt = _expand_kv(leaves[1], Hq).transpose(1, 2)
        vt = _expand_kv(leaves[2], Hq).transpose(1, 2)
        out = torch.nn.functional.scaled_dot_product_attention(qt, kt, vt, is_causal=causal, scale=scale)
    return out.detach().transpose(1, 2).contiguous(), _SdpaGraph(leaves, out)


def backward(dout, q, k, v, o, lse, *, causal=True, scale=None, out=None):
    """``out`` = optional (dq, dk, dv) [B,S,H,hd] views to write into (e.g. one packed dQKV buffer)."""
    hd = q.shape[-1]
    scale = 1.0 / math.sqrt(hd) if scale is None else scale
    if _use_kernel(q):
        q, k, v, o, dout = _rows(q), _rows(k), _rows(v), _rows(o), _rows(dout)
        dq, dk, dv = out if out is not None else (None, None, None)
        return tuple(_ops.extension().attention_bwd(dout, q, k, v, o, lse, causal, scale, dq, dk, dv))
    if isinstance(lse, _SdpaGraph):
        grads = tuple(torch.autograd.grad(lse.out, lse.leaves, dout.transpose(1, 2)))
    else:
        grads = _reference_bwd(dout, q, k, v, o, lse, causal, scale)
    if out is not None:
        for dst, g in zip(out, grads):
            dst.copy_(g)
        return tuple(out)
    return grads
