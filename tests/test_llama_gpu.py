"""Llama-8B shapes on the GPU kernels against fp32 PyTorch references.

Shapes of the 8B decoder: d_model 4096, 32 query / 8 KV heads of 128, SwiGLU
hidden 14336, RoPE theta 500000, sequences of 4096 tokens.  The block test
compares one ``LlamaBlock`` (custom kernels, bf16) forward and backward with
an independent fp32 formula of the same block under autograd.
"""

import math

import pytest
import torch
import torch.nn.functional as F

from meshtrain_b200 import ops
from meshtrain_b200.ops import attention_impl

pytestmark = pytest.mark.gpu

D, H, HK, HD, FFN, THETA = 4096, 32, 8, 128, 14336, 500000.0


def _close(out, ref, tol):
    out, ref = out.float(), ref.float()
    scale = ref.abs().max().item() + 1e-6
    err = (out - ref).abs().max().item()
    assert err <= tol * scale, f"max abs err {err:.3e} vs scale {scale:.3e}"


def _rel_l2(out, ref):
    out, ref = out.float(), ref.float()
    return ((out - ref).norm() / (ref.norm() + 1e-12)).item()


@pytest.fixture(autouse=True)
def _custom_kernels():
    torch.manual_seed(0)
    ops.set_backend("custom")
    yield
    torch.cuda.synchronize()
    assert ops.read_status(torch.cuda.current_device()) == 0


def test_gqa_attention_seq4096_hd128():
    B, S = 1, 4096
    q = torch.randn(B, S, H, HD, device="cuda").to(torch.bfloat16)
    k = torch.randn(B, S, HK, HD, device="cuda").to(torch.bfloat16)
    v = torch.randn(B, S, HK, HD, device="cuda").to(torch.bfloat16)
    do = torch.randn(B, S, H, HD, device="cuda").to(torch.bfloat16)
    scale = 1.0 / math.sqrt(HD)
    o, lse = ops.attention(q, k, v, causal=True)
    o_ref, lse_ref = attention_impl._reference_fwd(q, k, v, True, scale)
    _close(o, o_ref, 2e-2)
    _close(lse, lse_ref, 1e-3)
    dq, dk, dv = ops.attention_bwd(do, q, k, v, o, lse, causal=True)
    rq, rk, rv = attention_impl._reference_bwd(do, q, k, v, o_ref, lse_ref, True, scale)
    for got, want in ((dq, rq), (dk, rk), (dv, rv)):
        _close(got, want, 3e-2)
        assert _rel_l2(got, want) < 1e-2


def test_swiglu_epilogue_ffn14336():
    M = 1024
    x = (torch.randn(M, D, device="cuda") * 0.5).to(torch.bfloat16)
    wg = (torch.randn(FFN, D, device="cuda") * 0.02).to(torch.bfloat16)
    wu = (torch.randn(FFN, D, device="cuda") * 0.02).to(torch.bfloat16)
    act, raw = ops.swiglu_linear(x, ops.interleave_gate_up(wg, wu))
    g = x.float() @ wg.float().t()
    u = x.float() @ wu.float().t()
    rg, ru = ops.split_gate_up(raw)
    _close(rg, g, 2e-2)
    _close(ru, u, 2e-2)
    _close(act, F.silu(g) * u, 2e-2)
    dout = torch.randn(M, FFN, device="cuda").to(torch.bfloat16)
    draw = ops.swiglu_bwd(dout, raw)
    # d/dg silu(g) u = u * s (1 + g (1 - s)),  d/du = silu(g)
    gf, uf = rg.float(), ru.float()
    s = torch.sigmoid(gf)
    dg = dout.float() * uf * s * (1 + gf * (1 - s))
    du = dout.float() * F.silu(gf)
    _close(draw, ops.merge_gate_up(dg, du), 2e-2)


def _rope(x, theta):
    """Rotate-half rotary embedding of x [B, S, heads, hd] by absolute position."""
    B, S, n, hd = x.shape
    half = hd // 2
    inv = theta ** (-torch.arange(half, device=x.device, dtype=torch.float64) * 2.0 / hd)
    ang = torch.arange(S, device=x.device, dtype=torch.float64)[:, None] * inv[None]
    cos, sin = ang.cos().float()[None, :, None], ang.sin().float()[None, :, None]
    x1, x2 = x[..., :half], x[..., half:]
    return torch.cat([x1 * cos - x2 * sin, x2 * cos + x1 * sin], dim=-1)


def _rms(x, w, eps):
    return x * torch.rsqrt(x.pow(2).mean(-1, keepdim=True) + eps) * w


def _llama_block_fp32(x, p, eps):
    """Pre-norm Llama block: x + Wo·attn(RoPE(q), RoPE(k), v) then x + down(silu(gate)·up)."""
    B, S, _ = x.shape
    h = _rms(x, p["attn_norm.weight"], eps)
    qkv = h @ p["wqkv.weight"].t()
    q = qkv[..., : H * HD].view(B, S, H, HD)
    k = qkv[..., H * HD:(H + HK) * HD].view(B, S, HK, HD)
    v = qkv[..., (H + HK) * HD:].view(B, S, HK, HD)
    q, k = _rope(q, THETA), _rope(k, THETA)
    o = F.scaled_dot_product_attention(q.transpose(1, 2), k.transpose(1, 2), v.transpose(1, 2), is_causal=True,
                                       enable_gqa=True)
    x1 = x + o.transpose(1, 2).reshape(B, S, D) @ p["wo.weight"].t()
    h2 = _rms(x1, p["mlp_norm.weight"], eps)
    g, u = ops.split_gate_up(p["w_gate_up.weight"].t())  # columns of W^T are interleaved in blocks of 16
    return x1 + (F.silu(h2 @ g) * (h2 @ u)) @ p["w_down.weight"].t()


def test_llama_block_forward_backward_at_8b_shapes():
    from meshtrain_b200.models.llama import LlamaBlock

    B, S = 1, 4096
    torch.manual_seed(3)
    block = LlamaBlock(D, H, HK, FFN, rope_theta=THETA, init_std=0.02).cuda().to(torch.bfloat16)
    x = torch.randn(B, S, D, device="cuda").to(torch.bfloat16)
    dy = torch.randn(B, S, D, device="cuda").to(torch.bfloat16)

    saved: dict = {}
    y = block.fwd(x, saved)
    grads = {n: torch.zeros(p.shape, device="cuda", dtype=torch.float32) for n, p in block.named_parameters()}
    dx = block.bwd(dy, saved, grads)
    torch.cuda.synchronize()

    from torch.nn.attention import SDPBackend, sdpa_kernel

    with sdpa_kernel([SDPBackend.MATH]):
        params = {n: p.detach().float().requires_grad_(True) for n, p in block.named_parameters()}
        xf = x.float().requires_grad_(True)
        y_ref = _llama_block_fp32(xf, params, block.eps)
        y_ref.backward(dy.float())

    assert _rel_l2(y, y_ref) < 2e-2
    assert _rel_l2(dx, xf.grad) < 3e-2
    for name, g in grads.items():
        assert _rel_l2(g, params[name].grad) < 3e-2, name
