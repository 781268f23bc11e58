"""tcgen05 flash attention (forward + backward) against the fp32 PyTorch reference."""

import math

import pytest
import torch

from meshtrain_b200 import ops
from meshtrain_b200.ops import attention_impl

pytestmark = pytest.mark.gpu


def _close(out, ref, tol):
    out, ref = out.float(), ref.float()
    scale = ref.abs().max().item() + 1e-6
    err = (out - ref).abs().max().item()
    assert err <= tol * scale, f"max abs err {err:.3e} vs scale {scale:.3e}"


@pytest.fixture(autouse=True)
def _status():
    torch.manual_seed(0)
    ops.set_backend("custom")
    yield
    torch.cuda.synchronize()
    assert ops.read_status(torch.cuda.current_device()) == 0


CASES = [
    # B, S, Hq, Hk, hd
    (1, 128, 1, 1, 64),
    (2, 256, 4, 4, 64),
    (1, 384, 2, 2, 128),
    (2, 200, 4, 2, 64),     # S not a multiple of the tile
    (1, 512, 8, 2, 128),    # GQA 4:1
    (1, 1024, 4, 4, 64),
    (2, 200, 4, 2, 128),    # head dim 128, S not a multiple of either tile height
    (1, 1000, 8, 2, 128),   # head dim 128, GQA 4:1, eight partial 64-query tiles past the diagonal
]


@pytest.mark.parametrize("B,S,Hq,Hk,hd", CASES)
def test_attention_forward(B, S, Hq, Hk, hd):
    dev = "cuda"
    qkv = torch.randn(B, S, (Hq + 2 * Hk) * hd, device=dev).to(torch.bfloat16)
    q = qkv[..., : Hq * hd].view(B, S, Hq, hd)
    k = qkv[..., Hq * hd:(Hq + Hk) * hd].view(B, S, Hk, hd)
    v = qkv[..., (Hq + Hk) * hd:].view(B, S, Hk, hd)
    o, lse = ops.attention(q, k, v, causal=True)
    o_ref, lse_ref = attention_impl._reference_fwd(q, k, v, True, 1.0 / math.sqrt(hd))
    _close(o, o_ref, 2e-2)
    _close(lse, lse_ref, 1e-3)


@pytest.mark.parametrize("B,S,Hq,Hk,hd", CASES)
def test_attention_backward(B, S, Hq, Hk, hd):
    dev = "cuda"
    q = torch.randn(B, S, Hq, hd, device=dev).to(torch.bfloat16)
    k = torch.randn(B, S, Hk, hd, device=dev).to(torch.bfloat16)
    v = torch.randn(B, S, Hk, hd, device=dev).to(torch.bfloat16)
    do = torch.randn(B, S, Hq, hd, device=dev).to(torch.bfloat16)
    scale = 1.0 / math.sqrt(hd)
    o_ref, lse_ref = attention_impl._reference_fwd(q, k, v, True, scale)
    o, lse = ops.attention(q, k, v, causal=True)
    dq, dk, dv = ops.attention_bwd(do, q, k, v, o, lse, causal=True)
    rq, rk, rv = attention_impl._reference_bwd(do, q, k, v, o_ref, lse_ref, True, scale)
    _close(dv, rv, 3e-2)
    _close(dk, rk, 3e-2)
    _close(dq, rq, 3e-2)


def test_attention_packed_outputs():
    B, S, H, hd = 2, 256, 4, 64
    qkv = torch.randn(B * S, 3 * H * hd, device="cuda").to(torch.bfloat16)
    views = lambda t: tuple(t[:, i * H * hd:(i + 1) * H * hd].view(B, S, H, hd) for i in range(3))  # noqa: E731
    q, k, v = views(qkv)
    o, lse = ops.attention(q, k, v)
    do = torch.randn_like(o)
    dqkv = torch.empty_like(qkv)
    ops.attention_bwd(do, q, k, v, o, lse, out=views(dqkv))
    dq, dk, dv = ops.attention_bwd(do, q, k, v, o, lse)
    for a, b in zip(views(dqkv), (dq, dk, dv)):
        torch.testing.assert_close(a.float(), b.float(), rtol=1e-2, atol=1e-2)


@pytest.mark.parametrize("hd", [64, 128])
def test_attention_backward_not_causal(hd):
    dev = "cuda"
    B, S, Hq, Hk = 2, 320, 4, 2
    q = torch.randn(B, S, Hq, hd, device=dev).to(torch.bfloat16)
    k = torch.randn(B, S, Hk, hd, device=dev).to(torch.bfloat16)
    v = torch.randn(B, S, Hk, hd, device=dev).to(torch.bfloat16)
    do = torch.randn(B, S, Hq, hd, device=dev).to(torch.bfloat16)
    scale = 1.0 / math.sqrt(hd)
    o_ref, lse_ref = attention_impl._reference_fwd(q, k, v, False, scale)
    o, lse = ops.attention(q, k, v, causal=False)
    _close(o, o_ref, 2e-2)
    dq, dk, dv = ops.attention_bwd(do, q, k, v, o, lse, causal=False)
    rq, rk, rv = attention_impl._reference_bwd(do, q, k, v, o_ref, lse_ref, False, scale)
    _close(dv, rv, 3e-2)
    _close(dk, rk, 3e-2)
    _close(dq, rq, 3e-2)
