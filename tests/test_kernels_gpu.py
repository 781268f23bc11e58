"""Numerics of the hand-written sm_100a kernels against fp32 PyTorch references.

Every test runs the kernel through ``meshtrain_b200.ops`` (backend "custom")
and compares with the same math in fp32 PyTorch on the same bf16 inputs.
"""

import math

import pytest
import torch

from meshtrain_b200 import ops

pytestmark = pytest.mark.gpu

DEV = "cuda"


def _close(out, ref, tol=2e-2):
    out = out.float()
    ref = ref.float()
    scale = ref.abs().max().item() + 1e-6
    err = (out - ref).abs().max().item()
    assert err <= tol * scale, f"max abs err {err:.3e} vs scale {scale:.3e}"


def _bf(*shape, scale=1.0):
    return (torch.randn(*shape, device=DEV) * scale).to(torch.bfloat16)


@pytest.fixture(autouse=True)
def _seed_and_status():
    torch.manual_seed(0)
    ops.set_backend("custom")
    yield
    torch.cuda.synchronize()
    assert ops.read_status(torch.cuda.current_device()) == 0, "a kernel reported a wait timeout"


GEMM_SHAPES = [(128, 128, 64), (256, 512, 128), (1000, 1000, 200), (130, 257, 72), (4096, 3840, 1280),
               (2048, 1280, 5120), (8, 24, 16), (384, 2304, 768)]


@pytest.mark.parametrize("M,N,K", GEMM_SHAPES)
def test_gemm_forward(M, N, K):
    x, w, b = _bf(M, K), _bf(N, K, scale=0.05), _bf(N)
    y = ops.linear(x, w, b)
    _close(y, x.float() @ w.float().t() + b.float())


@pytest.mark.parametrize("M,N,K", GEMM_SHAPES)
def test_gemm_dgrad(M, N, K):
    # dx[M,K] = dy[M,N] @ W[N,K]  (B operand MN-major)
    dy, w = _bf(M, N), _bf(N, K, scale=0.05)
    _close(ops.linear_dgrad(dy, w), dy.float() @ w.float())


@pytest.mark.parametrize("M,N,K", GEMM_SHAPES)
def test_gemm_wgrad_accumulates(M, N, K):
    # dW[N,K] += dy^T[N,M] @ x[M,K]  (both operands MN-major), fp32 accumulate
    dy, x = _bf(M, N), _bf(M, K)
    acc = torch.randn(N, K, device=DEV)
    acc0 = acc.clone()
    bg = torch.zeros(N, device=DEV)
    ops.linear_wgrad_(dy, x, acc, bg)
    ref = acc0 + dy.float().t() @ x.float()
    _close(acc, ref, tol=1e-2)
    _close(bg, dy.float().sum(0), tol=1e-2)


@pytest.mark.parametrize("M,N,K", [(512, 2048, 256), (1000, 4096, 1280), (77, 512, 64)])
def test_gemm_gelu_epilogue(M, N, K):
    x, w, b = _bf(M, K), _bf(N, K, scale=0.05), _bf(N)
    g, h = ops.linear(x, w, b, gelu=True)
    href = x.float() @ w.float().t() + b.float()
    _close(h, href)
    _close(g, torch.nn.functional.gelu(h.float()))


@pytest.mark.parametrize("M,N,K", [(512, 1280, 5120), (333, 256, 128)])
def test_gemm_residual_epilogue(M, N, K):
    x, w, b, r = _bf(M, K), _bf(N, K, scale=0.02), _bf(N), _bf(M, N)
    y = ops.linear(x, w, b, residual=r)
    _close(y, x.float() @ w.float().t() + b.float() + r.float())


@pytest.mark.parametrize("M,N,K", [(512, 1280, 5120), (200, 320, 640)])
def test_gemm_dgelu_epilogue(M, N, K):
    # dh[M,K] = (dy[M,N] @ W2[N,K]) * gelu'(h[M,K])
    dy, w, h = _bf(M, N), _bf(N, K, scale=0.05), _bf(M, K)
    out = ops.linear_dgrad(dy, w, gelu_pre=h)
    _close(out, (dy.float() @ w.float()) * ops.gelu_grad(h.float()))


@pytest.mark.parametrize("M,F,K", [(512, 1024, 256), (300, 512, 128)])
def test_gemm_swiglu_epilogue(M, F, K):
    x = _bf(M, K)
    wg, wu = _bf(F, K, scale=0.05), _bf(F, K, scale=0.05)
    wgu = ops.interleave_gate_up(wg, wu)
    act, raw = ops.swiglu_linear(x, wgu)
    g = x.float() @ wg.float().t()
    u = x.float() @ wu.float().t()
    rg, ru = ops.split_gate_up(raw)
    _close(rg, g)
    _close(ru, u)
    _close(act, torch.nn.functional.silu(rg.float()) * ru.float())
    dout = _bf(M, F)
    draw = ops.swiglu_bwd(dout, raw)
    with ops.use_backend("torch"):
        ref = ops.swiglu_bwd(dout.cpu(), raw.cpu())
    _close(draw, ref.to(DEV))


@pytest.mark.parametrize("T,d", [(4096, 1280), (100, 1024), (37, 4096), (513, 256), (8, 64), (301, 1536),
                                 (250, 2048), (99, 3072), (5, 2560)])
def test_layernorm_fwd_bwd(T, d):
    x, g, b = _bf(T, d), _bf(d), _bf(d)
    y, m, r = ops.layernorm(x, g, b)
    yref = torch.nn.functional.layer_norm(x.float(), (d,), g.float(), b.float(), 1e-5)
    _close(y, yref)
    dy, dres = _bf(T, d), _bf(T, d)
    dg, db = torch.zeros(d, device=DEV), torch.zeros(d, device=DEV)
    dx = ops.layernorm_bwd(dy, x, g, m, r, dres, dg, db)
    xr = x.float().requires_grad_()
    gr = g.float().requires_grad_()
    br = b.float().requires_grad_()
    out = torch.nn.functional.layer_norm(xr, (d,), gr, br, 1e-5)
    out.backward(dy.float())
    _close(dx, xr.grad + dres.float())
    _close(dg, gr.grad, tol=1e-2)
    _close(db, br.grad, tol=1e-2)


@pytest.mark.parametrize("T,d", [(4096, 4096), (77, 1280), (16, 64), (129, 2048), (33, 3584)])
def test_rmsnorm_fwd_bwd(T, d):
    x, g = _bf(T, d), _bf(d)
    y, r = ops.rmsnorm(x, g)
    xf = x.float()
    yref = xf * torch.rsqrt(xf.pow(2).mean(-1, keepdim=True) + 1e-5) * g.float()
    _close(y, yref)
    dy = _bf(T, d)
    dg = torch.zeros(d, device=DEV)
    dx = ops.rmsnorm_bwd(dy, x, g, r, None, dg)
    xr = x.float().requires_grad_()
    gr = g.float().requires_grad_()
    out = xr * torch.rsqrt(xr.pow(2).mean(-1, keepdim=True) + 1e-5) * gr
    out.backward(dy.float())
    _close(dx, xr.grad)
    _close(dg, gr.grad, tol=1e-2)


@pytest.mark.parametrize("V,d,S,B", [(1000, 256, 64, 4), (50257, 1280, 2048, 4), (128256, 512, 4096, 1)])
def test_embedding_fwd_bwd(V, d, S, B):
    ids = torch.randint(0, V, (B, S), device=DEV)
    ids[0, :17] = 7  # a long run of one token id
    tok, pos = _bf(V, d), _bf(S, d)
    out = ops.embedding(ids, tok, pos, S)
    ref = tok.float()[ids.reshape(-1)] + pos.float()[torch.arange(B * S, device=DEV) % S]
    _close(out, ref)
    dy = _bf(B * S, d)
    tref = torch.zeros(V, d, device=DEV).index_add_(0, ids.reshape(-1), dy.float())
    pref = dy.float().reshape(B, S, d).sum(0)
    runs = []
    for _ in range(2):  # each row is summed in a fixed order: identical bits on every run
        tg, pg = torch.full((V, d), 0.5, device=DEV), torch.full((S, d), 0.25, device=DEV)
        ops.embedding_bwd_(ids, dy, tg, pg, S)
        _close(tg - 0.5, tref, tol=1e-3)
        _close(pg - 0.25, pref, tol=1e-3)
        runs.append((tg, pg))
    assert torch.equal(runs[0][0], runs[1][0]) and torch.equal(runs[0][1], runs[1][1])


@pytest.mark.parametrize("T,V", [(256, 50257), (64, 1024), (33, 128256), (7, 100)])
def test_cross_entropy_chunk(T, V):
    vpad = (V + 7) // 8 * 8
    logits = torch.zeros(T, vpad, device=DEV, dtype=torch.bfloat16)
    logits[:, :V] = _bf(T, V, scale=3.0)
    tg = torch.randint(0, V, (T,), device=DEV)
    lf = logits[:, :V].float().clone().requires_grad_()
    loss_ref = torch.nn.functional.cross_entropy(lf, tg)
    loss_ref.backward()
    loss = torch.zeros((), device=DEV)
    ops.cross_entropy_chunk_(logits, V, tg, loss, 1.0 / T, 1.0 / T)
    assert abs(loss.item() - loss_ref.item()) < 1e-3 * max(1.0, abs(loss_ref.item()))
    _close(logits[:, :V], lf.grad, tol=2e-2)


def test_adam_matches_torch():
    n = 100_003
    p = torch.randn(n, device=DEV)
    g = torch.randn(n, device=DEV)
    m, v = torch.zeros(n, device=DEV), torch.zeros(n, device=DEV)
    pb = torch.empty(n, device=DEV, dtype=torch.bfloat16)
    pr = p.clone().requires_grad_()
    opt = torch.optim.Adam([pr], lr=1e-2, weight_decay=0.0)
    for step in range(1, 4):
        pr.grad = g.clone()
        opt.step()
        ops.adam_(p, g, m, v, pb, lr=1e-2, beta1=0.9, beta2=0.999, eps=1e-8, weight_decay=0.0, decoupled=False,
                  step=step)
    assert (p - pr.detach()).abs().max().item() < 1e-5
    assert ((pb.float() - p).abs() <= p.abs() * 2.0 ** -8 + 1e-6).all()  # bf16 copy-out is a rounding of p


def test_rope_roundtrip_and_reference():
    T, H, hd, S = 128, 6, 128, 64
    qk = _bf(T, H * hd + 64)
    ref = qk.clone().cpu()
    with ops.use_backend("torch"):
        ops.rope_(ref, S, H, hd, 500000.0)
    out = qk.clone()
    ops.rope_(out, S, H, hd, 500000.0)
    _close(out.cpu(), ref)
    ops.rope_(out, S, H, hd, 500000.0, inverse=True)
    _close(out, qk, tol=3e-2)


def test_gemm_launch_counter_counts():
    x, w = _bf(64, 64), _bf(64, 64)
    before = ops.launches()
    ops.linear(x, w)
    assert ops.launches() == before + 1


@pytest.mark.parametrize("T,N", [(8192, 1280), (1000, 3840), (77, 100), (3, 5120), (4099, 264)])
def test_colsum_accumulates(T, N):
    dy = _bf(T, N)
    out = torch.randn(N, device=DEV)
    ref = out + dy.float().sum(0)
    ops.extension().colsum_(ops._mat(dy), out)
    _close(out, ref, tol=1e-2)
