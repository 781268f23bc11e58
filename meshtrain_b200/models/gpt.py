"""Decoder-only GPT (pre-LayerNorm, GELU, learned positions, biases) as a layer list.

Layers: [Embedding] + L x [Block] + [LMHead]; the same structure and parameter
names as the reference's tiny Transformer (reference
models/tiny_transformer.py:19-102), so configs written for it (type
``tiny_transformer``) build this model.

Per block, forward on the kernel path is 6 launches + attention:
    LN1 -> QKV GEMM(+bias) -> flash attention -> proj GEMM(+bias+residual)
    -> LN2 -> fc1 GEMM(+bias, GELU, keeps pre-activation) -> fc2 GEMM(+bias+residual)
and backward fuses GELU' into the fc2 dgrad epilogue, the residual gradient
into the LayerNorm backward, and accumulates every weight gradient in fp32 in
the wgrad GEMM epilogue.
"""

from __future__ import annotations

import torch
from torch import nn
from torch.nn import functional as F

from meshtrain_b200 import ops
from meshtrain_b200.models.base import ModelSpec, PipelineLayer, arithmetic_tokens, uniform_tokens


def _init_linear(lin: nn.Linear, std: float | None) -> None:
    if std is not None:
        nn.init.normal_(lin.weight, 0.0, std)
        if lin.bias is not None:
            nn.init.zeros_(lin.bias)


class Embedding(PipelineLayer):
    takes_integer_input = True

    def __init__(self, vocab_size: int, d_model: int, max_seq_len: int, init_std: float | None = None,
                 learned_pos: bool = True):
        super().__init__()
        self.tok = nn.Embedding(vocab_size, d_model)
        self.pos = nn.Embedding(max_seq_len, d_model) if learned_pos else None
        self.seq_len = max_seq_len
        if init_std is not None:
            nn.init.normal_(self.tok.weight, 0.0, init_std)
            if self.pos is not None:
                nn.init.normal_(self.pos.weight, 0.0, init_std)

    def fwd(self, tokens, saved):
        B, S = tokens.shape
        out = ops.embedding(tokens, self.tok.weight, None if self.pos is None else self.pos.weight, S)
        saved["ids"] = tokens
        return out.view(B, S, -1)

    def bwd(self, dy, saved, grads):
        ids = saved["ids"]
        S = ids.shape[1]
        ops.embedding_bwd_(ids, dy, grads["tok.weight"], grads.get("pos.weight"), S)
        return None

    def forward(self, tokens):  # autograd path
        if ops.backend() == "torch" or not tokens.is_cuda:
            positions = torch.arange(tokens.shape[1], device=tokens.device)
            out = self.tok(tokens)
            return out + self.pos(positions)[None] if self.pos is not None else out
        return super().forward(tokens)


class Block(PipelineLayer):
    def __init__(self, d_model: int, n_heads: int, mlp_ratio: int = 4, init_std: float | None = None,
                 n_layers_for_scaling: int | None = None, eps: float = 1e-5):
        super().__init__()
        if d_model % n_heads:
            raise ValueError("d_model must be divisible by n_heads")
        self.n_heads = n_heads
        self.eps = eps
        self.ln1 = nn.LayerNorm(d_model, eps=eps)
        self.qkv = nn.Linear(d_model, 3 * d_model)
        self.proj = nn.Linear(d_model, d_model)
        self.ln2 = nn.LayerNorm(d_model, eps=eps)
        self.fc1 = nn.Linear(d_model, mlp_ratio * d_model)
        self.fc2 = nn.Linear(mlp_ratio * d_model, d_model)
        for lin in (self.qkv, self.proj, self.fc1, self.fc2):
            _init_linear(lin, init_std)

    # The block is two residual halves; each half is also usable as a pipeline
    # layer of its own (models/split.py), so a stage boundary may fall between them.
    HALVES = (("ln1", "qkv", "proj"), ("ln2", "fc1", "fc2"))

    def attn_fwd(self, x, saved):
        B, S, d = x.shape
        H = self.n_heads
        hd = d // H
        x2 = x.reshape(B * S, d)
        y1, m1, r1 = ops.layernorm(x2, self.ln1.weight, self.ln1.bias, self.eps)
        qkv = ops.linear(y1, self.qkv.weight, self.qkv.bias)
        q = qkv[:, :d].view(B, S, H, hd)
        k = qkv[:, d:2 * d].view(B, S, H, hd)
        v = qkv[:, 2 * d:].view(B, S, H, hd)
        o, lse = ops.attention(q, k, v, causal=True)
        x1 = ops.linear(o.reshape(B * S, d), self.proj.weight, self.proj.bias, residual=x2)
        saved.update(shape=(B, S, d), x=x2, y1=y1, m1=m1, r1=r1, qkv=qkv, o=o, lse=lse)
        return x1.view(B, S, d)

    def mlp_fwd(self, x, saved):
        B, S, d = x.shape
        x1 = x.reshape(B * S, d)
        y2, m2, r2 = ops.layernorm(x1, self.ln2.weight, self.ln2.bias, self.eps)
        g, h = ops.linear(y2, self.fc1.weight, self.fc1.bias, gelu=True)
        out = ops.linear(g, self.fc2.weight, self.fc2.bias, residual=x1)
        saved.update(shape=(B, S, d), x1=x1, y2=y2, m2=m2, r2=r2, h=h, g=g)
        return out.view(B, S, d)

    def mlp_bwd(self, dy, saved, grads):
        B, S, d = saved["shape"]
        dy2 = dy.reshape(B * S, d)
        dh = ops.linear_dgrad(dy2, self.fc2.weight, gelu_pre=saved["h"])
        ops.linear_wgrad_(dy2, saved["g"], grads["fc2.weight"], grads["fc2.bias"])
        dln2 = ops.linear_dgrad(dh, self.fc1.weight)
        ops.linear_wgrad_(dh, saved["y2"], grads["fc1.weight"], grads["fc1.bias"])
        del dh
        dx1 = ops.layernorm_bwd(dln2, saved["x1"], self.ln2.weight, saved["m2"], saved["r2"], dy2,
                                grads["ln2.weight"], grads["ln2.bias"])
        return dx1.view(B, S, d)

    def attn_bwd(self, dy, saved, grads):
        B, S, d = saved["shape"]
        H = self.n_heads
        hd = d // H
        T = B * S
        dx1 = dy.reshape(T, d)
        do = ops.linear_dgrad(dx1, self.proj.weight)
        ops.linear_wgrad_(dx1, saved["o"].reshape(T, d), grads["proj.weight"], grads["proj.bias"])
        qkv = saved["qkv"]
        q = qkv[:, :d].view(B, S, H, hd)
        k = qkv[:, d:2 * d].view(B, S, H, hd)
        v = qkv[:, 2 * d:].view(B, S, H, hd)
        dqkv = torch.empty_like(qkv)
        ops.attention_bwd(do.view(B, S, H, hd), q, k, v, saved["o"], saved["lse"], causal=True,
                          out=(dqkv[:, :d].view(B, S, H, hd), dqkv[:, d:2 * d].view(B, S, H, hd),
                               dqkv[:, 2 * d:].view(B, S, H, hd)))
        del do
        dln1 = ops.linear_dgrad(dqkv, self.qkv.weight)
        ops.linear_wgrad_(dqkv, saved["y1"], grads["qkv.weight"], grads["qkv.bias"])
        dx = ops.layernorm_bwd(dln1, saved["x"], self.ln1.weight, saved["m1"], saved["r1"], dx1,
                               grads["ln1.weight"], grads["ln1.bias"])
        return dx.view(B, S, d)

    def fwd(self, x, saved):
        return self.mlp_fwd(self.attn_fwd(x, saved), saved)

    def bwd(self, dy, saved, grads):
        return self.attn_bwd(self.mlp_bwd(dy, saved, grads), saved, grads)

    # autograd / CPU path of each half (the reference's module arithmetic)
    def attn_torch(self, x):
        b, t, d = x.shape
        q, k, v = self.qkv(self.ln1(x)).split(d, dim=-1)
        q, k, v = (z.view(b, t, self.n_heads, d // self.n_heads).transpose(1, 2) for z in (q, k, v))
        a = F.scaled_dot_product_attention(q, k, v, is_causal=True)
        return x + self.proj(a.transpose(1, 2).reshape(b, t, d))

    def mlp_torch(self, x):
        return x + self.fc2(F.gelu(self.fc1(self.ln2(x))))

    def forward(self, x):  # autograd path
        if ops.backend() == "torch" or not x.is_cuda:
            return self.mlp_torch(self.attn_torch(x))
        return super().forward(x)


class LMHead(PipelineLayer):
    """Final LayerNorm + vocabulary projection.

    ``fwd`` returns logits (autograd / reference path).  The engine instead
    calls ``fwd_loss``: token-chunked logits GEMM -> in-place softmax-CE
    forward+backward -> dgrad/wgrad GEMMs, so full logits are never stored.
    """

    def __init__(self, d_model: int, vocab_size: int, init_std: float | None = None, eps: float = 1e-5,
                 norm: str = "layernorm", bias: bool = True):
        super().__init__()
        self.norm_kind = norm
        self.ln = nn.LayerNorm(d_model, eps=eps) if norm == "layernorm" else RMSNormParam(d_model, eps)
        self.out = nn.Linear(d_model, vocab_size, bias=bias)
        self.vocab = vocab_size
        self.eps = eps
        _init_linear(self.out, init_std)

    def _norm(self, x2):
        if self.norm_kind == "layernorm":
            return ops.layernorm(x2, self.ln.weight, self.ln.bias, self.eps)
        y, r = ops.rmsnorm(x2, self.ln.weight, self.eps)
        return y, None, r

    def _norm_bwd(self, dy, x2, m, r, grads):
        if self.norm_kind == "layernorm":
            return ops.layernorm_bwd(dy, x2, self.ln.weight, m, r, None, grads["ln.weight"], grads["ln.bias"])
        return ops.rmsnorm_bwd(dy, x2, self.ln.weight, r, None, grads["ln.weight"])

    def fwd(self, x, saved):
        B, S, d = x.shape
        x2 = x.reshape(B * S, d)
        y, m, r = self._norm(x2)
        logits = ops.linear(y, self.out.weight, self.out.bias)
        saved.update(shape=(B, S, d), x=x2, y=y, m=m, r=r)
        return logits.view(B, S, -1)

    def bwd(self, dy, saved, grads):
        B, S, d = saved["shape"]
        T = B * S
        dl = dy.reshape(T, -1)
        dyn = ops.linear_dgrad(dl, self.out.weight)
        ops.linear_wgrad_(dl, saved["y"], grads["out.weight"], grads.get("out.bias"))
        return self._norm_bwd(dyn, saved["x"], saved["m"], saved["r"], grads).view(B, S, d)

    def fwd_loss(self, x, targets, saved, grads, loss_sum: torch.Tensor, grad_scale: float,
                 chunk_tokens: int | None = None) -> None:
        """Loss forward + full backward of this layer for one microbatch.

        ``loss_sum += mean CE`` (fp32 device scalar); parameter gradients are
        accumulated with the mean-CE gradient times ``grad_scale``; the input
        gradient is kept in ``saved["dx"]`` for ``bwd_from_loss``.
        """
        B, S, d = x.shape
        T = B * S
        V = self.vocab
        x2 = x.reshape(T, d)
        tg = targets.reshape(T)
        y, m, r = self._norm(x2)
        vpad = (V + 7) // 8 * 8
        if chunk_tokens is None:
            chunk_tokens = max(128, min(T, (1 << 30) // (vpad * 2)))
        dy = torch.empty_like(x2)
        logits = torch.empty(min(chunk_tokens, T), vpad, device=x.device, dtype=x.dtype)
        for c0 in range(0, T, chunk_tokens):
            c1 = min(T, c0 + chunk_tokens)
            lg = logits[: c1 - c0]
            yc = y[c0:c1]
            if ops._custom(yc, self.out.weight):
                ops.extension().gemm(yc, False, self.out.weight, False, lg, ops.EPI_BF16, self.out.bias, None, None, 0.0)
            else:
                lg[:, :V] = ops.linear(yc, self.out.weight, self.out.bias)
            ops.cross_entropy_chunk_(lg, V, tg[c0:c1], loss_sum, 1.0 / T, grad_scale / T)
            dl = lg[:, :V]
            ops.linear_dgrad(dl, self.out.weight, out=dy[c0:c1])  # straight into this chunk's rows
            ops.linear_wgrad_(dl, yc, grads["out.weight"], grads.get("out.bias"))
        saved["dx"] = self._norm_bwd(dy, x2, m, r, grads).view(B, S, d)

    def forward(self, x):  # autograd path
        if ops.backend() == "torch" or not x.is_cuda:
            return self.out(self.ln(x))
        return super().forward(x)


class RMSNormParam(nn.Module):
    """Parameter container for RMSNorm (``weight`` only)."""

    def __init__(self, d: int, eps: float = 1e-5):
        super().__init__()
        self.weight = nn.Parameter(torch.ones(d))
        self.eps = eps

    def forward(self, x):
        xf = x.float()
        return (xf * torch.rsqrt(xf.pow(2).mean(-1, keepdim=True) + self.eps) * self.weight.float()).to(x.dtype)


class GPTSpec(ModelSpec):
    """GPT / reference ``tiny_transformer`` model family."""

    name = "gpt"
    required_ops = ("embedding", "linear", "layer_norm", "gelu", "sdpa", "cross_entropy")

    def __init__(self, layers: int = 6, hidden_size: int = 256, heads: int = 4, vocab_size: int = 256,
                 seq_len: int = 64, seed: int = 0, dtype: torch.dtype = torch.float32, mlp_ratio: int = 4,
                 init_std: float | None = None, data: str = "arithmetic"):
        super().__init__(seed, dtype)
        self.n_blocks = layers
        self.d_model = hidden_size
        self.n_heads = heads
        self.vocab_size = vocab_size
        self.seq_len = seq_len
        self.mlp_ratio = mlp_ratio
        self.init_std = init_std
        self.data = data

    @property
    def num_layers(self) -> int:
        return self.n_blocks + 2

    def layer_name(self, index: int) -> str:
        if index == 0:
            return "embedding"
        if index == self.num_layers - 1:
            return "lm_head"
        return f"block{index - 1}"

    def _make_layer(self, index: int) -> nn.Module:
        if index == 0:
            return Embedding(self.vocab_size, self.d_model, self.seq_len, self.init_std)
        if index == self.num_layers - 1:
            return LMHead(self.d_model, self.vocab_size, self.init_std)
        return Block(self.d_model, self.n_heads, self.mlp_ratio, self.init_std)

    def loss_fn(self, output, target):
        return F.cross_entropy(output.reshape(-1, output.shape[-1]).float(), target.reshape(-1))

    def make_batch(self, step: int, batch_size: int):
        gen = uniform_tokens if self.data == "uniform" else arithmetic_tokens
        return gen(self.seed, step, batch_size, self.seq_len, self.vocab_size)

    def boundary_shape(self, microbatch_size: int):
        return (microbatch_size, self.seq_len, self.d_model)

    def flops_per_token(self) -> float:
        d, L, S, V = self.d_model, self.n_blocks, self.seq_len, self.vocab_size
        per_layer = 2 * (3 * d * d + d * d + 2 * self.mlp_ratio * d * d)  # forward GEMMs
        attn = 2 * S * d  # causal QK^T + PV, forward, averaged over positions
        fwd = L * (per_layer + attn) + 2 * d * V
        return 3.0 * fwd


__all__ = ["GPTSpec", "Embedding", "Block", "LMHead", "RMSNormParam"]
