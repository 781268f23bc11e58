"""Llama-style decoder (RMSNorm, RoPE, grouped-query attention, SwiGLU, no biases).

The reference has no such model type (reference config.py:23 allows only
``mlp`` and ``tiny_transformer``); it is added here so the 8B-class configs
can run.  Layers: [Embedding (no positions)] + L x [LlamaBlock] + [LMHead
(RMSNorm, no bias)].

Kernel path per block: RMSNorm -> QKV GEMM -> RoPE(q, k) in place -> GQA flash
attention -> o-proj GEMM(+residual) -> RMSNorm -> gate/up GEMM with the SwiGLU
epilogue (raw gate/up kept for backward) -> down GEMM(+residual).
"""

from __future__ import annotations

import torch
from torch import nn
from torch.nn import functional as F

from meshtrain_b200 import ops
from meshtrain_b200.models.base import ModelSpec, PipelineLayer, arithmetic_tokens, uniform_tokens
from meshtrain_b200.models.gpt import Embedding, LMHead, RMSNormParam


class LlamaBlock(PipelineLayer):
    def __init__(self, d_model: int, n_heads: int, n_kv_heads: int, ffn_hidden: int, rope_theta: float = 500000.0,
                 init_std: float | None = 0.02, eps: float = 1e-5):
        super().__init__()
        if d_model % n_heads or n_heads % n_kv_heads:
            raise ValueError("d_model % n_heads and n_heads % n_kv_heads must be 0")
        if ffn_hidden % 16:
            raise ValueError("ffn_hidden must be a multiple of 16")
        self.n_heads, self.n_kv_heads = n_heads, n_kv_heads
        self.head_dim = d_model // n_heads
        self.ffn_hidden = ffn_hidden
        self.theta = rope_theta
        self.eps = eps
        qkv_out = (n_heads + 2 * n_kv_heads) * self.head_dim
        self.attn_norm = RMSNormParam(d_model, eps)
        self.wqkv = nn.Linear(d_model, qkv_out, bias=False)
        self.wo = nn.Linear(d_model, d_model, bias=False)
        self.mlp_norm = RMSNormParam(d_model, eps)
        # rows in blocks of 32 = [16 gate | 16 up] so the GEMM epilogue sees both
        self.w_gate_up = nn.Linear(d_model, 2 * ffn_hidden, bias=False)
        self.w_down = nn.Linear(ffn_hidden, d_model, bias=False)
        if init_std is not None:
            for lin in (self.wqkv, self.wo, self.w_gate_up, self.w_down):
                nn.init.normal_(lin.weight, 0.0, init_std)

    def _split(self, qkv, B, S):
        H, Hk, hd = self.n_heads, self.n_kv_heads, self.head_dim
        q = qkv[:, : H * hd].view(B, S, H, hd)
        k = qkv[:, H * hd:(H + Hk) * hd].view(B, S, Hk, hd)
        v = qkv[:, (H + Hk) * hd:].view(B, S, Hk, hd)
        return q, k, v

    # Two residual halves, each usable as a pipeline layer of its own (models/split.py).
    HALVES = (("attn_norm", "wqkv", "wo"), ("mlp_norm", "w_gate_up", "w_down"))

    def attn_fwd(self, x, saved):
        B, S, d = x.shape
        T = B * S
        x2 = x.reshape(T, d)
        y1, r1 = ops.rmsnorm(x2, self.attn_norm.weight, self.eps)
        qkv = ops.linear(y1, self.wqkv.weight)
        ops.rope_(qkv, S, self.n_heads + self.n_kv_heads, self.head_dim, self.theta)
        q, k, v = self._split(qkv, B, S)
        o, lse = ops.attention(q, k, v, causal=True)
        x1 = ops.linear(o.reshape(T, d), self.wo.weight, residual=x2)
        saved.update(shape=(B, S, d), x=x2, y1=y1, r1=r1, qkv=qkv, o=o, lse=lse)
        return x1.view(B, S, d)

    def mlp_fwd(self, x, saved):
        B, S, d = x.shape
        x1 = x.reshape(B * S, d)
        y2, r2 = ops.rmsnorm(x1, self.mlp_norm.weight, self.eps)
        act, raw = ops.swiglu_linear(y2, self.w_gate_up.weight)
        out = ops.linear(act, self.w_down.weight, residual=x1)
        saved.update(shape=(B, S, d), x1=x1, y2=y2, r2=r2, raw=raw, act=act)
        return out.view(B, S, d)

    def mlp_bwd(self, dy, saved, grads):
        B, S, d = saved["shape"]
        dy2 = dy.reshape(B * S, d)
        dact = ops.linear_dgrad(dy2, self.w_down.weight)
        ops.linear_wgrad_(dy2, saved["act"], grads["w_down.weight"])
        draw = ops.swiglu_bwd(dact, saved["raw"])
        del dact
        dln2 = ops.linear_dgrad(draw, self.w_gate_up.weight)
        ops.linear_wgrad_(draw, saved["y2"], grads["w_gate_up.weight"])
        del draw
        dx1 = ops.rmsnorm_bwd(dln2, saved["x1"], self.mlp_norm.weight, saved["r2"], dy2, grads["mlp_norm.weight"])
        return dx1.view(B, S, d)

    def attn_bwd(self, dy, saved, grads):
        B, S, d = saved["shape"]
        T = B * S
        H, Hk, hd = self.n_heads, self.n_kv_heads, self.head_dim
        dx1 = dy.reshape(T, d)
        do = ops.linear_dgrad(dx1, self.wo.weight)
        ops.linear_wgrad_(dx1, saved["o"].reshape(T, d), grads["wo.weight"])
        q, k, v = self._split(saved["qkv"], B, S)
        dqkv = torch.empty_like(saved["qkv"])
        ops.attention_bwd(do.view(B, S, H, hd), q, k, v, saved["o"], saved["lse"], causal=True,
                          out=self._split(dqkv, B, S))
        del do
        ops.rope_(dqkv, S, H + Hk, hd, self.theta, inverse=True)
        dln1 = ops.linear_dgrad(dqkv, self.wqkv.weight)
        ops.linear_wgrad_(dqkv, saved["y1"], grads["wqkv.weight"])
        dx = ops.rmsnorm_bwd(dln1, saved["x"], self.attn_norm.weight, saved["r1"], dx1, grads["attn_norm.weight"])
        return dx.view(B, S, d)

    def fwd(self, x, saved):
        return self.mlp_fwd(self.attn_fwd(x, saved), saved)

    def bwd(self, dy, saved, grads):
        return self.attn_bwd(self.mlp_bwd(dy, saved, grads), saved, grads)


class LlamaSpec(ModelSpec):
    name = "llama"
    required_ops = ("embedding", "linear", "rms_norm", "silu", "sdpa", "cross_entropy")

    def __init__(self, layers: int = 32, hidden_size: int = 4096, heads: int = 32, kv_heads: int = 8,
                 ffn_hidden: int = 14336, vocab_size: int = 128256, seq_len: int = 4096, rope_theta: float = 500000.0,
                 seed: int = 0, dtype: torch.dtype = torch.bfloat16, init_std: float | None = 0.02,
                 data: str = "uniform"):
        super().__init__(seed, dtype)
        self.n_blocks = layers
        self.d_model = hidden_size
        self.n_heads = heads
        self.n_kv_heads = kv_heads
        self.ffn_hidden = ffn_hidden
        self.vocab_size = vocab_size
        self.seq_len = seq_len
        self.rope_theta = rope_theta
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
            return Embedding(self.vocab_size, self.d_model, self.seq_len, self.init_std, learned_pos=False)
        if index == self.num_layers - 1:
            return LMHead(self.d_model, self.vocab_size, self.init_std, norm="rmsnorm", bias=False)
        return LlamaBlock(self.d_model, self.n_heads, self.n_kv_heads, self.ffn_hidden, self.rope_theta,
                          self.init_std)

    def loss_fn(self, output, target):
        return F.cross_entropy(output.reshape(-1, output.shape[-1]).float(), target.reshape(-1))

    def make_batch(self, step: int, batch_size: int):
        gen = uniform_tokens if self.data == "uniform" else arithmetic_tokens
        return gen(self.seed, step, batch_size, self.seq_len, self.vocab_size)

    def boundary_shape(self, microbatch_size: int):
        return (microbatch_size, self.seq_len, self.d_model)

    def flops_per_token(self) -> float:
        d, L, S, V = self.d_model, self.n_blocks, self.seq_len, self.vocab_size
        hd = d // self.n_heads
        qkv = d * (self.n_heads + 2 * self.n_kv_heads) * hd
        per_layer = 2 * (qkv + d * d + 3 * d * self.ffn_hidden)
        attn = 2 * S * d
        return 3.0 * (L * (per_layer + attn) + 2 * d * V)
