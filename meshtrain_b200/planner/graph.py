"""Per-layer profiles used by the planner.

``profile_model`` pushes one microbatch through each layer on the ``meta``
device and records parameters, input/output bytes, autograd-saved bytes and
forward FLOPs (reference planner/graph.py:25-82).  ``analytic_profile`` gives
the same fields in closed form for the GPT / Llama layers as the GPU engine
runs them (flash attention saves O and the logsumexp, never the T x T scores;
the fused LM head keeps one logits chunk).
"""

from __future__ import annotations

from dataclasses import asdict, dataclass

import torch
from torch.utils.flop_counter import FlopCounterMode


@dataclass
class LayerProfile:
    index: int
    name: str
    params: int
    param_bytes: int
    input_bytes: int
    activation_bytes: int  # output bytes of the layer (one microbatch)
    saved_bytes: int       # activations kept for backward (one microbatch)
    flops: float           # forward FLOPs (one microbatch)
    recompute_bytes: int = 0  # activations re-materialised during the layer's backward (recompute)

    @property
    def output_bytes(self) -> int:
        return self.activation_bytes

    def to_dict(self) -> dict:
        return asdict(self)


# Flash attention runs at about a third of the GEMMs' FLOP rate on B200 (measured at the
# 0.48B GPT shapes: ~390 TFLOP/s forward/backward against ~1200 for the linear layers), so
# its FLOPs count three times toward a layer's cost.
ATTENTION_COST_WEIGHT = 3.0


def _half_flops(spec) -> tuple[float, float]:
    """Effective forward FLOPs per token of a block's attention and MLP halves."""
    d, S = spec.d_model, spec.seq_len
    attn = ATTENTION_COST_WEIGHT * 2 * S * d  # causal QK^T and PV, averaged over positions
    if spec.name == "gpt":
        return 2 * 4 * d * d + attn, 2 * 2 * spec.mlp_ratio * d * d
    hd = d // spec.n_heads
    return 2 * (d * (spec.n_heads + 2 * spec.n_kv_heads) * hd + d * d) + attn, 2 * 3 * d * spec.ffn_hidden


def analytic_layer_flops(spec) -> list[float]:
    """Effective forward FLOPs per token of each layer (transformer families), else parameter counts."""
    kind = getattr(spec, "name", "")
    if kind in ("gpt", "llama"):
        d, V = spec.d_model, spec.vocab_size
        a, m = _half_flops(spec)
        mid = [float(a), float(m)] if getattr(spec, "split_blocks", False) else [float(a + m)]
        return [float(4 * d)] + mid * spec.n_blocks + [float(2 * d * V + 6 * V)]
    return [float(max(c, 1)) for c in spec.layer_parameter_counts()]


def analytic_profile(spec, microbatch_size: int) -> list[LayerProfile]:
    """Closed-form profiles of GPT / Llama layers under the GPU engine (bf16 activations)."""
    kind = spec.name
    if kind not in ("gpt", "llama"):
        raise ValueError("analytic profiles cover the gpt and llama families")
    T = microbatch_size * spec.seq_len
    d, V = spec.d_model, spec.vocab_size
    eb = torch.empty((), dtype=spec.dtype).element_size()
    counts = spec.layer_parameter_counts()
    fl = analytic_layer_flops(spec)
    act = T * d * eb
    out = []
    for i in range(spec.num_layers):
        if i == 0:
            saved, inp = T * 8, T * 8  # token ids
        elif i == spec.num_layers - 1:
            vpad = (V + 7) // 8 * 8
            chunk = min(T, max(128, (1 << 30) // (vpad * 2)))
            saved, inp = 3 * act + chunk * vpad * eb, act
        else:
            # attention half: x, normed x, qkv, o (+ fp32 row stats, lse); MLP half: x1, normed x1,
            # pre-activation and activation (+ fp32 row stats)
            if kind == "gpt":
                f = spec.mlp_ratio * d
                attn = T * eb * (d + d + 3 * d + d) + T * 4 * (2 + spec.n_heads)
                mlp = T * eb * (d + d + 2 * f) + T * 4 * 2
            else:
                hd = d // spec.n_heads
                qkv = (spec.n_heads + 2 * spec.n_kv_heads) * hd
                attn = T * eb * (d + d + qkv + d) + T * 4 * (1 + spec.n_heads)
                mlp = T * eb * (d + d + 3 * spec.ffn_hidden) + T * 4
            if getattr(spec, "split_blocks", False):
                saved = attn if (i - 1) % 2 == 0 else mlp
            else:
                saved = attn + mlp
            inp = act
        out.append(LayerProfile(i, spec.layer_name(i), counts[i], counts[i] * eb, inp, act if i < spec.num_layers - 1
                                else 4, saved, fl[i] * T))
    return out


def _saved_bytes_of(module, x):
    params = {id(p) for p in module.parameters()}
    saved = 0

    def pack(t):
        nonlocal saved
        base = t._base if t._base is not None else t
        if id(t) not in params and id(base) not in params:
            saved += t.numel() * t.element_size()
        return t

    with torch.autograd.graph.saved_tensors_hooks(pack, lambda t: t):
        y = module(x)
    return saved, y


def profile_model(spec, microbatch_size: int) -> list[LayerProfile]:
    """Profile every layer on the meta device with one microbatch (autograd path)."""
    from meshtrain_b200 import ops

    profiles = []
    x, _ = spec.make_batch(0, microbatch_size)
    with torch.device("meta"), ops.use_backend("torch"):
        h = x.to("meta")
        if h.is_floating_point():
            h = h.to(spec.dtype)
        for i in range(spec.num_layers):
            layer = spec._make_layer(i).to(spec.dtype)
            pcount = sum(p.numel() for p in layer.parameters())
            pbytes = sum(p.numel() * p.element_size() for p in layer.parameters())
            inp = h.detach().requires_grad_(h.is_floating_point())
            counter = FlopCounterMode(display=False)
            with counter:
                saved, y = _saved_bytes_of(layer, inp)
            profiles.append(LayerProfile(i, spec.layer_name(i), pcount, pbytes, inp.numel() * inp.element_size(),
                                         y.numel() * y.element_size(), saved, float(counter.get_total_flops())))
            h = y
    return profiles


def profiles_for(spec, microbatch_size: int) -> list[LayerProfile]:
    """Closed-form profiles for the GPT / Llama families (as the GPU engine runs them), meta-device
    profiling of the autograd modules for every other model."""
    if getattr(spec, "name", "") in ("gpt", "llama"):
        return analytic_profile(spec, microbatch_size)
    return profile_model(spec, microbatch_size)
