"""Per-layer profiles used by the planner.

``profile_model`` pushes one microbatch through each layer on the ``meta``
device and records parameters, input/output bytes, autograd-saved bytes and
forward FLOPs (reference planner/graph.py:25-82).  ``analytic_layer_flops``
gives the closed-form forward FLOPs per token of the transformer layers,
which is what the GPU partitioner balances.
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
    output_bytes: int
    saved_bytes: int      # autograd-saved activations per microbatch (reference-style accounting)
    forward_flops: float  # per microbatch

    def to_dict(self) -> dict:
        return asdict(self)


def analytic_layer_flops(spec) -> list[float]:
    """Forward FLOPs per token of each layer (transformer families), else parameter counts."""
    kind = getattr(spec, "name", "")
    if kind in ("gpt", "llama"):
        d, S, V = spec.d_model, spec.seq_len, spec.vocab_size
        if kind == "gpt":
            block = 2 * (4 * d * d + 2 * spec.mlp_ratio * d * d)
        else:
            hd = d // spec.n_heads
            block = 2 * (d * (spec.n_heads + 2 * spec.n_kv_heads) * hd + d * d + 3 * d * spec.ffn_hidden)
        block += 2 * S * d  # causal attention
        head = 2 * d * V + 6 * V  # logits GEMM + softmax-CE
        emb = 4 * d
        return [float(emb)] + [float(block)] * spec.n_blocks + [float(head)]
    return [float(max(c, 1)) for c in spec.layer_parameter_counts()]


def _saved_bytes_of(module, x) -> tuple[int, torch.Tensor]:
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
    """Profile every layer on the meta device with one microbatch."""
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
            profiles.append(LayerProfile(
                index=i, name=spec.layer_name(i), params=pcount, param_bytes=pbytes,
                input_bytes=inp.numel() * inp.element_size(), output_bytes=y.numel() * y.element_size(),
                saved_bytes=saved, forward_flops=float(counter.get_total_flops())))
            h = y
    return profiles
