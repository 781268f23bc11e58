"""Small deterministic MLP used to prove pipeline-autograd correctness.

Linear and GELU layers alternate over ``sizes`` (default [128, 512, 512, 256,
10] -> 7 partitionable layers); labels are the argmax of a fixed random
teacher (reference models/mlp_test.py:20-59).
"""

from __future__ import annotations

import torch
from torch import nn
from torch.nn import functional as F

from meshtrain_b200 import ops
from meshtrain_b200.models.base import ModelSpec, PipelineLayer


class LinearLayer(PipelineLayer):
    def __init__(self, n_in: int, n_out: int):
        super().__init__()
        self.lin = nn.Linear(n_in, n_out)

    def fwd(self, x, saved):
        saved["x"] = x
        return ops.linear(x, self.lin.weight, self.lin.bias)

    def bwd(self, dy, saved, grads):
        x = saved["x"]
        ops.linear_wgrad_(dy, x, grads["lin.weight"], grads["lin.bias"])
        return ops.linear_dgrad(dy, self.lin.weight)

    def forward(self, x):
        return self.lin(x)


class GELULayer(PipelineLayer):
    def fwd(self, x, saved):
        saved["x"] = x
        return F.gelu(x)

    def bwd(self, dy, saved, grads):
        return dy * ops.gelu_grad(saved["x"])

    def forward(self, x):
        return F.gelu(x)


class MLPSpec(ModelSpec):
    name = "mlp"
    required_ops = ("linear", "gelu", "cross_entropy")

    def __init__(self, sizes: list[int] | None = None, seed: int = 0, dtype: torch.dtype = torch.float32):
        super().__init__(seed, dtype)
        self.sizes = list(sizes or [128, 512, 512, 256, 10])
        if len(self.sizes) < 2:
            raise ValueError("MLP needs at least input and output size")
        self._layers: list[tuple[str, int]] = []
        for i in range(len(self.sizes) - 1):
            self._layers.append(("linear", i))
            if i < len(self.sizes) - 2:
                self._layers.append(("gelu", i))
        g = torch.Generator().manual_seed(seed + 12345)
        self._teacher = torch.randn(self.sizes[0], self.sizes[-1], generator=g)

    @property
    def num_layers(self) -> int:
        return len(self._layers)

    def layer_name(self, index: int) -> str:
        kind, i = self._layers[index]
        return f"{kind}{i}"

    def _make_layer(self, index: int) -> nn.Module:
        kind, i = self._layers[index]
        if kind == "linear":
            return LinearLayer(self.sizes[i], self.sizes[i + 1])
        return GELULayer()

    def loss_fn(self, output, target):
        return F.cross_entropy(output.float(), target)

    def make_batch(self, step: int, batch_size: int):
        g = torch.Generator().manual_seed(self.seed * 100_003 + step)
        x = torch.randn(batch_size, self.sizes[0], generator=g)
        y = (x @ self._teacher).argmax(dim=-1)
        return x.to(self.dtype), y

    def boundary_shape(self, microbatch_size: int):
        raise NotImplementedError("MLP boundaries depend on the cut point")
