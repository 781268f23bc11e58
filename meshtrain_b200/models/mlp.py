"""A small deterministic MLP: the model the pipeline's gradient-equivalence tests train.

It has the role of the reference's test MLP (models/mlp_test.py:20-59): layers
whose boundaries have different widths, cheap enough to run many stages on
a CPU, with an exact single-process oracle.  Each layer carries an explicit
forward/backward pair for the device engine and a plain ``forward`` for the
autograd path.
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
    """Linear layers of widths ``sizes`` with a GELU between consecutive ones.

    Every Linear and every GELU is its own partitionable layer, so the default
    widths [128, 512, 512, 256, 10] give 7 layers and boundaries of every
    width.  Labels come from a fixed random linear teacher (the argmax of
    ``x @ T``), so the task is learnable and the loss falls within a few steps.
    """

    name = "mlp"
    required_ops = ("linear", "gelu", "cross_entropy")
    DEFAULT_SIZES = (128, 512, 512, 256, 10)

    def __init__(self, sizes: list[int] | None = None, seed: int = 0, dtype: torch.dtype = torch.float32):
        super().__init__(seed, dtype)
        self.sizes = list(sizes) if sizes else list(self.DEFAULT_SIZES)
        if len(self.sizes) < 2:
            raise ValueError("MLP needs at least input and output size")
        # (kind, index of the linear it follows): linear0 gelu0 linear1 gelu1 ... linearN
        kinds = [("linear", i) if j == 0 else ("gelu", i)
                 for i in range(len(self.sizes) - 1) for j in range(2 if i < len(self.sizes) - 2 else 1)]
        self._layers = kinds
        teacher_rng = torch.Generator().manual_seed(seed + 12345)
        self._teacher = torch.randn(self.sizes[0], self.sizes[-1], generator=teacher_rng)

    @property
    def num_layers(self) -> int:
        return len(self._layers)

    def layer_name(self, index: int) -> str:
        kind, i = self._layers[index]
        return f"{kind}{i}"

    def _make_layer(self, index: int) -> nn.Module:
        kind, i = self._layers[index]
        return LinearLayer(self.sizes[i], self.sizes[i + 1]) if kind == "linear" else GELULayer()

    def loss_fn(self, output, target):
        return F.cross_entropy(output.float(), target)

    def make_batch(self, step: int, batch_size: int):
        rng = torch.Generator().manual_seed(self.seed * 100_003 + step)  # the per-step data seed
        x = torch.randn(batch_size, self.sizes[0], generator=rng)
        labels = torch.argmax(x @ self._teacher, dim=-1)
        return x.to(self.dtype), labels

    def boundary_shape(self, microbatch_size: int):
        raise NotImplementedError("MLP boundaries depend on the cut point")
