"""Half-block partition units: each transformer block as two pipeline layers.

A stage boundary of the reference always falls between whole layers
(reference planner/partition.py works on the model's layer list).  On B200 a
GPT/Llama block's two residual halves (attention, MLP) take similar time, so
letting a boundary fall between them halves the partition granularity: with
24 blocks and an LM head worth about two blocks over 8 stages, the largest
stage drops from 4 blocks to 3.5.

``SplitBlockSpec`` wraps a GPT or Llama spec.  Unit 0 is the embedding, units
1 .. 2L are the attention and MLP halves of blocks 0 .. L-1, the last unit is
the LM head.  A half is built from its whole block (same per-layer seed, so the
same parameters as the unsplit model) and keeps only its own half's modules,
under the block's parameter names.  ``global_layer(unit)`` is the wrapped
model's layer index, so tensor IDs ``model.layers.<g>.<name>`` and checkpoints
are the same as the unsplit model's.
"""

from __future__ import annotations

from torch import nn

from meshtrain_b200 import ops
from meshtrain_b200.models.base import ModelSpec, PipelineLayer


class BlockHalf(PipelineLayer):
    """The attention (``which`` = 0) or MLP (1) residual half of a block."""

    def __init__(self, block: nn.Module, which: int):
        super().__init__()
        self.which = which
        mine, other = block.HALVES[which], block.HALVES[1 - which]
        for name in other:  # drop the other half's parameters
            setattr(block, name, None)
        for name in mine:
            self.add_module(name, getattr(block, name))
        self.__dict__["_block"] = block  # the arithmetic lives on the block; not a registered submodule

    def fwd(self, x, saved):
        b = self._block
        return b.attn_fwd(x, saved) if self.which == 0 else b.mlp_fwd(x, saved)

    def bwd(self, dy, saved, grads):
        b = self._block
        return b.attn_bwd(dy, saved, grads) if self.which == 0 else b.mlp_bwd(dy, saved, grads)

    def forward(self, x):
        b = self._block
        torch_path = getattr(b, "attn_torch", None) is not None and (ops.backend() == "torch" or not x.is_cuda)
        if torch_path:
            return b.attn_torch(x) if self.which == 0 else b.mlp_torch(x)
        return super().forward(x)


class SplitBlockSpec(ModelSpec):
    """A GPT / Llama spec whose blocks are split into attention and MLP pipeline units."""

    def __init__(self, base: ModelSpec):
        super().__init__(base.seed, base.dtype)
        if not hasattr(base, "n_blocks"):
            raise ValueError("half-block units need a transformer spec (gpt or llama)")
        self.base = base
        self.name = base.name
        self.required_ops = base.required_ops
        self.split_blocks = True

    def __getattr__(self, item):  # model dimensions, data kind, ... of the wrapped spec
        if item == "base":
            raise AttributeError(item)
        return getattr(self.base, item)

    @property
    def num_layers(self) -> int:
        return self.base.num_layers + self.base.n_blocks

    def _unit(self, index: int) -> tuple[int, int | None]:
        """(wrapped layer index, half or None for a whole layer)."""
        if index == 0:
            return 0, None
        if index == self.num_layers - 1:
            return self.base.num_layers - 1, None
        return 1 + (index - 1) // 2, (index - 1) % 2

    def global_layer(self, index: int) -> int:
        return self._unit(index)[0]

    def layer_name(self, index: int) -> str:
        g, half = self._unit(index)
        name = self.base.layer_name(g)
        return name if half is None else f"{name}.{'attn' if half == 0 else 'mlp'}"

    def _make_layer(self, index: int) -> nn.Module:
        g, half = self._unit(index)
        layer = self.base._make_layer(g)
        return layer if half is None else BlockHalf(layer, half)

    def build_layer(self, index: int, device=None) -> nn.Module:
        if not 0 <= index < self.num_layers:
            raise IndexError(index)
        g, half = self._unit(index)
        layer = self.base.build_layer(g, device)  # the wrapped model's seed schedule
        return layer if half is None else BlockHalf(layer, half)

    def loss_fn(self, output, target):
        return self.base.loss_fn(output, target)

    def make_batch(self, step: int, batch_size: int):
        return self.base.make_batch(step, batch_size)

    def boundary_shape(self, microbatch_size: int):
        return self.base.boundary_shape(microbatch_size)

    def flops_per_token(self) -> float:
        return self.base.flops_per_token()

    def parameter_count(self) -> int:
        return self.base.parameter_count()

    def describe(self) -> dict:
        d = self.base.describe()
        d.update(num_layers=self.num_layers, partition_units="half-blocks")
        return d


def split_blocks(spec: ModelSpec) -> ModelSpec:
    return spec if isinstance(spec, SplitBlockSpec) else SplitBlockSpec(spec)


__all__ = ["SplitBlockSpec", "BlockHalf", "split_blocks"]
