"""Compression of boundary tensors on host (TCP) links.

The reference declares ``CompressionPolicy`` (future.py:34-43: ``encode(tensor, link)``
/ ``decode(payload, meta)``) and leaves it empty.  ``Downcast`` implements it by
sending fp32 activations and activation gradients as 16-bit floats: half the
bytes on a slow link (the LAN / emulated 100 Mbit/s setups the host runtime
serves), at the cost of rounding every boundary tensor.  The receiving stage
turns them back into its compute dtype before use.  It is off by default
(``network.compression: none``) because it changes the numerics: a pipeline no
longer matches one process bit for bit.  A reference stage cannot read a 16-bit
payload (its TCP receive path goes through numpy), so compression is for links
between this package's stages only.

Tensors that are not fp32 (token ids, targets, bf16 activations) cross unchanged.
"""

from __future__ import annotations

import torch

from meshtrain_b200.future import CompressionPolicy
from meshtrain_b200.networking.packet import DTYPE_NAMES, WIRE_DTYPES
from meshtrain_b200.networking.serialization import bytes_to_tensor, tensor_to_bytes

WIRE_FORMATS = {"bf16": torch.bfloat16, "fp16": torch.float16}


class Downcast(CompressionPolicy):
    def __init__(self, wire_dtype: torch.dtype):
        if wire_dtype not in (torch.bfloat16, torch.float16):
            raise ValueError(f"wire dtype must be bfloat16 or float16, not {wire_dtype}")
        self.wire_dtype = wire_dtype

    def wire(self, tensor: torch.Tensor) -> torch.Tensor:
        """The tensor as it crosses the link."""
        return tensor.to(self.wire_dtype) if tensor.dtype == torch.float32 else tensor

    def encode(self, tensor, link: tuple[str, str]) -> tuple[bytes, dict]:
        sent = self.wire(tensor.detach().cpu())
        meta = {"dtype": DTYPE_NAMES[sent.dtype], "shape": list(sent.shape), "original": DTYPE_NAMES[tensor.dtype]}
        return tensor_to_bytes(sent), meta

    def decode(self, payload: bytes, meta: dict):
        received = bytes_to_tensor(payload, meta["dtype"], meta["shape"])
        return received.to(WIRE_DTYPES[meta["original"]])


def policy(name: str | None) -> Downcast | None:
    """The policy for ``network.compression`` (None for "none")."""
    if name in (None, "none"):
        return None
    if name not in WIRE_FORMATS:
        raise ValueError(f"unknown link compression {name!r} (none, bf16, fp16)")
    return Downcast(WIRE_FORMATS[name])
