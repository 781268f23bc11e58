"""Data-plane packets: a validated JSON header plus an optional raw tensor payload.

Wire-compatible with the reference's ``TensorPacket`` (reference
runtime/tensor_packet.py:19-144): same message-type numbers, dtype names and
header fields, so stages of either implementation can exchange frames.  The
payload is always the C-contiguous bytes of a CPU tensor; nothing is pickled.
"""

from __future__ import annotations

import enum
import math
import uuid
from dataclasses import dataclass, field
from typing import Any

import torch


class MessageType(enum.IntEnum):
    FORWARD_ACTIVATION = 1
    BACKWARD_GRADIENT = 2
    TARGET = 3
    CONTROL = 4
    ACK = 5
    ERROR = 6


WIRE_DTYPES: dict[str, torch.dtype] = {
    "float32": torch.float32, "float64": torch.float64, "float16": torch.float16, "bfloat16": torch.bfloat16,
    "int64": torch.int64, "int32": torch.int32, "int16": torch.int16, "int8": torch.int8, "uint8": torch.uint8,
    "bool": torch.bool,
}
DTYPE_NAMES: dict[torch.dtype, str] = {v: k for k, v in WIRE_DTYPES.items()}
_ITEMSIZE = {name: torch.empty((), dtype=dt).element_size() for name, dt in WIRE_DTYPES.items()}
_SCALARS = (str, int, float, bool, type(None))
MAX_STR = 256
MAX_DIMS = 16


def itemsize(dtype_name: str) -> int:
    return _ITEMSIZE[dtype_name]


def _nonneg_int(v: Any) -> bool:
    return isinstance(v, int) and not isinstance(v, bool) and v >= 0


@dataclass
class TensorPacket:
    message_type: MessageType
    job_id: str = ""
    step_id: int = 0
    microbatch_id: int = 0
    source_worker: str = ""
    destination_worker: str = ""
    shape: tuple[int, ...] = ()
    dtype: str | None = None  # None: no tensor payload
    payload: bytes | memoryview = b""
    tensor_id: str = field(default_factory=lambda: uuid.uuid4().hex[:16])
    meta: dict[str, Any] = field(default_factory=dict)

    @property
    def has_tensor(self) -> bool:
        return self.dtype is not None

    @property
    def expected_payload_bytes(self) -> int:
        return 0 if self.dtype is None else math.prod(self.shape) * itemsize(self.dtype)

    def header(self) -> dict[str, Any]:
        return {
            "tensor_id": self.tensor_id, "job_id": self.job_id, "step_id": self.step_id,
            "microbatch_id": self.microbatch_id, "message_type": int(self.message_type),
            "shape": list(self.shape), "dtype": self.dtype, "source_worker": self.source_worker,
            "destination_worker": self.destination_worker, "meta": self.meta,
        }

    @classmethod
    def from_header(cls, header: Any, payload) -> "TensorPacket":
        """Validate an untrusted header field by field; ValueError on anything unexpected."""
        if not isinstance(header, dict):
            raise ValueError("packet header must be an object")
        try:
            mtype = MessageType(int(header["message_type"]))
        except (KeyError, ValueError, TypeError) as exc:
            raise ValueError(f"invalid message_type: {header.get('message_type')!r}") from exc
        ints = {}
        for name in ("step_id", "microbatch_id"):
            v = header.get(name, 0)
            if not _nonneg_int(v):
                raise ValueError(f"field {name!r} must be a non-negative int")
            ints[name] = v
        strs = {}
        for name in ("job_id", "source_worker", "destination_worker", "tensor_id"):
            v = header.get(name, "")
            if not isinstance(v, str) or len(v) > MAX_STR:
                raise ValueError(f"field {name!r} must be a string of at most {MAX_STR} chars")
            strs[name] = v
        shape = header.get("shape", [])
        if not isinstance(shape, list) or len(shape) > MAX_DIMS or not all(_nonneg_int(d) for d in shape):
            raise ValueError(f"invalid shape: {shape!r}")
        dtype = header.get("dtype")
        if dtype is not None and dtype not in WIRE_DTYPES:
            raise ValueError(f"unsupported dtype: {dtype!r}")
        meta = header.get("meta", {})
        if not isinstance(meta, dict) or not all(isinstance(k, str) and isinstance(v, _SCALARS) for k, v in meta.items()):
            raise ValueError("meta must be a flat object of scalars")
        pkt = cls(message_type=mtype, shape=tuple(shape), dtype=dtype, payload=payload, meta=meta, **ints, **strs)
        if len(payload) != pkt.expected_payload_bytes:
            raise ValueError(f"payload size {len(payload)} does not match shape {tuple(shape)} and dtype {dtype} "
                             f"({pkt.expected_payload_bytes} bytes)")
        return pkt
