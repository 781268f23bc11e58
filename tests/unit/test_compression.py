"""Link compression: fp32 boundary tensors cross host links as 16-bit floats."""

import pytest
import torch

from meshtrain_b200.networking.compression import Downcast, policy


def test_policy_names():
    assert policy(None) is None and policy("none") is None
    assert policy("bf16").wire_dtype is torch.bfloat16 and policy("fp16").wire_dtype is torch.float16
    with pytest.raises(ValueError):
        policy("int8")
    with pytest.raises(ValueError):
        Downcast(torch.float32)


def test_encode_decode_round_trip():
    codec = policy("bf16")
    x = torch.randn(4, 8, 16)
    payload, meta = codec.encode(x, ("a", "b"))
    assert len(payload) == x.numel() * 2 and meta["dtype"] == "bfloat16" and meta["original"] == "float32"
    back = codec.decode(payload, meta)
    assert back.dtype == torch.float32 and back.shape == x.shape
    assert torch.allclose(back, x, rtol=1e-2, atol=1e-2)
    ids = torch.randint(0, 100, (4, 8))
    assert codec.wire(ids) is ids  # token ids and targets cross unchanged
