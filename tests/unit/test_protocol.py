import struct

import pytest
import torch
from hypothesis import given, settings, strategies as st

from meshtrain_b200.networking.packet import DTYPE_NAMES, MessageType, TensorPacket
from meshtrain_b200.networking.protocol import (MAGIC, PREFIX, ProtocolError, decode_packet, encode_packet,
                                               parse_prefix)
from meshtrain_b200.networking.serialization import packet_to_tensor, tensor_to_packet


def _pkt(**kw):
    t = torch.arange(12, dtype=torch.float32).reshape(3, 4)
    return tensor_to_packet(t, MessageType.FORWARD_ACTIVATION, job_id="j", step_id=2, microbatch_id=1,
                            source_worker="a", destination_worker="b", **kw)


def test_roundtrip_keeps_header_and_tensor():
    p = _pkt()
    q = decode_packet(encode_packet(p))
    assert q.header() == p.header()
    assert torch.equal(packet_to_tensor(q), torch.arange(12, dtype=torch.float32).reshape(3, 4))


def test_prefix_layout_is_msht_v1():
    frame = encode_packet(_pkt())
    magic, version, reserved, hlen, plen = PREFIX.unpack(frame[:PREFIX.size])
    assert (magic, version, reserved, plen) == (MAGIC, 1, 0, 48)
    assert PREFIX.size == 18 and len(frame) == 18 + hlen + 48


@pytest.mark.parametrize("dtype", list(DTYPE_NAMES))
def test_all_wire_dtypes(dtype):
    t = (torch.randn(5, 3) * 10).to(dtype)
    q = decode_packet(encode_packet(tensor_to_packet(t, MessageType.BACKWARD_GRADIENT)))
    assert torch.equal(packet_to_tensor(q), t)


def test_non_contiguous_and_empty_tensors():
    t = torch.randn(4, 6).t()
    assert torch.equal(packet_to_tensor(decode_packet(encode_packet(tensor_to_packet(t, MessageType.TARGET)))), t)
    e = torch.empty(0, 7)
    assert packet_to_tensor(decode_packet(encode_packet(tensor_to_packet(e, MessageType.TARGET)))).shape == (0, 7)


def test_rejects_bad_prefix():
    frame = encode_packet(_pkt())
    with pytest.raises(ProtocolError, match="magic"):
        decode_packet(b"XXXX" + frame[4:])
    with pytest.raises(ProtocolError, match="version"):
        decode_packet(frame[:4] + b"\x02" + frame[5:])
    with pytest.raises(ProtocolError):
        parse_prefix(frame[:10])
    with pytest.raises(ProtocolError, match="exceeds"):
        parse_prefix(frame[:PREFIX.size], max_payload_bytes=8)


def test_rejects_payload_size_mismatch_and_bad_fields():
    p = _pkt()
    p.payload = bytes(p.payload)[:-4]
    with pytest.raises(ProtocolError):
        decode_packet(encode_packet(p))
    for field, value in [("step_id", -1), ("dtype", "complex128"), ("message_type", 99), ("shape", [-1, 2]),
                         ("job_id", "x" * 1000)]:
        h = _pkt().header()
        h[field] = value
        import json
        head = json.dumps(h).encode()
        frame = PREFIX.pack(MAGIC, 1, 0, len(head), 48) + head + bytes(48)
        with pytest.raises(ProtocolError):
            decode_packet(frame)


def test_control_packet_without_tensor():
    p = TensorPacket(MessageType.CONTROL, job_id="j", meta={"kind": "stop", "n": 3})
    q = decode_packet(encode_packet(p))
    assert not q.has_tensor and q.meta == {"kind": "stop", "n": 3}


@settings(max_examples=200, deadline=None)
@given(st.binary(min_size=0, max_size=200))
def test_random_bytes_never_crash_the_decoder(data):
    try:
        decode_packet(data)
    except ProtocolError:
        pass


@settings(max_examples=100, deadline=None)
@given(st.integers(0, 3), st.lists(st.integers(0, 4), min_size=0, max_size=4), st.integers(0, 2**31))
def test_roundtrip_random_shapes(kind, shape, step):
    t = torch.randn(*shape) if shape else torch.randn(())
    p = tensor_to_packet(t, MessageType(kind + 1), step_id=step)
    q = decode_packet(encode_packet(p))
    assert q.step_id == step and torch.equal(packet_to_tensor(q), t)


def test_header_length_field_is_checked():
    frame = bytearray(encode_packet(_pkt()))
    struct.pack_into(">I", frame, 6, 0)
    with pytest.raises(ProtocolError, match="header length"):
        decode_packet(bytes(frame))
