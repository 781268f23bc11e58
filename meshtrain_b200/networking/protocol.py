"""MSHT v1 framing of TensorPackets (big-endian; reference networking/protocol.py:25-91).

    offset size field
    0      4    magic b"MSHT"
    4      1    version (1)
    5      1    reserved (0)
    6      4    header length (UTF-8 JSON)
    10     8    payload length
    18     H    header
    18+H   P    payload

Kept byte-identical to the reference so mixed deployments interoperate.
"""

from __future__ import annotations

import json
import struct

from meshtrain_b200.networking.packet import TensorPacket

MAGIC = b"MSHT"
VERSION = 1
PREFIX = struct.Struct(">4sBBIQ")
PREFIX_SIZE = PREFIX.size
MAX_HEADER_BYTES = 64 * 1024
DEFAULT_MAX_PAYLOAD_BYTES = 2 * 1024 ** 3


class ProtocolError(ValueError):
    """A malformed, oversized or otherwise invalid frame."""


def encode_head(packet: TensorPacket) -> bytes:
    header = json.dumps(packet.header(), separators=(",", ":")).encode()
    if len(header) > MAX_HEADER_BYTES:
        raise ProtocolError(f"header too large ({len(header)} bytes)")
    return PREFIX.pack(MAGIC, VERSION, 0, len(header), len(packet.payload)) + header


def encode_packet(packet: TensorPacket) -> bytes:
    return encode_head(packet) + bytes(packet.payload)


def parse_prefix(prefix: bytes, max_payload_bytes: int = DEFAULT_MAX_PAYLOAD_BYTES) -> tuple[int, int]:
    if len(prefix) != PREFIX_SIZE:
        raise ProtocolError("truncated frame prefix")
    magic, version, _reserved, hlen, plen = PREFIX.unpack(prefix)
    if magic != MAGIC:
        raise ProtocolError(f"bad magic {magic!r}")
    if version != VERSION:
        raise ProtocolError(f"unsupported protocol version {version}")
    if not 0 < hlen <= MAX_HEADER_BYTES:
        raise ProtocolError(f"invalid header length {hlen}")
    if plen > max_payload_bytes:
        raise ProtocolError(f"payload of {plen} bytes exceeds limit {max_payload_bytes}")
    return hlen, plen


def parse_header(raw: bytes):
    try:
        return json.loads(bytes(raw).decode("utf-8"))
    except (UnicodeDecodeError, json.JSONDecodeError) as exc:
        raise ProtocolError(f"malformed header: {exc}") from exc


def packet_from_header(header, payload) -> TensorPacket:
    try:
        return TensorPacket.from_header(header, payload)
    except ValueError as exc:
        raise ProtocolError(str(exc)) from exc


def decode_body(header_bytes: bytes, payload) -> TensorPacket:
    return packet_from_header(parse_header(header_bytes), payload)


def decode_packet(frame: bytes, max_payload_bytes: int = DEFAULT_MAX_PAYLOAD_BYTES) -> TensorPacket:
    hlen, plen = parse_prefix(frame[:PREFIX_SIZE], max_payload_bytes)
    if len(frame) != PREFIX_SIZE + hlen + plen:
        raise ProtocolError("frame length does not match prefix")
    return decode_body(frame[PREFIX_SIZE:PREFIX_SIZE + hlen], frame[PREFIX_SIZE + hlen:])
