"""HIVE wire protocol, version 1 (`seedplane/hive/protocol.py:1-80` of the reference).

A frame is a fixed 28-byte header in network byte order — magic b"SPH1", version (u8, 1), message
kind (u8), flags (u16), request id (u64), lease sequence (u64), payload length (u32) — followed by
the payload, compact UTF-8 JSON for every message of v1. The layout and the message numbers are
the reference's, so agents and brokers of either implementation talk to each other. Model tensors
never travel over this protocol.
"""
from __future__ import annotations

import json
import socket
import struct
from dataclasses import dataclass
from enum import IntEnum

MAGIC = b"SPH1"
VERSION = 1
HEADER = struct.Struct("!4sBBHQQI")
MAX_PAYLOAD = 64 * 1024 * 1024


class Message(IntEnum):
    AUTH_CHALLENGE = 1
    AUTH = 2
    HELLO = 3
    READY = 4
    PULL = 5
    WORK = 6
    RESULT = 7
    STOP = 8
    WAIT = 9
    ERROR = 10


@dataclass(frozen=True)
class Frame:
    kind: Message
    request_id: int = 0
    sequence: int = 0
    payload: bytes = b""
    flags: int = 0


def json_payload(value) -> bytes:
    return json.dumps(value, ensure_ascii=False, separators=(",", ":")).encode("utf-8")


def parse_json(payload: bytes):
    return json.loads(payload.decode("utf-8"))


def encode_frame(frame: Frame) -> bytes:
    if len(frame.payload) > MAX_PAYLOAD:
        raise ValueError(f"HIVE payload exceeds {MAX_PAYLOAD} bytes")
    return HEADER.pack(MAGIC, VERSION, int(frame.kind), frame.flags, frame.request_id, frame.sequence,
                       len(frame.payload)) + frame.payload


def send_frame(sock: socket.socket, frame: Frame) -> None:
    sock.sendall(encode_frame(frame))


def recv_exact(sock: socket.socket, size: int) -> bytes:
    """Exactly `size` bytes, however the transport fragments them; ConnectionError on EOF."""
    buf = bytearray(size)
    view = memoryview(buf)
    got = 0
    while got < size:
        n = sock.recv_into(view[got:], size - got)
        if n == 0:
            raise ConnectionError("HIVE peer closed the connection")
        got += n
    return bytes(buf)


def recv_frame(sock: socket.socket) -> Frame:
    magic, version, kind, flags, request_id, sequence, length = HEADER.unpack(recv_exact(sock, HEADER.size))
    if magic != MAGIC:
        raise ValueError("invalid HIVE frame magic")
    if version != VERSION:
        raise ValueError(f"unsupported HIVE protocol version {version}")
    if length > MAX_PAYLOAD:
        raise ValueError(f"HIVE payload length {length} exceeds limit")
    try:
        message = Message(kind)
    except ValueError as exc:
        raise ValueError(f"unknown HIVE message type {kind}") from exc
    return Frame(message, request_id, sequence, recv_exact(sock, length) if length else b"", flags)
