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
    """Compact UTF-8 JSON (no spaces after separators, non-ASCII kept as is)."""
    return json.dumps(value, separators=(",", ":"), ensure_ascii=False).encode("utf-8")


def parse_json(payload: bytes):
    return json.loads(bytes(payload).decode("utf-8"))


def encode_frame(frame: Frame) -> bytes:
    n = len(frame.payload)
    if n > MAX_PAYLOAD:
        raise ValueError(f"a HIVE payload of {n} bytes is over the {MAX_PAYLOAD}-byte limit")
    head = HEADER.pack(MAGIC, VERSION, int(frame.kind), frame.flags, frame.request_id, frame.sequence, n)
    return head + bytes(frame.payload)


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
            raise ConnectionError(f"the HIVE peer hung up after {got} of {size} bytes")
        got += n
    return bytes(buf)


def _checked_kind(magic: bytes, version: int, kind: int, length: int) -> Message:
    """The message kind of a header, after the checks that make the rest of it trustworthy."""
    if magic != MAGIC:
        raise ValueError(f"not a HIVE frame (magic {magic!r})")
    if version != VERSION:
        raise ValueError(f"HIVE protocol version {version} is not supported (this side speaks {VERSION})")
    if length > MAX_PAYLOAD:
        raise ValueError(f"a HIVE frame announces {length} payload bytes, over the {MAX_PAYLOAD}-byte limit")
    if kind not in _KINDS:
        raise ValueError(f"HIVE message kind {kind} is unknown")
    return Message(kind)


_KINDS = frozenset(int(m) for m in Message)


def recv_frame(sock: socket.socket) -> Frame:
    magic, version, kind, flags, request_id, sequence, length = HEADER.unpack(recv_exact(sock, HEADER.size))
    message = _checked_kind(magic, version, kind, length)
    payload = recv_exact(sock, length) if length else b""
    return Frame(message, request_id, sequence, payload, flags)
