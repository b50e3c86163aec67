"""Length-prefixed pickle framing for the two TCP channels (uplink, downlink).

Frame = 4-byte big-endian payload length + pickle payload (reference offload/common/network.py:
6-50). Receives read straight into a preallocated buffer with `recv_into` instead of growing a
bytes object, so large residual payloads do not cost quadratic copies.
"""
from __future__ import annotations

import pickle
import socket
import struct
from typing import Any, Optional

_HDR = struct.Struct(">I")
MAX_FRAME = (1 << 32) - 1


def encode_frame(obj: Any) -> bytes:
    body = pickle.dumps(obj, protocol=pickle.HIGHEST_PROTOCOL)
    if len(body) > MAX_FRAME:
        raise ValueError(f"message of {len(body)} bytes exceeds the 4-byte length prefix")
    return _HDR.pack(len(body)) + body


def send_msg(sock: socket.socket, data: Any) -> None:
    """Send one framed message; raises on a broken connection."""
    sock.sendall(encode_frame(data))


def _recv_exact(sock: socket.socket, n: int) -> Optional[memoryview]:
    buf = bytearray(n)
    view = memoryview(buf)
    got = 0
    while got < n:
        try:
            k = sock.recv_into(view[got:], n - got)
        except OSError:
            return None
        if k == 0:
            return None
        got += k
    return view


def recv_msg(sock: socket.socket) -> Optional[Any]:
    """Receive one framed message. Returns None when the peer closed or the link failed."""
    hdr = _recv_exact(sock, _HDR.size)
    if hdr is None:
        return None
    (length,) = _HDR.unpack(hdr)
    body = _recv_exact(sock, length) if length else memoryview(b"")
    if body is None:
        return None
    try:
        return pickle.loads(body)
    except Exception as exc:  # corrupt frame: report and treat as a closed link
        print(f"[network] undecodable frame ({length} bytes): {exc}")
        return None
