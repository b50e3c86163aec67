"""TCP endpoints of the server: the uplink receiver and the downlink sender (one process each).

Protocol (reference offload/server/modules.py:9-169): the uplink's first message is
('CONFIG', ExperimentConfig); later messages are Patch objects (stamped with their arrival time
here), ('TIME_SYNC', t) tuples or 'STOP'. The downlink first sends (DOWNLINK_READY, server_time)
and then results; on a broken downlink the sender reconnects and resends the pending result.
Either side may listen or, with reverse connect, dial the mobile.
"""
from __future__ import annotations

import multiprocessing
import socket
import time

from ..common.network import recv_msg, send_msg

DOWNLINK_READY = "__APPCORR_DOWNLINK_READY__"


def connect_with_retry(host: str, port: int, label: str, retry_s: float = 1.0, max_tries: int = 0) -> socket.socket:
    tries = 0
    while True:
        s = socket.socket(socket.AF_INET, socket.SOCK_STREAM)
        s.settimeout(5.0)
        try:
            s.connect((host, port))
            s.settimeout(None)
            s.setsockopt(socket.IPPROTO_TCP, socket.TCP_NODELAY, 1)
            print(f"{label} connected to {host}:{port}", flush=True)
            return s
        except OSError as exc:
            s.close()
            tries += 1
            if max_tries and tries >= max_tries:
                raise
            print(f"{label} connection failed ({exc}); retrying in {retry_s}s", flush=True)
            time.sleep(retry_s)


def accept_one(host: str, port: int, label: str) -> socket.socket:
    with socket.socket(socket.AF_INET, socket.SOCK_STREAM) as srv:
        srv.setsockopt(socket.SOL_SOCKET, socket.SO_REUSEADDR, 1)
        srv.bind((host, port))
        srv.listen(1)
        print(f"{label} listening on {host}:{port}", flush=True)
        conn, addr = srv.accept()
    conn.setsockopt(socket.IPPROTO_TCP, socket.TCP_NODELAY, 1)
    print(f"{label} connection from {addr}", flush=True)
    return conn


class ServerReceiver(multiprocessing.Process):
    def __init__(self, port, sched_queue, control_queue, shutdown_event, listen_host="0.0.0.0", connect_host=None):
        super().__init__(daemon=True)
        self.port, self.sched_queue, self.control_queue = port, sched_queue, control_queue
        self.shutdown_event = shutdown_event
        self.listen_host, self.connect_host = listen_host, connect_host

    def run(self):
        conn = (connect_with_retry(self.connect_host, self.port, "[ServerReceiver]") if self.connect_host
                else accept_one(self.listen_host, self.port, "[ServerReceiver]"))
        with conn:
            self.handle(conn)
        print("[ServerReceiver] uplink closed; requesting shutdown", flush=True)
        self.shutdown_event.set()

    def handle(self, conn) -> None:
        first = recv_msg(conn)
        if not (isinstance(first, tuple) and first and first[0] == "CONFIG"):
            if isinstance(first, tuple) and first and first[0] == "ERROR":
                print(f"[ServerReceiver] client reported an error before CONFIG: {first[1]}", flush=True)
            else:
                print(f"[ServerReceiver] handshake failed: expected CONFIG, got {type(first).__name__}", flush=True)
            return
        print(f"[ServerReceiver] handshake ok, scheduler {first[1].scheduler_policy_name}", flush=True)
        self.control_queue.put(first)
        while True:
            msg = recv_msg(conn)
            if msg is None or msg == "STOP":
                return
            if isinstance(msg, tuple):
                if msg and msg[0] == "TIME_SYNC":
                    self.control_queue.put(msg)
                else:
                    print(f"[ServerReceiver] ignoring control message {msg[0]!r}", flush=True)
                continue
            if hasattr(msg, "arrival_time"):
                msg.arrival_time = time.time()
            self.sched_queue.put(msg)


class ServerSender(multiprocessing.Process):
    def __init__(self, port, input_queue, listen_host="0.0.0.0", connect_host=None):
        super().__init__(daemon=True)
        self.port, self.input_queue = port, input_queue
        self.listen_host, self.connect_host = listen_host, connect_host

    def run(self):
        pending = None
        while True:
            conn = (connect_with_retry(self.connect_host, self.port, "[ServerSender]") if self.connect_host
                    else accept_one(self.listen_host, self.port, "[ServerSender]"))
            try:
                with conn:
                    send_msg(conn, (DOWNLINK_READY, time.time()))
                    pending = self.pump(conn, pending)
                    if pending == "STOP":
                        return
            except OSError as exc:
                print(f"[ServerSender] link lost ({exc}); reconnecting", flush=True)

    def pump(self, conn, pending):
        item = pending
        while True:
            if item is None:
                item = self.input_queue.get()
            if item == "STOP":
                return "STOP"
            try:
                send_msg(conn, item)
            except OSError as exc:
                print(f"[ServerSender] send failed ({exc}); will resend after reconnect", flush=True)
                return item
            item = None
