"""Mobile-side TCP endpoints (reference offload/mobile/modules.py:9-105): the sender streams
CONFIG / TIME_SYNC / patches uplink; the receiver forwards results (and time-sync replies) from
the downlink to the source process, reconnecting when the server restarts its sender."""
from __future__ import annotations

import multiprocessing

from ..common.network import recv_msg, send_msg
from ..common.protocol import InferenceResult
from ..server.modules import DOWNLINK_READY, accept_one, connect_with_retry


class MobileSender(multiprocessing.Process):
    def __init__(self, server_ip, server_port, input_queue, listen=False, listen_host="0.0.0.0"):
        super().__init__(daemon=True)
        self.server_ip, self.server_port, self.input_queue = server_ip, server_port, input_queue
        self.listen, self.listen_host = listen, listen_host

    def run(self):
        sock = (accept_one(self.listen_host, self.server_port, "[MobileSender]") if self.listen
                else connect_with_retry(self.server_ip, self.server_port, "[MobileSender]"))
        with sock:
            while True:
                item = self.input_queue.get()
                send_msg(sock, item)
                if item == "STOP":
                    return


class MobileReceiver(multiprocessing.Process):
    def __init__(self, server_ip, server_port, feedback_queue, listen=False, listen_host="0.0.0.0"):
        super().__init__(daemon=True)
        self.server_ip, self.server_port, self.feedback_queue = server_ip, server_port, feedback_queue
        self.listen, self.listen_host = listen, listen_host

    def run(self):
        while True:
            sock = (accept_one(self.listen_host, self.server_port, "[MobileReceiver]") if self.listen
                    else connect_with_retry(self.server_ip, self.server_port, "[MobileReceiver]"))
            with sock:
                while True:
                    msg = recv_msg(sock)
                    if msg is None:
                        print("[MobileReceiver] downlink closed; waiting for reconnect", flush=True)
                        break
                    if isinstance(msg, (InferenceResult, float)):
                        self.feedback_queue.put(msg)
                    elif isinstance(msg, tuple) and msg and msg[0] == DOWNLINK_READY:
                        print(f"[MobileReceiver] downlink ready (server time {msg[1]:.6f})", flush=True)
