"""Scheduler process: buffers patches, feeds them (and approx-progress feedback) to the
scheduling policy, forwards Tasks to the worker (reference offload/server/scheduler.py:9-85).

Instead of a fixed 1 ms sleep, the loop blocks up to 1 ms on the patch queue, so a newly arrived
patch is scheduled without waiting out a poll period.
"""
from __future__ import annotations

import itertools
import multiprocessing
import queue
from typing import List

from ..common.protocol import Patch
from ..policies import get_scheduler


def drain(q, limit: int = 1 << 16) -> list:
    out = []
    for _ in range(limit):
        try:
            out.append(q.get_nowait())
        except queue.Empty:
            break
    return out


class SchedulerModule(multiprocessing.Process):
    def __init__(self, input_queue, worker_queue, control_queue, feedback_queue=None):
        super().__init__(daemon=True)
        self.input_queue, self.worker_queue = input_queue, worker_queue
        self.control_queue, self.feedback_queue = control_queue, feedback_queue
        self.buffer: List[Patch] = []
        self.config = None
        self.policy = None
        self.task_ids = itertools.count()

    def handle_control(self, cmd, data) -> bool:
        if cmd == "CONFIG":
            self.config = data
            self.policy = get_scheduler(data.scheduler_policy_name, data)
            self.buffer = []
            self.task_ids = itertools.count()
            self.worker_queue.put(("CONFIG", data))
            print(f"[Scheduler] configured with {data.scheduler_policy_name}", flush=True)
        elif cmd == "TIME_SYNC":
            self.worker_queue.put(("TIME_SYNC", data))
        elif cmd == "STOP":
            self.worker_queue.put("STOP")
            return False
        return True

    def step(self, feedback: list) -> None:
        """Let the policy emit every Task the current buffer and feedback allow."""
        if self.policy is None or self.config is None:
            return
        while True:
            kw = {"feedback_events": feedback} if feedback else {}
            task = self.policy.decide(self.buffer, self.config, self.task_ids, **kw)
            feedback = []
            if task is None:
                return
            self.buffer = self.buffer[len(task.payload):]
            self.worker_queue.put(("TASK", task))

    def run(self):
        print("[Scheduler] started", flush=True)
        while True:
            for msg in drain(self.control_queue):
                cmd, data = msg if isinstance(msg, tuple) else (msg, None)
                if not self.handle_control(cmd, data):
                    return
            try:
                self.buffer.append(self.input_queue.get(timeout=0.001))
            except queue.Empty:
                pass
            self.buffer.extend(drain(self.input_queue))
            feedback = []
            if self.feedback_queue is not None:
                feedback = [d for (kind, _req, d) in drain(self.feedback_queue) if kind == "APPROX_DONE"]
            self.step(feedback)
