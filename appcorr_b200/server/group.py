"""Multi-rank serving behind `offload.server.main --tp N --dp M`.

The reference worker is a single process on one GPU (offload/server/worker.py:32-768). Here a
server hosts M data-parallel replicas of N tensor-parallel ranks each (one process per GPU):

    scheduler --(request_id % M)--> replica r:  leader (rank 0 of the replica)
                                                  decoder thread -> launcher -> reaper -> sender
                                                  every (task, decoded input) is published once
                                                  into a shared-memory broadcast ring
                                                followers (ranks 1..N-1)
                                                  read the ring and run the same instructions;
                                                  their kernels meet the leader's in the fused
                                                  tensor-parallel collectives

Only the leader answers the client. The ring (appcorr_b200._runtime.ShmRing, C++) carries each
task once, however many followers there are; its waits are bounded.

Group health (parallel/health.py). Every rank beats a heartbeat in the replica's store. Between
two requests the leader checks the group: a rank that announced its exit (`bye/<rank>`) or whose
heartbeat stopped is dead. The leader then publishes a REFORM record with the survivors; the
survivors build a new process group over themselves (plan_fallback picks the largest usable
tensor-parallel degree; left-over survivors go idle), reload the model at that degree and keep
serving. A rank leaves only between requests, with nothing of its in flight.

On a CPU host (no tensor-parallel engine) the ranks of a replica each run the executor on the
whole model and, after every task, all-reduce a digest of their results over the group, so the
group, the ring and the re-forming are exercised end to end (the serving test over gloo).
"""
from __future__ import annotations

import os
import pickle
import time
import traceback
import zlib
from typing import Any, Dict, List, Optional

import torch

from ..common.protocol import OpType, Task
from ..policies import get_transmission
from .worker import WorkerModule, new_session

RING_CAPACITY = 1 << 27          # 128 MiB of records per replica
_DECODER_KEYS = ("mobile_pscore_hint",)
HB_INTERVAL = 0.1
HB_TIMEOUT = 2.0


class ReplicaRouter:
    """worker_queue stand-in for the scheduler: TASKs go to replica request_id % M, CONFIG and
    STOP to every replica, TIME_SYNC to replica 0 (one answer)."""

    def __init__(self, queues: List[Any]):
        self.queues = list(queues)

    def put(self, msg) -> None:
        if msg == "STOP":
            for q in self.queues:
                q.put("STOP")
            return
        kind, payload = msg
        if kind == "TASK":
            self.queues[payload.request_id % len(self.queues)].put(msg)
        elif kind == "TIME_SYNC":
            self.queues[0].put(msg)
        else:
            for q in self.queues:
                q.put(msg)


def _digest(preds) -> float:
    """Order-independent number summarising a task's predictions (replica consistency check)."""
    try:
        blob = pickle.dumps(preds, protocol=4)
    except Exception:
        blob = repr(preds).encode()
    return float(zlib.crc32(blob) % 1000003)


class GroupWorker(WorkerModule):
    """One rank of a replica. Rank 0 behaves like WorkerModule and also publishes every task to
    the ring; ranks > 0 execute the published stream."""

    def __init__(self, input_queue, output_queue, feedback_queue, *, replica: int, rank: int, tp: int,
                 port: int, ring_name: str, device: Optional[str] = None, leave_after: int = -1):
        super().__init__(input_queue, output_queue, feedback_queue, device=device)
        self.replica, self.rank, self.tp = replica, rank, tp
        self.port, self.ring_name = port, ring_name
        self.leave_after = leave_after  # test hook: a follower that leaves after this many tasks
        self.members: List[int] = list(range(tp))
        self.group = None
        self._seen: set = set()

    # ------------------------------------------------------------------ group
    def _init_group(self) -> None:
        import torch.distributed as dist

        from ..parallel.health import Heartbeat

        backend = "nccl" if (torch.cuda.is_available() and self.device.type == "cuda") else "gloo"
        import datetime

        self.store = dist.TCPStore("127.0.0.1", self.port, self.tp, self.rank == 0,
                                   timeout=datetime.timedelta(seconds=60))
        # a short collective timeout: a member that vanished ends the next collective with an
        # error instead of a long hang
        dist.init_process_group(backend, store=self.store, rank=self.rank, world_size=self.tp,
                                timeout=datetime.timedelta(seconds=60))
        self.group = None  # the default group until a re-form
        self.hb = Heartbeat(self.store, self.rank, self.tp, interval=HB_INTERVAL)
        from .. import _runtime

        if self.rank == 0:
            self.ring = _runtime.ShmRing(self.ring_name, RING_CAPACITY, max(self.tp - 1, 1), True)
            self.store.set("ring_ready", "1")
        else:
            self.store.wait(["ring_ready"])
            self.ring = _runtime.ShmRing(self.ring_name, create=False)

    def _dead(self) -> List[int]:
        dead = set(self.hb.dead_ranks(HB_TIMEOUT))
        for r in self.members:
            if r != 0 and self.store.check([f"bye/{r}"]):
                dead.add(r)
        return sorted(r for r in dead if r in self.members)

    def _publish(self, kind: str, payload) -> None:
        if self.tp == 1:
            return
        rec = pickle.dumps((kind, payload), protocol=pickle.HIGHEST_PROTOCOL)
        deadline = time.monotonic() + 30.0
        while not self.ring.push(rec, 1.0):
            dead = self._dead()
            if dead:  # a follower died without reading: stop waiting for it
                for r in dead:
                    if 0 < r < self.tp and self.ring.attached(r - 1):
                        self.ring.detach(r - 1)
            if time.monotonic() > deadline:
                raise RuntimeError("ring: followers stopped reading")

    def _reform_if_needed(self) -> None:
        """Leader, between requests: drop dead ranks and rebuild the group over the survivors."""
        if self.tp == 1 or len(self.members) == 1:
            return
        dead = self._dead()
        if not dead:
            return
        from ..parallel.health import plan_fallback

        alive = [r for r in self.members if r not in dead]
        cfg = getattr(self.executor, "cfg", None)
        heads = getattr(cfg, "num_heads", 64) if cfg is not None else 64
        hidden = getattr(cfg, "ffn_hidden", 64) if cfg is not None else 64
        plan = plan_fallback(alive, heads, hidden)
        new_members = plan.groups[0] if plan.groups else [0]
        for r in dead + [r for r in alive if r not in new_members]:
            if 0 < r < self.tp and self.ring.attached(r - 1):
                self.ring.detach(r - 1)
        print(f"[Group {self.replica}] ranks {dead} left; re-forming over {new_members} (tp={plan.tp})", flush=True)
        self._publish("REFORM", {"members": new_members, "idle": [r for r in alive if r not in new_members]})
        self._apply_reform(new_members)

    def _apply_reform(self, members: List[int]) -> None:
        from ..parallel.health import reform_group

        self.members = list(members)
        self.group = reform_group(self.members) if len(self.members) > 1 else None
        if self.config is not None and self.rank in self.members:
            self.config.tp_size = len(self.members) if self._tp_engine() else 1
            self.executor = None
            self.load_model()

    def _tp_engine(self) -> bool:
        return self.device.type == "cuda" and self.tp > 1

    def _group_size(self) -> int:
        return len(self.members)

    # ------------------------------------------------------------------ model
    def load_model(self) -> None:
        """A fresh executor for the current group: the tensor-parallel engine shards over the
        group's members (GPU); CPU ranks each hold the whole model."""
        from .model import get_model_executor

        self.config.tp_size = self._group_size() if self._tp_engine() else 1
        ex = get_model_executor(self.config.model_name, self.device)
        ex.tp_group = self.group
        ex.load_model(self.config.model_name, self.config)
        self.executor = ex

    # ------------------------------------------------------------------ process
    def run(self):
        self.device = torch.device(self.device_name or ("cuda" if torch.cuda.is_available() else "cpu"))
        if self.device.type == "cuda":
            torch.cuda.set_device(self.device)
        try:
            self._init_group()
            if self.rank == 0:
                super_run = WorkerModule.run
                super_run(self)
            else:
                with torch.inference_mode():
                    self.follower_loop()
        except Exception as exc:
            print(f"!!! [Group {self.replica}/{self.rank}] {exc}", flush=True)
            traceback.print_exc()
        finally:
            try:
                self.hb.stop()
            except Exception:
                pass
            if self.rank == 0:
                try:
                    self.ring.close()
                    self.ring.unlink()
                except Exception:
                    pass

    # leader: the WorkerModule loops, with publishing and health checks folded in
    def launcher_loop(self):
        while True:
            msg = self.gpu_queue.get()
            if msg == "STOP":
                self._publish("STOP", None)
                self.monitor_queue.put("STOP")
                return
            kind, payload = msg
            try:
                if kind == "CONFIG":
                    self._publish("CONFIG", payload)
                    self.config = payload
                    self.sessions = {}
                    try:
                        self.load_model()
                    finally:
                        self._config_ready.set()
                    print(f"[Group {self.replica}] configured: {payload.model_name} on {self.device}, "
                          f"tp={self._group_size()}", flush=True)
                elif kind == "TIME_SYNC":
                    self.output_queue.put(time.time())
                elif kind == "TASK":
                    task, decoded = payload
                    if task.request_id not in self._seen:  # first task of a request
                        self._seen.add(task.request_id)
                        self._reform_if_needed()
                    ctx = self.sessions.setdefault(task.request_id, new_session())
                    # the decoder's side products travel with the task (mobile score hints)
                    extras = {k: ctx[k] for k in _DECODER_KEYS if k in ctx}
                    self._publish("TASK", (task, decoded, extras))
                    ctx["input"] = decoded
                    self.execute(task, ctx)
                    self._consistency(task, ctx)
            except Exception as exc:
                print(f"!!! [Group {self.replica}] {exc}", flush=True)
                traceback.print_exc()

    def _consistency(self, task: Task, ctx: Dict[str, Any]) -> None:
        """CPU group: every rank all-reduces the digest of its predictions after a response task;
        the leader checks that all members agree."""
        if self._tp_engine() or len(self.members) == 1 or self.rank not in self.members:
            return
        if not any(i.op_type == OpType.SEND_RESPONSE for i in task.instructions):
            return
        import torch.distributed as dist

        d = _digest(ctx.get("_pending_preds", []))
        t = torch.tensor([d, d * d, 1.0], dtype=torch.float64)
        dist.all_reduce(t, group=self.group)
        n = t[2].item()
        mean = t[0].item() / n
        if abs(t[1].item() / n - mean * mean) > 1e-6 * max(1.0, mean * mean):
            print(f"!!! [Group {self.replica}] replica ranks disagree on request {task.request_id}", flush=True)
        ctx["_group_size"] = int(n)

    # follower
    def follower_loop(self):
        cid = self.rank - 1
        done = 0
        sessions: Dict[int, Dict[str, Any]] = {}
        while True:
            rec = self.ring.pop(cid, 1.0)
            if rec is None:
                if self.ring.closed():
                    return
                continue
            kind, payload = pickle.loads(rec)
            if kind == "STOP":
                return
            if kind == "CONFIG":
                self.config = payload
                self.policy = get_transmission(payload.transmission_policy_name)
                sessions = {}
                self.load_model()
            elif kind == "REFORM":
                if self.rank not in payload["members"]:
                    print(f"[Group {self.replica}/{self.rank}] idle after re-form", flush=True)
                    return
                self._apply_reform(payload["members"])
            elif kind == "TASK":
                task, decoded, extras = payload
                ctx = sessions.setdefault(task.request_id, new_session())
                ctx["input"] = decoded
                ctx.update(extras)
                for ins in task.instructions:
                    self.dispatch(ins, task, ctx)
                    if ins.op_type == OpType.FREE_SESSION:
                        sessions.pop(task.request_id, None)
                leaving = False
                if any(i.op_type == OpType.SEND_RESPONSE for i in task.instructions):
                    done += 1
                    # test hook: leave between requests. The exit is announced before this
                    # request's last collective, so the leader sees it before the next request.
                    leaving = 0 <= self.leave_after <= done
                    if leaving:
                        self.store.set(f"bye/{self.rank}", "1")
                self._consistency(task, ctx)
                if leaving:
                    print(f"[Group {self.replica}/{self.rank}] leaving after {done} requests", flush=True)
                    return


def launch_group(tp: int, dp: int, worker_q, result_q, feedback_q, device: Optional[str], ctx, base_port: int,
                 leave: Optional[Dict[int, int]] = None):
    """Processes of M replicas x N ranks, and the scheduler-side router. Devices: cuda:(r*N + t)
    when CUDA is present (and no --device override), else the CPU."""
    leave = leave or {}
    queues = [ctx.Queue() for _ in range(dp)]
    procs = []
    for r in range(dp):
        ring = f"/appcorr_ring_{os.getpid()}_{r}"
        for t in range(tp):
            dev = device
            if dev is None and torch.cuda.is_available():
                dev = f"cuda:{r * tp + t}"
            procs.append(GroupWorker(queues[r] if t == 0 else ctx.Queue(), result_q, feedback_q, replica=r, rank=t,
                                     tp=tp, port=base_port + r, ring_name=ring, device=dev,
                                     leave_after=leave.get(r * tp + t, -1)))
    return ReplicaRouter(queues), procs
