"""Worker process: decoder thread -> GPU launcher -> reaper thread
(reference offload/server/worker.py:32-768).

* Decoder thread: accumulates each request's patches and decodes them on the CPU. For the
  Laplacian family on a CUDA device it only unpacks crops (`decode_pyramid`); pixel
  reconstruction happens on the GPU inside LOAD_INPUT. The decoded input travels with the task to
  the launcher, so a later decode never races an earlier launch.
* Launcher (main thread): dispatches every instruction to the model executor without
  synchronising, bracketing each with a CUDA event pair and an NVTX range
  `APPCORR_INSTR|req=..|task=..|seq=..|op=..`.
* Reaper thread: waits for each end event, converts GPU time to wall clock through an anchor
  event, records server events, feeds APPROX_DONE back to the scheduler, builds and sends the
  InferenceResult on SEND_RESPONSE and frees the session on FREE_SESSION.
"""
from __future__ import annotations

import json
import multiprocessing
import queue
import threading
import time
import traceback
from dataclasses import dataclass, field
from typing import Any, Dict, Optional

import numpy as np
import torch

from ..common.protocol import InferenceResult, Instruction, OpType, Task
from ..policies import get_transmission

_SKIPPABLE = {OpType.LOAD_INPUT, OpType.PREPARE_TOKENS, OpType.FULL_INFERENCE, OpType.APPROX_FORWARD,
              OpType.CORRECT_FORWARD, OpType.HEAD_INFERENCE, OpType.DECIDE_EXIT}
_INCREMENTAL_DECODE = {"COCOWindowProgressiveLaplacian", "NYUAppCorrProgressiveLaplacian"}


@dataclass
class MonitorJob:
    op_type: OpType
    req_id: int
    task: Task
    params: dict
    start_ev: Any = None
    end_ev: Any = None
    t_start: float = 0.0
    t_end: float = 0.0
    meta: Any = None


def new_session() -> Dict[str, Any]:
    return {"events": [], "patch_buffer": [], "input": None, "final_results": {}}


class WorkerModule(multiprocessing.Process):
    def __init__(self, input_queue, output_queue, feedback_queue=None, device: Optional[str] = None):
        super().__init__(daemon=True)
        self.input_queue, self.output_queue, self.feedback_queue = input_queue, output_queue, feedback_queue
        self.device_name = device
        self.sessions: Dict[int, Dict[str, Any]] = {}
        self.config = None
        self.policy = None
        self.executor = None
        self._model_identity = None

    # ------------------------------------------------------------------ process
    def run(self):
        self.device = torch.device(self.device_name or ("cuda" if torch.cuda.is_available() else "cpu"))
        if self.device.type == "cuda":
            torch.cuda.set_device(self.device)
        self.gpu_queue: "queue.Queue" = queue.Queue()
        self.monitor_queue: "queue.Queue" = queue.Queue()
        self._config_ready = threading.Event()
        self.anchor_cpu = time.time()
        self.anchor_ev = None
        if self.device.type == "cuda":
            self.anchor_ev = torch.cuda.Event(enable_timing=True)
            self.anchor_ev.record()
        threads = [threading.Thread(target=self.decoder_loop, daemon=True),
                   threading.Thread(target=self.reaper_loop, daemon=True)]
        for t in threads:
            t.start()
        try:
            with torch.inference_mode():
                self.launcher_loop()
        finally:
            if self.device.type == "cuda":
                torch.cuda.synchronize(self.device)
                # ends a `nsys profile --capture-range=cudaProfilerApi` capture at worker exit
                try:
                    torch.cuda.profiler.stop()
                except RuntimeError:
                    pass
            for t in threads:
                t.join(timeout=5)

    # ------------------------------------------------------------------ decoder thread
    def _pyramid_on_gpu(self) -> bool:
        return (self.device.type == "cuda" and hasattr(self.policy, "decode_pyramid")
                and not self.policy.preserve_shape(self.config)
                and type(self.policy).__name__ in {"LaplacianPyramidPolicy", "ProgressiveLPyramidPolicy",
                                                   "NYUAppCorrLaplacianPolicy", "NYUAppCorrProgressiveLaplacianPolicy",
                                                   "COCOWindowProgressiveLaplacianPolicy"})

    def decode_task(self, task: Task, ctx: Dict[str, Any]):
        if not task.payload or not any(i.op_type == OpType.LOAD_INPUT for i in task.instructions):
            return ctx.get("input")
        arrived = max((p.arrival_time for p in task.payload), default=0.0)
        if arrived > 0:
            ctx["events"].append({"type": "SERVER_RECEIVE", "start": arrived, "end": arrived, "params": {},
                                  "timer": "cpu", "detail": False, "include_in_latency_stats": True})
        ctx["patch_buffer"].extend(task.payload)
        patches = ctx["patch_buffer"]
        t0 = time.time()
        if self._pyramid_on_gpu():
            decoded = self.policy.decode_pyramid(patches, self.config)
        else:
            prev = ctx.get("input") if self.config.transmission_policy_name in _INCREMENTAL_DECODE else None
            decoded = self.policy.decode(patches, self.config, canvas=prev)
        ctx["events"].append({"type": "Decode", "start": t0, "end": time.time(), "params": {}, "timer": "cpu",
                              "detail": False, "include_in_latency_stats": True})
        ctx["input"] = decoded
        self._mobile_hint(patches, ctx)
        return decoded

    def _mobile_hint(self, patches, ctx) -> None:
        """Per-token mobile score [B, P] from the finest-level residual patches' pscore_hint."""
        res = [p for p in patches if p.group_id > 0 and p.res_level == 0]
        if not res:
            return
        H, W = self.config.image_shape[:2]
        ph, pw = self.config.patch_size
        hint = ctx.get("mobile_pscore_hint")
        shape = (self.config.batch_size, (H // ph) * (W // pw))
        if not isinstance(hint, torch.Tensor) or tuple(hint.shape) != shape:
            hint = torch.zeros(shape, dtype=torch.float32)
        for p in res:
            if p.image_idx < shape[0] and p.spatial_idx < shape[1]:
                hint[p.image_idx, p.spatial_idx] = float(p.pscore_hint)
        ctx["mobile_pscore_hint"] = hint

    def decoder_loop(self):
        while True:
            msg = self.input_queue.get()
            if msg == "STOP":
                self.gpu_queue.put("STOP")
                return
            kind, payload = msg
            try:
                if kind == "CONFIG":
                    self.config = payload
                    self.policy = get_transmission(payload.transmission_policy_name)
                    self.gpu_queue.put(msg)
                elif kind == "TIME_SYNC":
                    self.gpu_queue.put(msg)
                elif kind == "TASK":
                    self._config_ready.wait()
                    ctx = self.sessions.setdefault(payload.request_id, new_session())
                    self.gpu_queue.put(("TASK", (payload, self.decode_task(payload, ctx))))
            except Exception as exc:
                print(f"!!! [Decoder] {exc}", flush=True)
                traceback.print_exc()

    # ------------------------------------------------------------------ launcher
    def load_model(self) -> None:
        from .model import get_model_executor

        ident = (self.config.model_name, json.dumps(self.config.dataset_kwargs, sort_keys=True, default=str),
                 json.dumps(self.config.input_profile_kwargs, sort_keys=True, default=str), str(self.device))
        if self.executor is not None and ident == self._model_identity:
            return
        self.executor = get_model_executor(self.config.model_name, self.device)
        self.executor.load_model(self.config.model_name, self.config)
        self._model_identity = ident

    def launcher_loop(self):
        while True:
            msg = self.gpu_queue.get()
            if msg == "STOP":
                self.monitor_queue.put("STOP")
                return
            kind, payload = msg
            try:
                if kind == "CONFIG":
                    self.config = payload
                    if payload.device:
                        self.device = torch.device(payload.device)
                    self.sessions = {}
                    try:
                        self.load_model()
                    finally:
                        self._config_ready.set()  # never leave the decoder waiting on a failed load
                    print(f"[Worker] configured: {payload.model_name} on {self.device}", flush=True)
                elif kind == "TIME_SYNC":
                    self.output_queue.put(time.time())
                elif kind == "TASK":
                    task, decoded = payload
                    ctx = self.sessions.setdefault(task.request_id, new_session())
                    ctx["input"] = decoded
                    self.execute(task, ctx)
            except Exception as exc:
                print(f"!!! [Worker] {exc}", flush=True)
                traceback.print_exc()

    def _mark(self):
        if self.device.type == "cuda":
            ev = torch.cuda.Event(enable_timing=True)
            ev.record()
            return ev
        return time.time()

    def execute(self, task: Task, ctx: Dict[str, Any]) -> None:
        try:
            with torch.cuda.nvtx.range(f"APPCORR_SESSION|req={task.request_id}|task={task.task_id}"):
                for ins in task.instructions:
                    seq = ctx.get("_seq", 0)
                    ctx["_seq"] = seq + 1
                    name = f"APPCORR_INSTR|req={task.request_id}|task={task.task_id}|seq={seq}|op={ins.op_type.name}"
                    start = self._mark()
                    with torch.cuda.nvtx.range(name):
                        meta = self.dispatch(ins, task, ctx)
                    end = self._mark()
                    job = MonitorJob(ins.op_type, task.request_id, task, dict(ins.params), meta=meta)
                    if self.device.type == "cuda":
                        job.start_ev, job.end_ev = start, end
                    else:
                        job.t_start, job.t_end = start, end
                    self.monitor_queue.put(job)
        except Exception as exc:
            print(f"!!! [Worker] pipeline error (req {task.request_id}): {exc}", flush=True)
            traceback.print_exc()
            self.sessions.pop(task.request_id, None)
            # answer the client instead of leaving it to its result timeout
            self.output_queue.put(InferenceResult(task.task_id, time.time(), [{"error": str(exc)}] * self.config.batch_size,
                                                  [{"type": "ERROR", "start": time.time(), "end": time.time(),
                                                    "params": {"message": str(exc)}}]))

    def dispatch(self, ins: Instruction, task: Task, ctx: Dict[str, Any]):
        ex, cfg, op = self.executor, self.config, ins.op_type
        ctx.setdefault("active_indices", list(range(cfg.batch_size)))
        if not ctx["active_indices"] and op in _SKIPPABLE:
            return {"skipped": True}
        if op == OpType.LOAD_INPUT:
            if ctx.get("input") is None:
                return None
            return ex.preprocess(ctx["input"], task, ctx, cfg)
        if op == OpType.PREPARE_TOKENS:
            return ex.prepare_tokens(task, ctx, cfg)
        if op == OpType.FULL_INFERENCE:
            return ex.full_inference(task, ctx, cfg)
        if op == OpType.APPROX_FORWARD:
            return ex.approx_forward(ins.params, ctx, cfg)
        if op == OpType.CORRECT_FORWARD:
            return ex.correct_forward(ins.params, ctx, cfg)
        if op == OpType.HEAD_INFERENCE:
            return ex.head_inference(task, ctx, cfg)
        if op == OpType.DECIDE_EXIT:
            return ex.decide_exit(task, ctx, cfg)
        if op == OpType.EXIT_ALL:
            ctx["final_results"].update(ex.get_final_results(task, ctx, cfg))
            ctx["active_indices"] = []
            return None
        if op == OpType.SEND_RESPONSE:
            if ctx["active_indices"]:
                ctx["final_results"].update(ex.get_final_results(task, ctx, cfg))
            fr = ctx["final_results"]
            ctx["_pending_preds"] = [fr.get(i, []) for i in range(cfg.batch_size)] if fr else []
            ctx["_stats"] = ex.cache_stats(ctx)
        return None

    # ------------------------------------------------------------------ reaper
    def _wall(self, ev) -> float:
        return self.anchor_cpu + self.anchor_ev.elapsed_time(ev) / 1000.0

    def reaper_loop(self):
        while True:
            job = self.monitor_queue.get()
            if job == "STOP":
                return
            try:
                if job.end_ev is not None:
                    job.end_ev.synchronize()
                    t0, t1 = self._wall(job.start_ev), self._wall(job.end_ev)
                else:
                    t0, t1 = job.t_start, job.t_end
                ctx = self.sessions.get(job.req_id)
                if ctx is None:
                    continue
                ev = {"type": job.op_type.name, "start": t0, "end": t1, "params": job.params,
                      "timer": "cuda" if job.end_ev is not None else "cpu", "detail": False,
                      "include_in_latency_stats": True}
                if job.meta:
                    ev["meta"] = job.meta
                ctx["events"].append(ev)
                if (job.op_type == OpType.APPROX_FORWARD and self.feedback_queue is not None
                        and not job.params.get("global_only", False)):
                    self.feedback_queue.put(("APPROX_DONE", job.req_id, job.params.get("layers", (0, 0))[1]))
                if job.op_type == OpType.SEND_RESPONSE:
                    self.send_result(job.task, ctx)
                if job.op_type == OpType.FREE_SESSION:
                    self.sessions.pop(job.req_id, None)
            except Exception as exc:
                print(f"!!! [Reaper] {exc}", flush=True)
                traceback.print_exc()

    def send_result(self, task: Task, ctx: Dict[str, Any]) -> None:
        stats = ctx.get("_stats") or {}
        plan = stats.get("plan", {})
        res = InferenceResult(
            task.task_id, time.time(), ctx.get("_pending_preds", []),
            [dict(e) for e in ctx.get("events", [])],
            cache_size_bytes=int(stats.get("total", 0)), cache_breakdown_bytes=dict(stats.get("breakdown", {})),
            token_pscore_kept_mass=float(plan.get("kept_mass", 0.0)),
            token_pscore_full_mass=float(plan.get("full_mass", 0.0)),
            partial_token_kept_patch=float(plan.get("kept_patches", 0.0)),
            partial_token_full_patch=float(plan.get("full_patches", 0.0)),
            partial_token_sample_count=float(plan.get("samples", 0.0)))
        self.output_queue.put(res)
