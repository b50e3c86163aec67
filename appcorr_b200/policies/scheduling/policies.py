"""Scheduling policies: turn buffered patches (and approx-progress feedback) into Tasks.

Three families, each a small configurable class rather than one file per policy:

* Whole-batch   wait for every group, then one pass (BatchCountBased, ADE20KSequential;
                reference scheduling/batch_count.py:5-89, ade20k_sequential.py:7-107).
* Two-phase     base group -> approx over all layers; residual -> correct + head
                (ADE20KApproxCorrect, NYUApproxCorrect; ade20k_approx_correct.py:7-99,
                nyu_approx_correct.py:7-93).
* Interleaved   transmission overlapped with compute: group g corrects layers [0, frontier) for
                the tokens it carried, then the approximate frontier advances, either by a fixed
                layer chunk per group (static: GroupTrigger, ADE20KWindowInterleaved,
                COCOWindowInterleaved; group_trigger.py:65-117, ade20k_window_trigger.py:8-97,
                coco_window_trigger.py:91-196) or one layer at a time to stay `ahead_layers` in
                front of the reaper's APPROX_DONE feedback (dynamic: DynamicGroupTrigger,
                ADE20KInterleavedDynamic, COCOWindowDynamic; dynamic_group_trigger.py:33-163,
                ade20k_interleaved_dynamic.py:8-194, coco_window_trigger.py:199-366).
  VGGTInterleaved splits the 48-stage VGGT axis by measured per-stage cost
  (vggt_interleaved.py:36-187).
"""
from __future__ import annotations

from typing import Any, List, Optional

from ...common.protocol import ExperimentConfig, Instruction, OpType, Patch, Task
from ..interface import ISchedulingPolicy
from .base import (
    I,
    appcorr_active,
    approx,
    correct,
    detector_global_mode,
    early_exit_probe,
    finish,
    global_source_approx,
    head_group,
    load_prepare,
    spread_boundaries,
    total_layers,
    whole_batch_size,
)


# ------------------------------------------------------------------------------ whole batch
class BatchCountBasedPolicy(ISchedulingPolicy):
    """Every group of the batch first, then FULL_INFERENCE (or approx-only over all layers)."""

    def __init__(self, config: Optional[ExperimentConfig] = None):
        self._num_groups = config.transmission_kwargs.get("num_groups") if config else None

    def _instructions(self, config: ExperimentConfig) -> List[Instruction]:
        if bool(config.scheduler_kwargs.get("approx_only", False)):
            L = int(config.transmission_kwargs.get("total_layers", 40))
            return load_prepare() + [approx(0, L)] + finish(exit_all=True)
        return [I(OpType.LOAD_INPUT), I(OpType.FULL_INFERENCE), I(OpType.SEND_RESPONSE), I(OpType.FREE_SESSION)]

    def decide(self, buffer: List[Patch], config: ExperimentConfig, task_id_gen: Any, **kwargs) -> Optional[Task]:
        if not buffer:
            return None
        if self._num_groups is None:
            self._num_groups = config.transmission_kwargs.get("num_groups")
        n = whole_batch_size(buffer, config, self._num_groups)
        if n is None:
            return None
        tid = next(task_id_gen)
        return Task(task_id=tid, request_id=tid, payload=buffer[:n], instructions=self._instructions(config))


class ADE20KSequentialPolicy(BatchCountBasedPolicy):
    """Whole batch through the decomposed path: prepare -> approx(all layers) -> head."""

    def _instructions(self, config: ExperimentConfig) -> List[Instruction]:
        return load_prepare() + [approx(0, total_layers(config))] + finish(exit_all=False)


# ------------------------------------------------------------------------------ two phase
class _TwoPhasePolicy(ISchedulingPolicy):
    def __init__(self, config: Optional[ExperimentConfig] = None):
        self._request_id: Optional[int] = None

    def decide(self, buffer: List[Patch], config: ExperimentConfig, task_id_gen: Any, **kwargs) -> Optional[Task]:
        hg = head_group(buffer)
        if hg is None:
            return None
        group, count = hg
        tid = next(task_id_gen)
        L = total_layers(config)
        if group == 0:
            self._request_id = tid
            return Task(tid, tid, buffer[:count], load_prepare() + [approx(0, L)])
        ins = load_prepare()
        if appcorr_active(config):
            ins.append(correct(L, group_id=0))
        ins += finish(exit_all=False)
        rid = self._request_id if self._request_id is not None else tid
        return Task(tid, rid, buffer[:count], ins)


class ADE20KApproxCorrectPolicy(_TwoPhasePolicy):
    pass


class NYUApproxCorrectPolicy(_TwoPhasePolicy):
    pass


# ------------------------------------------------------------------------------ interleaved (static)
class GroupTriggerPolicy(ISchedulingPolicy):
    """Static interleave with chunk = total_layers // num_groups (floor)."""

    def __init__(self, config: Optional[ExperimentConfig] = None):
        self.current_request_id: Optional[int] = None

    def decide(self, buffer: List[Patch], config: ExperimentConfig, task_id_gen: Any, **kwargs) -> Optional[Task]:
        hg = head_group(buffer)
        if hg is None:
            return None
        group, count = hg
        tid = next(task_id_gen)
        if group == 0 or self.current_request_id is None:
            self.current_request_id = tid
        return Task(tid, self.current_request_id, buffer[:count], self._pipeline(group, config))

    def _pipeline(self, g: int, config: ExperimentConfig) -> List[Instruction]:
        L = config.transmission_kwargs.get("total_layers", 40)
        n = config.transmission_kwargs.get("num_groups", 4)
        chunk = L // n
        ins = load_prepare()
        if g < n:
            lo, hi = g * chunk, (g + 1) * chunk
            if lo > 0:
                ins.append(correct(lo, g))
            ins.append(approx(lo, hi))
            if config.early_exit_enabled():
                ins += early_exit_probe()
            return ins
        ins.append(correct(L, g))
        if detector_global_mode(config) == "final_correct":
            ins.append(global_source_approx(config))
        return ins + finish()


class ADE20KWindowInterleavedPolicy(ISchedulingPolicy):
    """Static interleave whose group count is the per-image crop count carried by the patches."""

    def __init__(self, config: Optional[ExperimentConfig] = None):
        self.current_request_id: Optional[int] = None
        self.num_groups = 1

    def decide(self, buffer: List[Patch], config: ExperimentConfig, task_id_gen: Any, **kwargs) -> Optional[Task]:
        hg = head_group(buffer)
        if hg is None:
            return None
        group, count = hg
        tid = next(task_id_gen)
        if group == 0 or self.current_request_id is None:
            self.current_request_id = tid
            self.num_groups = 1
        n = int(getattr(buffer[0], "num_correction_groups", 0) or 0)
        if n > 0:
            self.num_groups = n
        return Task(tid, self.current_request_id, buffer[:count], self._pipeline(group, config))

    def _pipeline(self, g: int, config: ExperimentConfig) -> List[Instruction]:
        L = total_layers(config)
        n = max(self.num_groups, 1)
        b = spread_boundaries(L, n)
        ins = load_prepare()
        if g < n:
            if g > 0 and b[g] > 0:
                ins.append(correct(b[g], g))
            ins.append(approx(b[g], b[g + 1]))
            return ins
        return ins + [correct(L, g)] + finish()


class _FrontierMixin:
    """Tracks the deepest approximate layer already queued for the current request."""

    frontier: int = 0

    def _catch_up(self, ins: List[Instruction], g: int, to_end: int, L: int, **approx_extra) -> None:
        if self.frontier > 0:
            ins.append(correct(self.frontier, g))
        if self.frontier < to_end:
            ins.append(approx(self.frontier, to_end, **approx_extra))
            self.frontier = to_end


class COCOWindowInterleavedPolicy(_FrontierMixin, ISchedulingPolicy):
    """Fixed 3x3 detector windows (9 groups); static frontier over spread boundaries."""

    DEFAULT_WINDOW_GROUPS = 9

    def __init__(self, config: Optional[ExperimentConfig] = None):
        self.current_request_id: Optional[int] = None
        self.frontier = 0

    @classmethod
    def _num_windows(cls, config: ExperimentConfig) -> int:
        return int(config.scheduler_kwargs.get("num_window_groups",
                                               config.transmission_kwargs.get("num_window_groups",
                                                                              cls.DEFAULT_WINDOW_GROUPS)))

    def decide(self, buffer: List[Patch], config: ExperimentConfig, task_id_gen: Any, **kwargs) -> Optional[Task]:
        hg = head_group(buffer)
        if hg is None:
            return None
        group, count = hg
        tid = next(task_id_gen)
        if group == 0 or self.current_request_id is None:
            self.current_request_id = tid
            self.frontier = 0
        return Task(tid, self.current_request_id, buffer[:count], self._pipeline(group, config))

    def _pipeline(self, g: int, config: ExperimentConfig) -> List[Instruction]:
        L = total_layers(config)
        n = self._num_windows(config)
        b = spread_boundaries(L, n)
        mode = detector_global_mode(config)
        ins = load_prepare()
        if g == 0:
            if mode == "global_first":
                ins.append(global_source_approx(config))
            if self.frontier < b[1]:
                ins.append(approx(self.frontier, b[1], source_kind="local"))
                self.frontier = b[1]
            return ins
        if g < n:
            if self.frontier > 0:
                ins.append(correct(self.frontier, g))
            nxt = b[min(g + 1, n)]
            if self.frontier < nxt:
                ins.append(approx(self.frontier, nxt, source_kind="local"))
                self.frontier = nxt
            return ins
        self._catch_up(ins, g, L, L, source_kind="local")
        if mode == "final_correct":
            ins.append(global_source_approx(config))
        return ins + finish()


# ------------------------------------------------------------------------------ interleaved (dynamic)
class _DynamicFrontierPolicy(_FrontierMixin, ISchedulingPolicy):
    """Approximation runs ahead one layer at a time, `ahead_layers` in front of the deepest layer
    the reaper reported done; each residual group corrects [0, frontier) on arrival."""

    approx_extra: dict = {"source_kind": "local"}

    def __init__(self, config: Optional[ExperimentConfig] = None):
        self.current_request_id: Optional[int] = None
        self.frontier = 0
        self.current_group = -1
        self.ahead_layers = 2
        self.num_groups = 4
        if config is not None:
            self.ahead_layers = int(config.scheduler_kwargs.get("ahead_layers",
                                                                config.transmission_kwargs.get("ahead_layers", 2)))
            self.num_groups = self._configured_groups(config)

    def _configured_groups(self, config: ExperimentConfig) -> int:
        return int(config.scheduler_kwargs.get("num_groups", config.transmission_kwargs.get("num_groups", 4)))

    def _refresh_groups(self, config: ExperimentConfig, head: Patch) -> None:
        """Hook: update self.num_groups from the arriving group's header."""

    def _start_request(self, tid: int) -> None:
        self.current_request_id = tid
        self.frontier = 0
        self.current_group = 0

    def _run_ahead(self, ins: List[Instruction], config: ExperimentConfig, done: int) -> None:
        L = total_layers(config)
        if self.current_group == -1 or self.current_group >= self.num_groups:
            return
        lead = self.frontier - int(done)
        while lead < self.ahead_layers and self.frontier < L:
            ins.append(approx(self.frontier, self.frontier + 1, **self.approx_extra))
            self.frontier += 1
            lead += 1

    def decide(self, buffer: List[Patch], config: ExperimentConfig, task_id_gen: Any, **kwargs) -> Optional[Task]:
        feedback = kwargs.get("feedback_events", []) or []
        done = max(feedback) if feedback else None
        hg = head_group(buffer)
        if hg is not None:
            group, count = hg
            tid = next(task_id_gen)
            self._refresh_groups(config, buffer[0])
            if group == 0 or self.current_request_id is None:
                self._start_request(tid)
            if group != 0:
                self.current_group = group
            return Task(tid, self.current_request_id, buffer[:count], self._payload(group, config, done))
        if done is not None:
            ins: List[Instruction] = []
            self._run_ahead(ins, config, done)
            if ins:
                return Task(next(task_id_gen), self.current_request_id, [], ins)
        return None

    # hooks for the detector's global source
    def _on_first_group(self, ins: List[Instruction], config: ExperimentConfig) -> None:
        pass

    def _before_finish(self, ins: List[Instruction], config: ExperimentConfig) -> None:
        pass

    def _payload(self, g: int, config: ExperimentConfig, done: Optional[int]) -> List[Instruction]:
        L = total_layers(config)
        ins = load_prepare()
        if g == 0:
            self._on_first_group(ins, config)
            self._run_ahead(ins, config, done or 0)
            return ins
        if g < self.num_groups:
            if self.frontier > 0:
                ins.append(correct(self.frontier, g))
            if done is not None:
                self._run_ahead(ins, config, done)
            self._after_correct(ins, config)
            return ins
        self._catch_up(ins, g, L, L, **self.approx_extra)
        self._before_finish(ins, config)
        return ins + finish()

    def _after_correct(self, ins: List[Instruction], config: ExperimentConfig) -> None:
        if config.early_exit_enabled():
            ins += early_exit_probe()


class DynamicGroupTriggerPolicy(_DynamicFrontierPolicy):
    """Group-count from transmission_kwargs; the first `ahead_layers` layers are queued as soon as
    a group arrives with nothing approximated yet."""

    approx_extra: dict = {}

    def _configured_groups(self, config: ExperimentConfig) -> int:
        return int(config.transmission_kwargs.get("num_groups", 4))

    def _refresh_groups(self, config: ExperimentConfig, head: Patch) -> None:
        self.num_groups = self._configured_groups(config)

    def _start_request(self, tid: int) -> None:
        super()._start_request(tid)
        self.current_group = -1

    def _payload(self, g: int, config: ExperimentConfig, done: Optional[int]) -> List[Instruction]:
        L = total_layers(config)
        ins = load_prepare()
        self.current_group = g
        if g < self.num_groups:
            if self.frontier > 0:
                ins.append(correct(self.frontier, g))
            if self.frontier == 0:
                for _ in range(self.ahead_layers):
                    if self.frontier < L:
                        ins.append(approx(self.frontier, self.frontier + 1))
                        self.frontier += 1
            if config.early_exit_enabled():
                ins += early_exit_probe()
            return ins
        self._catch_up(ins, g, L, L)
        if detector_global_mode(config) == "final_correct":
            ins.append(global_source_approx(config))
        return ins + finish()


class ADE20KInterleavedDynamicPolicy(_DynamicFrontierPolicy):
    def _refresh_groups(self, config: ExperimentConfig, head: Patch) -> None:
        n = int(getattr(head, "num_correction_groups", 0) or 0)
        if n > 0:
            self.num_groups = n


class COCOWindowDynamicPolicy(_DynamicFrontierPolicy):
    def _configured_groups(self, config: ExperimentConfig) -> int:
        return COCOWindowInterleavedPolicy._num_windows(config)

    def _refresh_groups(self, config: ExperimentConfig, head: Patch) -> None:
        self.num_groups = self._configured_groups(config)

    def _on_first_group(self, ins: List[Instruction], config: ExperimentConfig) -> None:
        if detector_global_mode(config) == "global_first":
            ins.append(global_source_approx(config))

    def _before_finish(self, ins: List[Instruction], config: ExperimentConfig) -> None:
        if detector_global_mode(config) == "final_correct":
            ins.append(global_source_approx(config))

    def _after_correct(self, ins: List[Instruction], config: ExperimentConfig) -> None:
        pass


# ------------------------------------------------------------------------------ VGGT
class VGGTInterleavedPolicy(ISchedulingPolicy):
    """One correction round per residual group over the 48-stage VGGT axis, with round
    boundaries at equal cumulative measured cost ("compute"), equal stage count ("uniform") or
    all at full depth ("full", a control)."""

    STAGE_COST_PATCH_EMBED = 28.7 / 24
    STAGE_COST_FRAME = 35.2 / 24
    STAGE_COST_GLOBAL = 25.7 / 19
    STAGE_COST_REGISTER = 1.2 / 5
    REGISTER_BLOCKS = (2, 6, 9, 14, 20)
    PATCH_EMBED_STAGES = 24

    def __init__(self, config: Optional[ExperimentConfig] = None):
        self._request_id: Optional[int] = None

    @classmethod
    def stage_costs(cls, depth: int, config: ExperimentConfig) -> List[float]:
        pe = int(config.scheduler_kwargs.get("pe_stages", cls.PATCH_EMBED_STAGES))
        reg = set(config.scheduler_kwargs.get("register_block_indices", cls.REGISTER_BLOCKS))
        costs = [cls.STAGE_COST_PATCH_EMBED] * min(pe, depth)
        costs += [cls.STAGE_COST_FRAME + (cls.STAGE_COST_REGISTER if i in reg else cls.STAGE_COST_GLOBAL)
                  for i in range(depth - len(costs))]
        return costs

    @classmethod
    def boundaries(cls, depth: int, rounds: int, config: ExperimentConfig) -> List[int]:
        if rounds <= 1:
            return [depth]
        mode = str(config.scheduler_kwargs.get("layer_split", "compute"))
        if mode == "full":
            return [depth] * rounds
        if mode == "uniform":
            return [min(depth, round(depth * (r + 1) / rounds)) for r in range(rounds)]
        if mode != "compute":
            raise ValueError(f"layer_split must be 'compute', 'uniform' or 'full', got {mode!r}")
        costs = cls.stage_costs(depth, config)
        total = sum(costs)
        out, acc, r = [], 0.0, 1
        for i, c in enumerate(costs):
            acc += c
            while r <= rounds and acc >= total * r / rounds - 1e-9:
                out.append(i + 1)
                r += 1
        out += [depth] * (rounds - len(out))
        return [min(x, depth) for x in out[:rounds]]

    def decide(self, buffer: List[Patch], config: ExperimentConfig, task_id_gen: Any, **kwargs) -> Optional[Task]:
        hg = head_group(buffer)
        if hg is None:
            return None
        group, count = hg
        rounds = max(1, int(config.transmission_kwargs.get("correction_groups", 1)))
        depth = total_layers(config, default=48)
        on = appcorr_active(config)
        tid = next(task_id_gen)
        b = self.boundaries(depth, rounds, config)
        ins = load_prepare()
        if group == 0:
            self._request_id = tid
            ins.append(approx(0, b[0]))
        else:
            prev, here = b[group - 1], b[min(group, rounds - 1)]
            if on and prev > 0:
                ins.append(correct(prev, group))
            if here > prev:
                ins.append(approx(prev, here))
            if group >= rounds:
                if on and prev < depth:
                    ins.append(correct(depth, group))
                ins += finish(exit_all=False)
        rid = self._request_id if self._request_id is not None else tid
        return Task(tid, rid, buffer[:count], ins)
