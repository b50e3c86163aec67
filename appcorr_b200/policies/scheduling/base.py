"""Instruction-list building blocks shared by the scheduling policies."""
from __future__ import annotations

from typing import List, Optional

from ...common.protocol import ExperimentConfig, Instruction, OpType, Patch, normalize_appcorr_kwargs

I = Instruction


def total_layers(config: ExperimentConfig, default: int = 40) -> int:
    return int(config.scheduler_kwargs.get("total_layers", config.transmission_kwargs.get("total_layers", default)))


def spread_boundaries(total: int, n: int) -> List[int]:
    """n+1 layer boundaries splitting `total` layers into n chunks, remainder to the first ones."""
    n = max(int(n), 1)
    base, rem = divmod(total, n)
    out = [0]
    for i in range(n):
        out.append(out[-1] + base + (1 if i < rem else 0))
    out[-1] = total
    return out


def load_prepare() -> List[Instruction]:
    return [I(OpType.LOAD_INPUT), I(OpType.PREPARE_TOKENS)]


def approx(start: int, end: int, **extra) -> Instruction:
    return I(OpType.APPROX_FORWARD, {"layers": (start, end), **extra})


def correct(end: int, group_id: int, start: int = 0) -> Instruction:
    return I(OpType.CORRECT_FORWARD, {"layers": (start, end), "group_id": group_id})


def finish(exit_all: bool = True) -> List[Instruction]:
    out = [I(OpType.HEAD_INFERENCE)]
    if exit_all:
        out.append(I(OpType.EXIT_ALL))
    return out + [I(OpType.SEND_RESPONSE), I(OpType.FREE_SESSION)]


def early_exit_probe() -> List[Instruction]:
    return [I(OpType.HEAD_INFERENCE), I(OpType.DECIDE_EXIT)]


def appcorr_active(config: ExperimentConfig) -> bool:
    opts = normalize_appcorr_kwargs(config.appcorr_kwargs, config.transmission_kwargs)
    return bool(opts.get("enabled", False) or opts.get("generated_from_client", False))


def detector_global_mode(config: ExperimentConfig) -> Optional[str]:
    """The detector's global-source mode when the client generated the global source, else None."""
    if getattr(config, "model_name", None) != "dinov3_detector":
        return None
    ak = getattr(config, "appcorr_kwargs", {}) or {}
    if not bool(ak.get("generated_from_client", False)):
        return None
    mode = str(ak.get("global_source_mode", "global_first"))
    return mode if mode in {"global_first", "final_correct", "approx"} else "global_first"


def global_source_approx(config: ExperimentConfig) -> Instruction:
    return approx(0, total_layers(config), global_only=True, source_kind="global")


def head_group(buffer: List[Patch]) -> Optional[tuple]:
    """(group_id, batch_group_total) of the front group when it is complete, else None."""
    if not buffer:
        return None
    head = buffer[0]
    if len(buffer) < head.batch_group_total:
        return None
    return head.group_id, head.batch_group_total


def patches_per_image(config: ExperimentConfig) -> int:
    H, W = config.image_shape[:2]
    ph, pw = config.patch_size
    keep_shape = bool(config.transmission_kwargs.get("preserve_input_shape", False))
    if config.transmission_policy_name in {"Laplacian", "ProgressiveLaplacian"}:
        total = 0
        for lvl in sorted(config.transmission_kwargs.get("pyramid_levels", [2, 1, 0]), reverse=True):
            s = 2 ** lvl
            h, w = (min(H, W) // s,) * 2 if keep_shape else (H // s, W // s)
            total += (-(-h // ph)) * (-(-w // pw))
        return total
    if keep_shape:
        return 1
    return (-(-H // ph)) * (-(-W // pw))


def whole_batch_size(buffer: List[Patch], config: ExperimentConfig, num_groups: Optional[int]) -> Optional[int]:
    """Patches in a complete batch (all transmission groups), or None while incomplete."""
    expected = (num_groups or 1) + 1 if config.transmission_policy_name == "ProgressiveLaplacian" else 1
    totals = {}
    for p in buffer:
        totals.setdefault(p.group_id, p.batch_group_total)
    if len(totals) < expected:
        return None
    total = sum(totals.values())
    if total <= 0:
        total = config.batch_size * patches_per_image(config)
    return total if len(buffer) >= total else None
