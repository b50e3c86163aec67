"""Model executor interface used by the worker's instruction dispatch.

Same operations as the reference ABC (offload/server/model/base.py:125-171): every compute
instruction of a Task maps to one method, and all methods take the per-request `context` dict
that the worker keeps for the session.
"""
from __future__ import annotations

import os
from abc import ABC, abstractmethod
from dataclasses import dataclass
from typing import Any, Dict, Optional

import numpy as np
import torch


@dataclass
class PyramidBatch:
    """Decoded-but-not-reconstructed Laplacian input of a batch.

    base: uint8 [B, h, w, 3] coarsest level. residual: one int16 canvas [B, 2h, 2w, 3] (zeros
    where a patch has not arrived), a list of them from coarse to fine (None entries for levels
    with nothing received), or None for the base-only approximation. `levels` (coarse first)
    fixes how many 2x steps reach full resolution; without it, one step per residual. The server
    reconstructs clip(pyrUp(cur) + residual) level by level on the GPU (kernel `pyrup_add`).
    """

    base: Any
    residual: Any = None
    target_shapes: Optional[list] = None
    levels: Optional[list] = None

    def residual_steps(self) -> list:
        res = self.residual
        if res is None:
            res = []
        elif not isinstance(res, (list, tuple)):
            res = [res]
        if self.levels:
            # one 2x step per level from the base down to level 0; a residual joins the step that
            # lands on its level (residual[i] belongs to levels[i + 1])
            by_level = {lvl: (res[i] if i < len(res) else None) for i, lvl in enumerate(self.levels[1:])}
            return [by_level.get(t) for t in range(self.levels[0] - 1, -1, -1)]
        return [res[i] if i < len(res) else None for i in range(max(len(res), 1))]


def resolve_device(device) -> torch.device:
    if device is None:
        return torch.device("cuda" if torch.cuda.is_available() else "cpu")
    return torch.device(device)


def to_device_uint8_images(batch: Any, device: torch.device) -> torch.Tensor:
    """list / ndarray / tensor of HWC uint8 images -> uint8 [B, H, W, 3] on `device`."""
    if isinstance(batch, torch.Tensor):
        t = batch
        if t.ndim == 3:
            t = t.unsqueeze(0)
        if t.shape[1] == 3 and t.shape[-1] != 3:
            t = t.permute(0, 2, 3, 1)
    else:
        if isinstance(batch, list):
            imgs = [b["image"] if isinstance(b, dict) else b for b in batch]
            arr = np.stack([np.asarray(i) for i in imgs])
        else:
            arr = np.asarray(batch)
            if arr.ndim == 3:
                arr = arr[None]
        if arr.dtype != np.uint8:
            arr = np.clip(arr, 0, 255).astype(np.uint8)
        t = torch.from_numpy(np.ascontiguousarray(arr))
        if device.type == "cuda":
            t = t.pin_memory()
    return t.to(device, non_blocking=True).contiguous()


class ModelExecutor(ABC):
    def __init__(self, device):
        self.device = resolve_device(device)
        self.model = None

    @staticmethod
    def weights_path(profile: Dict[str, Any], key: str) -> Optional[str]:
        p = profile.get(key)
        if not p:
            return None
        p = os.path.expanduser(p)
        return p if os.path.exists(p) else None

    @abstractmethod
    def load_model(self, model_name: str, config: Any): ...

    @abstractmethod
    def preprocess(self, batch_data: Any, task: Any, context: Dict[str, Any], config: Any): ...

    @abstractmethod
    def prepare_tokens(self, task: Any, context: Dict[str, Any], config: Any): ...

    @abstractmethod
    def approx_forward(self, params: Dict[str, Any], context: Dict[str, Any], config: Any): ...

    @abstractmethod
    def correct_forward(self, params: Dict[str, Any], context: Dict[str, Any], config: Any): ...

    @abstractmethod
    def head_inference(self, task: Any, context: Dict[str, Any], config: Any) -> Dict[str, Any]: ...

    @abstractmethod
    def full_inference(self, task: Any, context: Dict[str, Any], config: Any): ...

    def decide_exit(self, task: Any, context: Dict[str, Any], config: Any) -> Dict[str, Any]:
        return {"num_exits": 0}

    @abstractmethod
    def get_final_results(self, task: Any, context: Dict[str, Any], config: Any) -> Dict[int, Any]: ...

    def cache_stats(self, context: Dict[str, Any]) -> Dict[str, Any]:
        """Bytes held by the session's per-layer caches, by family (for InferenceResult)."""
        return {"total": 0, "breakdown": {}}
