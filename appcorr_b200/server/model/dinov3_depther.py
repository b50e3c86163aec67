"""DINOv3 backbone + DPT depth head (4 intermediate layers), monocular depth.

Reference: offload/server/model/dinov3_depther.py (load :47, approx :762, correct :835, head
:1087). The backbone runs on the approximate / correct engine with taps on the four layers the
head reads (evenly spaced, last = final layer); the head is models/conv.py DPTHead (see its
docstring for the differences). Output: fp32 depth at the input resolution.
"""
from __future__ import annotations

from typing import Any, Dict, List

import numpy as np
import torch
import torch.nn.functional as F

from ...models.conv import DPTHead, DPTHeadGPU
from .base import ModelExecutor
from .dinov3_common import DINOv3BackboneMixin


def tap_layers(depth: int, n: int = 4) -> List[int]:
    return [depth * (i + 1) // n - 1 for i in range(n)]


class DINOv3DeptherExecutor(DINOv3BackboneMixin, ModelExecutor):
    default_arch = "vit7b16"

    def __init__(self, device):
        super().__init__(device)
        self._init_backbone_state()
        self.head = None
        self.head_gpu = None

    def load_model(self, model_name: str, config: Any):
        profile = config.get_input_profile_config()
        self.load_backbone(model_name, config)
        self.taps = tap_layers(self.cfg.depth)
        if self.engine is not None:
            if getattr(self.engine, "world", 1) > 1:
                raise RuntimeError("the depther's dense taps run on single-GPU engines (use data parallelism)")
            self.engine.taps = tuple(self.taps)
        feats = int(profile.get("dpt_features", 256))
        head = DPTHead(self.cfg.embed_dim, features=feats)
        path = self.weights_path(profile, "depther_head_weights_path")
        if path is not None:
            head.load_state_dict(torch.load(path, map_location="cpu", weights_only=True), strict=True)
        else:
            head.init_weights(int(profile.get("seed", 0)))
        self.head = head.eval().to(self.device)
        if self.device.type == "cuda":
            self.head_gpu = DPTHeadGPU(self.head, self.device)
        self.model = self.engine or self.backbone

    def preprocess(self, batch_data, task, context, config):
        self.decode_inputs(batch_data, context)

    def prepare_tokens(self, task, context, config):
        self.backbone_prepare_tokens(context)
        return {}

    def approx_forward(self, params, context, config):
        return self.backbone_approx(params, context, config)

    def correct_forward(self, params, context, config):
        return self.backbone_correct(params, context, config)

    def head_inference(self, task, context, config) -> Dict[str, Any]:
        canvas = context["canvas"]
        B, H, W, _ = canvas.shape
        if self.engine is not None:
            sess = context["session"]
            gh, gw = sess.grid_hw
            taps = [self.engine.tap_features(sess, l) for l in self.taps]
            d = self.head_gpu.forward(taps, B, gh, gw)
        else:
            raise RuntimeError("the depther head runs on the GPU engine")
        context["depth"] = F.interpolate(d[:, None], size=(H, W), mode="bilinear", align_corners=False)[:, 0]
        return {}

    def full_inference(self, task, context, config):
        self.backbone_full(context, config)
        self.head_inference(task, context, config)

    def get_final_results(self, task, context, config) -> Dict[int, Any]:
        depth = context.get("depth")
        if depth is None:
            return {}
        host = depth.cpu().numpy()
        idx = context.get("active_indices")
        order = list(range(host.shape[0])) if idx is None else [int(i) for i in idx]
        return {orig: {"depth": np.ascontiguousarray(host[orig])} for orig in order if orig < host.shape[0]}

    def cache_stats(self, context):
        return self.backbone_cache_stats(context)
