"""DINOv3 backbone + DPT depth head (4 intermediate layers), monocular depth.

Reference: offload/server/model/dinov3_depther.py (load :47, preprocess onto the eval grid :179,
TTA sources :665-756, approx :762, correct :835, head :1087). The backbone runs on the approximate
/ correct engine with taps on the four layers the head reads (evenly spaced, last = final
layer); the head is models/conv.py DPTHead (see its docstring for the differences).

Sources: every image is brought onto the fixed `depther_eval_size` grid (768 in the NYU
profile; bilinear, rounded back to uint8 because the engine's patch embedding reads uint8) and,
with `depther_use_tta`, its horizontal mirror is a second source, so the approximate and
correction passes run once over all sources. The head's depth of a mirrored source is flipped
back, the two are averaged, and the mean is resized to the image's own resolution.
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
        self.eval_size = int(profile.get("depther_eval_size", 0))
        self.tta = bool(profile.get("depther_use_tta", False))
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
        canvas = context["canvas"]
        B, H, W, _ = canvas.shape
        E = self.eval_size or 0
        if E and (H, W) != (E, E):
            x = F.interpolate(canvas.permute(0, 3, 1, 2).float(), size=(E, E), mode="bilinear", align_corners=False)
            canvas = x.round_().clamp_(0, 255).to(torch.uint8).permute(0, 2, 3, 1).contiguous()
        if self.tta:  # sources: the images, then their mirrors
            canvas = torch.cat([canvas, torch.flip(canvas, dims=[2])], 0).contiguous()
        context["depther_layout"] = (B, H, W)
        context["canvas"] = canvas

    def prepare_tokens(self, task, context, config):
        self.backbone_prepare_tokens(context)
        return {}

    def approx_forward(self, params, context, config):
        return self.backbone_approx(params, context, config)

    def correct_forward(self, params, context, config):
        return self.backbone_correct(params, context, config)

    def head_inference(self, task, context, config) -> Dict[str, Any]:
        if self.engine is None:
            raise RuntimeError("the depther head runs on the GPU engine")
        n = context["canvas"].shape[0]
        B, H, W = context.get("depther_layout", (n, *context["canvas"].shape[1:3]))
        sess = context["session"]
        gh, gw = sess.grid_hw
        taps = [self.engine.tap_features(sess, l) for l in self.taps]
        d = self.head_gpu.forward(taps, n, gh, gw)                            # [n, h, w] fp32
        if n == 2 * B:  # mirrored sources: flip back and average with the originals
            d = 0.5 * (d[:B] + torch.flip(d[B:], dims=[2]))
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
