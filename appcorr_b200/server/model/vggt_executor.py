"""VGGT-style multi-view executor (full inference): frames of one sequence -> per-frame depth and
camera-pose encodings. See models/vggt.py for the model and its relation to the reference
(offload/server/model/vggt_omega.py, which is also full-inference only).

One request = one sequence: the batch axis is the frame axis, as in the reference.
"""
from __future__ import annotations

from typing import Any, Dict

import numpy as np
import torch
import torch.nn.functional as F

from ...models.conv import DPTHead, DPTHeadGPU
from ...models.engine import ViTEngine, random_weights
from ...models.vggt import VGGT_PRESETS, PoseHead
from .base import ModelExecutor
from .dinov3_common import DINOv3BackboneMixin


class VGGTExecutor(ModelExecutor):
    def __init__(self, device):
        super().__init__(device)
        self.engine = None
        self._sessions: Dict = {}

    def load_model(self, model_name: str, config: Any):
        if self.device.type != "cuda":
            raise RuntimeError("the VGGT executor runs on the sm_100a engine (CUDA device required)")
        profile = config.get_input_profile_config()
        self.vc = VGGT_PRESETS[str(profile.get("vggt_arch", "vggt_omega_1b"))]
        seed = int(profile.get("seed", 0))
        cfg = self.vc.vit()
        self.engine = ViTEngine(random_weights(cfg, self.device, seed), self.device,
                                DINOv3BackboneMixin.engine_precision(config))
        self.engine.taps = tuple(self.vc.tap_layers())
        torch.manual_seed(seed)
        self.depth_head = DPTHeadGPU(DPTHead(cfg.embed_dim, features=self.vc.dpt_features).init_weights(seed)
                                     .to(self.device), self.device)
        self.pose_head = PoseHead(cfg.embed_dim).to(self.device).eval()
        self.model = self.engine

    def preprocess(self, batch_data, task, context, config):
        frames = DINOv3BackboneMixin.decode_inputs(self, batch_data, context)   # [S, H, W, 3]
        f = self.vc.frame
        if frames.shape[1] != f or frames.shape[2] != f:
            frames = F.interpolate(frames.permute(0, 3, 1, 2).float(), size=(f, f), mode="bilinear",
                                   align_corners=False).round().clamp(0, 255).to(torch.uint8).permute(0, 2, 3, 1)
        context["frames"] = frames
        context["canvas"] = frames.reshape(1, -1, f, 3).contiguous()   # frames stacked top to bottom

    def prepare_tokens(self, task, context, config):
        canvas = context["canvas"]
        _, H, W, _ = canvas.shape
        sess = self._sessions.get((H, W))
        if sess is None:
            sess = self.engine.new_session(1, H, W)
            self._sessions = {(H, W): sess}
        self.engine.prepare_tokens(sess, canvas)
        context["session"] = sess
        return {}

    def approx_forward(self, params, context, config):
        raise NotImplementedError("VGGT runs full inference (as in the reference)")

    def correct_forward(self, params, context, config):
        raise NotImplementedError("VGGT runs full inference (as in the reference)")

    def full_inference(self, task, context, config):
        if "session" not in context:
            self.prepare_tokens(task, context, config)
        sess = context["session"]
        self.engine.approx(sess, 0, self.engine.cfg.depth, "none")
        self.head_inference(task, context, config)

    def head_inference(self, task, context, config) -> Dict[str, Any]:
        sess = context["session"]
        S = context["frames"].shape[0]
        g = self.vc.frame // self.vc.patch
        taps = [self.engine.tap_features(sess, l) for l in self.engine.taps]     # [S*g*g, D] each
        depth = self.depth_head.forward(taps, S, g, g)
        context["depth"] = F.interpolate(depth[:, None], size=(self.vc.frame, self.vc.frame), mode="bilinear",
                                         align_corners=False)[:, 0]
        pooled = self.engine.normed_tokens(sess).view(S, g * g, -1).float().mean(1)
        with torch.no_grad():
            context["pose_enc"] = self.pose_head(pooled)
        return {}

    def get_final_results(self, task, context, config) -> Dict[int, Any]:
        if "depth" not in context:
            return {}
        return {0: {"depth": context["depth"].float().cpu().numpy(),
                    "pose_enc": context["pose_enc"].float().cpu().numpy(),
                    "num_frames": int(context["depth"].shape[0])}}
