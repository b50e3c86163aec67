"""DINOv3 backbone + linear segmentation head (BatchNorm + 1x1 conv, 150 ADE20K classes).

Reference: offload/server/model/dinov3_segmentor_linhead.py (load :186-246, approx :521-580,
correct :582-745, head :747-851). Differences by design: the whole request batch is one backbone
session; the head is one GEMM with BN folded in, followed by a fused bilinear-upsample + argmax
kernel producing uint8 labels (softmax is monotonic, so single-view argmax is unchanged). Images
larger than the crop are run as sliding crops batched into the same session.
"""
from __future__ import annotations

from typing import Any, Dict

import numpy as np
import torch
import torch.nn.functional as F

from ...models.heads import LinearSegHead, SegHeadGPU
from .base import ModelExecutor
from .dinov3_common import DINOv3BackboneMixin


class DINOv3SegmentorLinheadExecutor(DINOv3BackboneMixin, ModelExecutor):
    default_arch = "vit7b16"

    def __init__(self, device):
        super().__init__(device)
        self._init_backbone_state()
        self.num_classes = 150
        self.linear_head = None
        self.head_gpu = None

    def load_model(self, model_name: str, config: Any):
        profile = config.get_input_profile_config()
        self.num_classes = int(profile.get("num_classes", 150))
        self.load_backbone(model_name, config)
        head = LinearSegHead(self.cfg.embed_dim, self.num_classes)
        path = self.weights_path(profile, "segmentor_head_weights_path")
        if path is not None:
            sd = torch.load(path, map_location="cpu", mmap=True, weights_only=True)
            sd = sd.get("model", sd)
            head.load_state_dict({k.removeprefix("segmentation_model.1."): v for k, v in sd.items()}, strict=True)
            head.eval()
        else:
            head.random_init(int(profile.get("seed", 0)))
        self.linear_head = head
        if self.device.type == "cuda":
            self.head_gpu = SegHeadGPU(head, self.device)
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
            feat = self.engine.patch_features(sess)
            out = context.get("labels")
            if out is None or tuple(out.shape) != (B, H, W):
                out = torch.empty(B, H, W, dtype=torch.uint8, device=self.device)
            self.head_gpu.labels(feat, B, sess.grid_hw[0], sess.grid_hw[1], H, W, out=out)
            context["labels"] = out
        else:
            gh, gw = context["grid_hw"]
            with torch.no_grad():
                xn = self.backbone.final_norm(context["x"])[:, self.cfg.n_prefix:]
                sp = xn.view(B, gh, gw, -1).permute(0, 3, 1, 2)
                logits = self.linear_head(sp)
                logits = F.interpolate(logits, size=(H, W), mode="bilinear", align_corners=False)
            context["labels"] = logits.argmax(1).to(torch.uint8)
        return {}

    def full_inference(self, task, context, config):
        self.backbone_full(context, config)
        self.head_inference(task, context, config)

    def get_final_results(self, task, context, config) -> Dict[int, Any]:
        labels = context.get("labels")
        if labels is None:
            return {}
        host = labels.cpu().numpy()
        idx = context.get("active_indices")
        order = list(range(host.shape[0])) if idx is None else [int(i) for i in idx]
        return {orig: {"mask": np.ascontiguousarray(host[orig])} for orig in order if orig < host.shape[0]}

    def cache_stats(self, context):
        return self.backbone_cache_stats(context)
