"""DINOv3 backbone + Mask2Former-style head (deformable-attention pixel decoder, query decoder,
mask classification), 150 ADE20K classes.

Reference: offload/server/model/dinov3_segmentor_m2f.py (load :131, correct :1215, head :2715).
The backbone runs on the same approximate / correct engine as the other DINOv3 executors; the head
is models/m2f.py (see its docstring for the differences from the reference head). Random-init
head weights unless `m2f_head_weights_path` names an M2FHead state dict.
"""
from __future__ import annotations

from typing import Any, Dict

import numpy as np
import torch
import torch.nn.functional as F

from ...models.m2f import M2FHead, M2FHeadGPU
from ...ops import kernels as K
from .base import ModelExecutor
from .dinov3_common import DINOv3BackboneMixin


class DINOv3SegmentorM2FExecutor(DINOv3BackboneMixin, ModelExecutor):
    default_arch = "vit7b16"

    def __init__(self, device):
        super().__init__(device)
        self._init_backbone_state()
        self.head = None
        self.head_gpu = None

    def load_model(self, model_name: str, config: Any):
        profile = config.get_input_profile_config()
        self.load_backbone(model_name, config)
        C = int(profile.get("num_classes", 150))
        head = M2FHead(self.cfg.embed_dim, num_classes=C, enc_layers=int(profile.get("m2f_enc_layers", 6)),
                       dec_layers=int(profile.get("m2f_dec_layers", 9)), queries=int(profile.get("m2f_queries", 100)))
        path = self.weights_path(profile, "m2f_head_weights_path")
        if path is not None:
            head.load_state_dict(torch.load(path, map_location="cpu", weights_only=True), strict=True)
        else:
            head.init_weights(int(profile.get("seed", 0)))
        self.head = head.eval().to(self.device)
        if self.device.type == "cuda":
            self.head_gpu = M2FHeadGPU(self.head, self.device)
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
        C = self.head.num_classes
        if self.engine is not None:
            sess = context["session"]
            gh, gw = sess.grid_hw
            feat = self.engine.patch_features(sess)
            sem = self.head_gpu.logits(feat, B, gh, gw).permute(0, 2, 3, 1).contiguous()
            out = context.get("labels")
            if out is None or tuple(out.shape) != (B, H, W):
                out = torch.empty(B, H, W, dtype=torch.uint8, device=self.device)
            K.upsample_argmax(sem, C, H, W, out)
            context["labels"] = out
        else:
            gh, gw = context["grid_hw"]
            with torch.no_grad():
                xn = self.backbone.final_norm(context["x"])[:, self.cfg.n_prefix:]
                sem = self.head(xn, gh, gw)
                sem = F.interpolate(sem, size=(H, W), mode="bilinear", align_corners=False)
            context["labels"] = sem.argmax(1).to(torch.uint8)
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
