"""DINOv3 backbone + DETR-style detection decoder
(reference offload/server/model/dinov3_detector.py:46-1714, PlainDETR head).

The backbone runs the approximate / correct passes like the other DINOv3 executors; the head
projects the final-normed patch tokens to the decoder width and runs the decoder
(appcorr_b200/models/detr.py) on the GPU kernels. Results per image: the top-100
(score, label, box[cx, cy, w, h] normalised to the image) detections.
Input-profile keys: backbone_arch (default vitl16), num_queries (300), num_classes (80),
decoder_layers (6), decoder_dim (256), decoder_heads (4).
"""
from __future__ import annotations

from typing import Any, Dict

import numpy as np
import torch

from ...models.detr import DetrDecoder, DetrDecoderGPU, postprocess
from .base import ModelExecutor
from .dinov3_common import DINOv3BackboneMixin


class DINOv3DetectorExecutor(DINOv3BackboneMixin, ModelExecutor):
    default_arch = "vitl16"

    def __init__(self, device):
        super().__init__(device)
        self._init_backbone_state()
        self.decoder = None
        self.decoder_gpu = None

    def load_model(self, model_name: str, config: Any):
        prof = config.get_input_profile_config()
        self.load_backbone(model_name, config)
        torch.manual_seed(int(prof.get("seed", 0)))
        self.decoder = DetrDecoder(self.cfg.embed_dim, d_model=int(prof.get("decoder_dim", 256)),
                                   heads=int(prof.get("decoder_heads", 4)), layers=int(prof.get("decoder_layers", 6)),
                                   num_queries=int(prof.get("num_queries", 300)),
                                   num_classes=int(prof.get("num_classes", 80))).eval()
        path = self.weights_path(prof, "detector_head_weights_path")
        if path is not None:
            self.decoder.load_state_dict(torch.load(path, map_location="cpu", weights_only=True), strict=True)
        if self.device.type == "cuda":
            self.decoder_gpu = DetrDecoderGPU(self.decoder, self.device)
        self.model = self.engine or self.backbone

    def preprocess(self, batch_data, task, context, config):
        self.decode_inputs(batch_data, context)

    def prepare_tokens(self, task, context, config):
        self.backbone_prepare_tokens(context)
        return {}

    def approx_forward(self, params, context, config):
        if params.get("global_only"):
            return {}
        return self.backbone_approx(params, context, config)

    def correct_forward(self, params, context, config):
        return self.backbone_correct(params, context, config)

    def head_inference(self, task, context, config) -> Dict[str, Any]:
        if self.engine is not None:
            sess = context["session"]
            feat = self.engine.patch_features(sess)
            out = self.decoder_gpu.forward(feat, sess.B, sess.grid_hw)
        else:
            with torch.no_grad():
                xn = self.backbone.final_norm(context["x"])[:, self.cfg.n_prefix:]
                out = self.decoder(xn, context["grid_hw"])
        context["detections"] = postprocess(out)
        return {}

    def full_inference(self, task, context, config):
        self.backbone_full(context, config)
        self.head_inference(task, context, config)

    def get_final_results(self, task, context, config) -> Dict[int, Any]:
        det = context.get("detections")
        if det is None:
            return {}
        scores, labels, boxes = (t.cpu().numpy() for t in det)
        active = context.get("active_indices", list(range(scores.shape[0])))
        return {int(i): {"scores": scores[i], "labels": labels[i].astype(np.int32), "boxes": boxes[i]}
                for i in active if i < scores.shape[0]}

    def cache_stats(self, context):
        return self.backbone_cache_stats(context)
