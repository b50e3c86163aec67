"""DINOv3 backbone + Mask2Former segmentor (ViT adapter, deformable pixel decoder, masked-attention
decoder), 150 ADE20K classes, with sliding-window sources.

Reference: offload/server/model/dinov3_segmentor_m2f.py (load :131, prepare :952, approx :1137,
correct :1215, multi-source correction batching :1424, crops :2118, crop-cover group map :2138,
head :2715). The backbone runs on the approximate / correct engine with taps on the adapter's
four interaction layers (every quarter of the depth; 4, 11, 17, 23 for 24 blocks); the adapter
and head are models/mask2former.py (reference checkpoint layout, `segmentation_model.*`).

Sources: with `server_inference_mode` "slide" (the official ADE20K profile: 896 crops, stride
596) every image is cut into its sliding windows and the windows of all images form the engine
batch, so the approximate pass, the correction passes (whose token groups are taken per window)
and the head run once over all sources; the head's class maps are averaged back onto each image
where windows overlap. "whole" runs each image as one source. GPU engine only.
"""
from __future__ import annotations

from typing import Any, Dict, List

import numpy as np
import torch

from ...models.mask2former import DINOv3M2FSegmentor, Mask2FormerGPU, semantic_map, slide_windows
from ...ops import kernels as K
from .base import ModelExecutor
from .dinov3_common import DINOv3BackboneMixin


def interaction_layers(depth: int) -> List[int]:
    """The adapter's tap layers: the paper's [4, 11, 17, 23] for 24 blocks, else every quarter."""
    if depth == 24:
        return [4, 11, 17, 23]
    return [i * (depth // 4) - 1 for i in range(1, 5)]


class DINOv3SegmentorM2FExecutor(DINOv3BackboneMixin, ModelExecutor):
    default_arch = "vit7b16"

    def __init__(self, device):
        super().__init__(device)
        self._init_backbone_state()
        self.seg = None
        self.seg_gpu = None

    def load_model(self, model_name: str, config: Any):
        profile = config.get_input_profile_config()
        self.load_backbone(model_name, config)
        if self.engine is None:
            raise RuntimeError("the Mask2Former segmentor runs on the GPU engine")
        if getattr(self.engine, "world", 1) > 1:
            raise RuntimeError("the adapter's dense taps run on single-GPU engines (use data parallelism)")
        self.taps = interaction_layers(self.cfg.depth)
        self.engine.taps = tuple(self.taps)
        self.num_classes = int(profile.get("num_classes", 150))
        seg = DINOv3M2FSegmentor(self.cfg.embed_dim, num_classes=self.num_classes,
                                 hidden=int(profile.get("m2f_hidden_dim", 2048)), patch=self.cfg.patch_size,
                                 adapter_heads=int(profile.get("m2f_adapter_heads", 16)),
                                 enc_layers=int(profile.get("m2f_enc_layers", 6)),
                                 dec_layers=int(profile.get("m2f_dec_layers", 9)),
                                 queries=int(profile.get("m2f_queries", 100)))
        path = self.weights_path(profile, "segmentor_head_weights_path")
        if path is not None:  # the reference's head checkpoint: every non-backbone key must load
            sd = torch.load(path, map_location="cpu", weights_only=True)
            sd = sd.get("model", sd)
            sd = {k: v for k, v in sd.items() if ".backbone." not in k}
            seg.load_state_dict(sd, strict=True)
        else:
            seg.init_weights(int(profile.get("seed", 0)))
        self.seg = seg.eval().to(self.device)
        self.seg_gpu = Mask2FormerGPU(self.seg, self.device)
        self.slide = profile.get("server_inference_mode", "whole") == "slide"
        self.crop = int(profile.get("server_crop_size", 896))
        self.stride = int(profile.get("server_stride", 596))
        self.model = self.engine

    # ------------------------------------------------------------------ sources
    def _to_sources(self, context: Dict[str, Any]) -> None:
        canvas = context["canvas"]
        B, H, W, _ = canvas.shape
        crops = slide_windows(H, W, self.crop, self.stride) if self.slide else [(0, H, 0, W)]
        context["m2f_layout"] = (B, H, W, crops)
        if len(crops) == 1 and crops[0] == (0, H, 0, W):
            return
        ch, cw = crops[0][1] - crops[0][0], crops[0][3] - crops[0][2]
        src = context.get("m2f_sources")
        n = B * len(crops)
        if src is None or tuple(src.shape) != (n, ch, cw, 3):
            src = context["m2f_sources"] = torch.empty(n, ch, cw, 3, dtype=torch.uint8, device=canvas.device)
        for b in range(B):  # source index = image * windows + window
            for k, (y1, y2, x1, x2) in enumerate(crops):
                src[b * len(crops) + k].copy_(canvas[b, y1:y2, x1:x2])
        context["canvas"] = src

    def preprocess(self, batch_data, task, context, config):
        self.decode_inputs(batch_data, context)
        self._to_sources(context)

    def prepare_tokens(self, task, context, config):
        self.backbone_prepare_tokens(context)
        return {}

    def approx_forward(self, params, context, config):
        return self.backbone_approx(params, context, config)

    def correct_forward(self, params, context, config):
        return self.backbone_correct(params, context, config)

    # ------------------------------------------------------------------ head
    def head_inference(self, task, context, config) -> Dict[str, Any]:
        B, H, W, crops = context["m2f_layout"]
        src = context["canvas"]
        n, h, w, _ = src.shape
        sess = context["session"]
        taps = [self.engine.tap_features(sess, l) for l in self.taps]
        mean = torch.tensor(K.IMAGENET_MEAN, device=self.device)
        std = torch.tensor(K.IMAGENET_STD, device=self.device)
        img = ((src.float() / 255 - mean) / std).to(torch.bfloat16).contiguous()
        with torch.no_grad():
            pred = self.seg_gpu.forward(img, taps, n)
            sem = semantic_map(pred, (h, w))                                    # [n, C, h, w]
        C = sem.shape[1]
        if len(crops) == 1 and crops[0] == (0, H, 0, W):
            full = sem
        else:
            full = torch.zeros(B, C, H, W, device=self.device)
            cnt = torch.zeros(1, 1, H, W, device=self.device)
            for k, (y1, y2, x1, x2) in enumerate(crops):
                full[:, :, y1:y2, x1:x2] += sem[k::len(crops)]
                cnt[:, :, y1:y2, x1:x2] += 1
            full = full / cnt
        context["labels"] = full.argmax(1).to(torch.uint8)
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
