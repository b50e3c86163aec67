"""CLIP zero-shot classifier: CLIP image tower on the approximate / correct ViT engine, cosine
scores against class text embeddings.

Reference: offload/server/model/openclip_executor.py:40-262. Profile keys: `clip_arch`
(models/clip.py CLIP_PRESETS, default clip_vitl14), `clip_text_embeds_path` (a [C, E] tensor of
class text embeddings; random unit vectors otherwise), `num_classes`, `seed`. Results: top-5
(class, probability) per image, as the classifier executor returns them.
"""
from __future__ import annotations

from typing import Any, Dict

import torch
import torch.nn.functional as F

from ...models.clip import CLIP_PRESETS, CLIPVision, clip_engine_weights
from ...models.engine import ViTEngine
from ...ops import kernels as K
from .base import ModelExecutor
from .dinov3_common import DINOv3BackboneMixin


class OpenCLIPExecutor(DINOv3BackboneMixin, ModelExecutor):
    def __init__(self, device):
        super().__init__(device)
        self._init_backbone_state()

    def load_model(self, model_name: str, config: Any):
        if self.device.type != "cuda":
            raise RuntimeError("the CLIP executor runs on the sm_100a engine (CUDA device required)")
        profile = config.get_input_profile_config()
        arch = str(profile.get("clip_arch", "clip_vitl14"))
        c = CLIP_PRESETS[arch]
        seed = int(profile.get("seed", 0))
        tower = CLIPVision(c).init_weights(seed).to(self.device)
        self.engine = ViTEngine(clip_engine_weights(tower, self.device), self.device,
                                self.engine_precision(config))
        self.proj_t = tower.proj.detach().t().contiguous().to(torch.bfloat16)        # [E, D]
        del tower
        self.cfg = self.engine.cfg
        path = self.weights_path(profile, "clip_text_embeds_path")
        if path is not None:
            text = torch.load(path, map_location="cpu", weights_only=True).float()
        else:
            g = torch.Generator().manual_seed(seed + 7)
            text = torch.randn(int(profile.get("num_classes", 1000)), c.embed_dim, generator=g)
        self.text = F.normalize(text, dim=-1).to(self.device)
        self.model = self.engine

    def preprocess(self, batch_data, task, context, config):
        self.decode_inputs(batch_data, context)

    def prepare_tokens(self, task, context, config):
        self.backbone_prepare_tokens(context)
        return {}

    def approx_forward(self, params, context, config):
        return self.backbone_approx(params, context, config)

    def correct_forward(self, params, context, config):
        return self.backbone_correct(params, context, config)

    def image_embeddings(self, context) -> torch.Tensor:
        sess = context["session"]
        cls_rows = (torch.arange(sess.B, device=self.device, dtype=torch.int32) * sess.N).contiguous()
        xn = torch.empty(sess.B, self.cfg.embed_dim, device=self.device, dtype=torch.bfloat16)
        K.layernorm(sess.x, self.engine.w.norm_w, self.engine.w.norm_b, self.cfg.norm_eps, xn, rows=cls_rows)
        E = self.proj_t.shape[0]
        emb = torch.empty(sess.B, E, device=self.device, dtype=torch.float32)
        K.gemm(xn, self.proj_t, emb, epi=K.EPI_F32)
        return F.normalize(emb, dim=-1)

    def head_inference(self, task, context, config) -> Dict[str, Any]:
        context["logits"] = 100.0 * self.image_embeddings(context) @ self.text.t()
        return {}

    def full_inference(self, task, context, config):
        self.backbone_full(context, config)
        self.head_inference(task, context, config)

    def get_final_results(self, task, context, config) -> Dict[int, Any]:
        lg = context.get("logits")
        if lg is None:
            return {}
        p = lg.float().softmax(-1)
        top = p.topk(min(5, p.shape[-1]), -1)
        idx, val = top.indices.cpu().tolist(), top.values.cpu().tolist()
        return {i: {"topk": [(int(c), float(v)) for c, v in zip(idx[i], val[i])]} for i in range(len(idx))}

    def cache_stats(self, context):
        return self.backbone_cache_stats(context)
