"""DINOv3 backbone + linear classifier (reference offload/server/model/dinov3_classifier.py:12-848).

Head: Linear(D * 2, 1000) on [normed CLS | mean of normed patch tokens] for ViT-7B
(hub/classifiers.py:35), Linear(D, 1000) on the normed CLS token for smaller presets unless
`use_avgpool` is set in the input profile. Results per image: top-5 class ids and their logits.
Early exit (DECIDE_EXIT): images whose top-1 softmax probability exceeds
scheduler_kwargs.threshold (metric "max_prob") or whose top1-top2 margin exceeds it ("margin")
leave the batch: their result is fixed and later instructions skip them.
"""
from __future__ import annotations

from typing import Any, Dict

import numpy as np
import torch

from ...models.heads import ClassifierHeadGPU, LinearClassifierHead
from ...ops import kernels as K
from .base import ModelExecutor
from .dinov3_common import DINOv3BackboneMixin


class DINOv3ClassifierExecutor(DINOv3BackboneMixin, ModelExecutor):
    default_arch = "vit7b16"

    def __init__(self, device):
        super().__init__(device)
        self._init_backbone_state()
        self.head = None
        self.head_gpu = None

    def load_model(self, model_name: str, config: Any):
        profile = config.get_input_profile_config()
        self.load_backbone(model_name, config)
        avg = bool(profile.get("use_avgpool", self.arch == "vit7b16"))
        self.head = LinearClassifierHead(self.cfg.embed_dim, int(profile.get("num_classes", 1000)), use_avgpool=avg)
        path = self.weights_path(profile, "classifier_head_weights_path")
        if path is not None:
            sd = torch.load(path, map_location="cpu", weights_only=True)
            self.head.linear.load_state_dict({k.split("linear.")[-1]: v for k, v in sd.items()}, strict=True)
        else:
            g = torch.Generator().manual_seed(int(profile.get("seed", 0)))
            with torch.no_grad():
                self.head.linear.weight.normal_(0, 0.02, generator=g)
                self.head.linear.bias.zero_()
        self.head.eval()
        if self.device.type == "cuda":
            self.head_gpu = ClassifierHeadGPU(self.head, self.device)
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

    def logits(self, context) -> torch.Tensor:
        if self.engine is not None:
            sess = context["session"]
            buf = self.engine.normed_tokens(sess)
            return self.head_gpu.logits(buf, sess.B, sess.N, self.cfg.n_prefix)
        with torch.no_grad():
            xn = self.backbone.final_norm(context["x"])
            npre = self.cfg.n_prefix
            return self.head(xn[:, 0], xn[:, npre:])

    def head_inference(self, task, context, config) -> Dict[str, Any]:
        context["logits"] = self.logits(context)
        return {}

    def full_inference(self, task, context, config):
        self.backbone_full(context, config)
        self.head_inference(task, context, config)

    def decide_exit(self, task, context, config) -> Dict[str, Any]:
        ee = config.get_early_exit_config()
        thr = float(ee.get("threshold", 1.0))
        metric = str(ee.get("metric", "max_prob"))
        probs = torch.softmax(context["logits"].float(), -1).cpu()
        top2 = probs.topk(2, -1).values
        score = top2[:, 0] - top2[:, 1] if metric == "margin" else top2[:, 0]
        active = context.get("active_indices", list(range(probs.shape[0])))
        keep, done = [], {}
        for orig in active:  # the session keeps every image; rows are indexed by original position
            if orig < score.shape[0] and float(score[orig]) >= thr:
                done[orig] = self._format(context["logits"][orig])
            else:
                keep.append(orig)
        context.setdefault("final_results", {}).update(done)
        context["active_indices"] = keep
        return {"num_exits": len(done)}

    @staticmethod
    def _format(row: torch.Tensor) -> Dict[str, Any]:
        v, i = row.float().topk(5)
        return {"topk": i.cpu().tolist(), "logits": v.cpu().tolist()}

    def get_final_results(self, task, context, config) -> Dict[int, Any]:
        lg = context.get("logits")
        if lg is None:
            return {}
        active = context.get("active_indices", list(range(lg.shape[0])))
        top_v, top_i = lg.float().topk(5, -1)
        top_v, top_i = top_v.cpu().numpy(), top_i.cpu().numpy()
        return {int(orig): {"topk": top_i[orig].tolist(), "logits": top_v[orig].tolist()}
                for orig in active if orig < lg.shape[0]}

    def cache_stats(self, context):
        return self.backbone_cache_stats(context)
