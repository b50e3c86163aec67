"""SAM 3-shaped executor: windowed-attention ViT tower on the approximate / correct engine.

Reference: offload/server/model/sam3_executor.py:41-190 (approx / correct on the vision tower,
stock model downstream). The tower is models/sam3.py (random init of the facebook/sam3 vision
geometry; no checkpoints offline). Token selection for the correction pass ranks tokens by how far
their input embedding moved between the approximate and the current canvas (the tower has no class
token for an attention score). Downstream of the tower, input profile key `sam3_head` selects:
"stock" -- as in the reference, the stock `transformers` Sam3Model (FPN neck, text and box-prompt
encoders, DETR encoder / decoder, mask decoder) fed with the tower features through
`vision_embeds`, prompted by the request's `input_boxes` (default one whole-image box) and text ids
(default the empty prompt); or "linear" (default) -- a linear per-patch segmentation
(BatchNorm-folded 1x1 head with fused upsample + argmax) on the raster-ordered tower features.
"""
from __future__ import annotations

from typing import Any, Dict

import numpy as np
import torch

from ...common.protocol import normalize_appcorr_kwargs
from ...models.engine import ViTEngine
from ...models.heads import LinearSegHead, SegHeadGPU
from ...models.sam3 import SAM3_PRESETS, SAM3Tower, build_stock_head, sam3_engine_weights, stock_head_forward
from ...ops import kernels as K
from .base import ModelExecutor
from .dinov3_common import DINOv3BackboneMixin


class Sam3Executor(ModelExecutor):
    def __init__(self, device):
        super().__init__(device)
        self.engine = None
        self.stock = None
        self._sessions: Dict = {}

    def load_model(self, model_name: str, config: Any):
        if self.device.type != "cuda":
            raise RuntimeError("the SAM 3 executor runs on the sm_100a engine (CUDA device required)")
        profile = config.get_input_profile_config()
        self.cfg = SAM3_PRESETS[str(profile.get("sam3_arch", "sam3_vitl14"))]
        seed = int(profile.get("seed", 0))
        tower = SAM3Tower(self.cfg).init_weights(seed).to(self.device)
        self.engine = ViTEngine(sam3_engine_weights(tower, self.device), self.device,
                                DINOv3BackboneMixin.engine_precision(config))
        del tower
        self.head_kind = str(profile.get("sam3_head", "linear"))
        if self.head_kind not in ("linear", "stock"):
            raise ValueError(f"sam3_head must be 'linear' or 'stock', got {self.head_kind!r}")
        head = LinearSegHead(self.cfg.embed_dim, int(profile.get("num_classes", 150)))
        head.random_init(seed)
        self.head_gpu = SegHeadGPU(head, self.device)
        self.num_classes = head.num_classes
        self.stock = build_stock_head(self.cfg, seed, self.device, torch.bfloat16) if self.head_kind == "stock" else None
        self.model = self.engine

    def preprocess(self, batch_data, task, context, config):
        canvas = DINOv3BackboneMixin.decode_inputs(self, batch_data, context)
        unit = self.cfg.patch_size * self.cfg.window_size
        B, H, W, _ = canvas.shape
        h, w = H // unit * unit, W // unit * unit
        context["canvas"] = canvas[:, (H - h) // 2:(H - h) // 2 + h, (W - w) // 2:(W - w) // 2 + w].contiguous()

    def prepare_tokens(self, task, context, config):
        canvas = context["canvas"]
        B, H, W, _ = canvas.shape
        key = (B, H, W)
        sess = self._sessions.get(key)
        if sess is None:
            sess = self.engine.new_session(B, H, W)
            self._sessions = {key: sess}
        self.engine.prepare_tokens(sess, canvas)
        context["session"] = sess
        return {}

    def approx_forward(self, params, context, config):
        sess = context["session"]
        self.engine.approx(sess, 0, self.cfg.depth, "none")
        prev = sess.extra.get("x_in_prev")
        if prev is None:
            prev = sess.extra["x_in_prev"] = torch.empty_like(sess.x_in)
        prev.copy_(sess.x_in)
        return {"precision": self.engine.precision["approx"]}

    def correct_forward(self, params, context, config):
        sess = context["session"]
        opts = normalize_appcorr_kwargs(config.appcorr_kwargs, config.transmission_kwargs)
        B, N = sess.B, sess.N
        score = sess.extra.get("score")
        if score is None:
            score = sess.extra["score"] = torch.empty(B, N, device=self.device)
            sess.extra["pre"] = torch.zeros(B, 0, device=self.device, dtype=torch.int32)
            sess.extra["cand"] = torch.arange(N, device=self.device, dtype=torch.int32).repeat(B, 1).contiguous()
        K.row_sqdist(sess.x_in, sess.extra["x_in_prev"], score.view(-1))
        self.engine.correct(sess, 0, self.cfg.depth, sess.extra["pre"], sess.extra["cand"], opts, server=score)
        return {}

    def features(self, context) -> torch.Tensor:
        """Final-normed tower features in raster order [B*gh*gw, D]."""
        sess = context["session"]
        normed = self.engine.normed_tokens(sess)
        inv = sess.extra.get("raster_rows")
        if inv is None:
            order = sess.extra["order"].long()
            r = torch.empty_like(order)
            r[order] = torch.arange(order.numel(), device=order.device)
            inv = (torch.arange(sess.B, device=order.device)[:, None] * sess.N + r[None]).reshape(-1)
            inv = sess.extra["raster_rows"] = inv.to(torch.int32).contiguous()
        out = torch.empty_like(normed)
        K.gather_rows(normed, inv, out)
        return out

    def head_inference(self, task, context, config) -> Dict[str, Any]:
        sess = context["session"]
        canvas = context["canvas"]
        B, H, W, _ = canvas.shape
        feat = self.features(context)
        context["vision_embeds"] = feat.view(B, sess.grid_hw[0], sess.grid_hw[1], -1)
        if self.stock is not None:
            out = stock_head_forward(self.stock, context["vision_embeds"], context.get("input_boxes"),
                                     context.get("input_ids"))
            context["output"] = out
            return {"num_masks": int(out.pred_masks.shape[1])}
        context["labels"] = self.head_gpu.labels(feat, B, sess.grid_hw[0], sess.grid_hw[1], H, W)
        return {}

    def full_inference(self, task, context, config):
        self.engine.approx(context["session"], 0, self.cfg.depth, "none")
        self.head_inference(task, context, config)

    def get_final_results(self, task, context, config) -> Dict[int, Any]:
        out = context.get("output") if self.stock is not None else None
        if out is not None:  # per image: the best-scoring query's mask, box and score
            return stock_results(out)
        labels = context.get("labels")
        if labels is None:
            return {}
        host = labels.cpu().numpy()
        return {i: {"mask": np.ascontiguousarray(host[i])} for i in range(host.shape[0])}

    def cache_stats(self, context) -> Dict[str, Any]:
        sess = context.get("session")
        if sess is None:
            return {"total": 0, "breakdown": {}}
        kv = (sess.kc.numel() + sess.vc.numel()) * 2
        inc = sess.bos.numel() * 2
        return {"total": kv + inc, "breakdown": {"kv": kv, "blocks_out_sum": inc}}


def stock_results(out) -> Dict[int, Any]:
    """Per image of a stock Sam3Model output: the highest-scoring query's binary mask (logit > 0,
    at the mask decoder's resolution), its normalised (cx, cy, w, h) box and its sigmoid score."""
    best = out.pred_logits.float().argmax(1)
    res = {}
    for i in range(best.shape[0]):
        q = int(best[i])
        res[i] = {"mask": np.ascontiguousarray((out.pred_masks[i, q] > 0).cpu().numpy().astype(np.uint8)),
                  "box": out.pred_boxes[i, q].float().cpu().tolist(),
                  "score": float(out.pred_logits[i, q].float().sigmoid())}
    return res
