"""VGGT-style multi-view executor: frames of one sequence -> per-frame depth and camera-pose
encodings, by full inference or by the approximate / correct walk over the 48-stage VGGT axis
(reference offload/server/model/vggt_omega.py:320-451, scheduled by VGGTInterleaved,
offload/policies/scheduling/vggt_interleaved.py:36-187). See models/vggt.py for the model.

Stage axis: stages 0..23 are the patch-embed blocks (engine layers 0..23), stages 24..47 the
aggregator frame/global pairs (engine layers 24 + 2i and 25 + 2i). APPROX_FORWARD {"layers":
(lo, hi)} walks stages [lo, hi) of the approximate pass from the running features; CORRECT_FORWARD
{"layers": (lo, hi)} recomputes, over stages [lo, hi), the tokens that this round's residual
patches carry (the arrived tokens; all tokens when the request carries no patch layout), keeping
`token_keep_ratio` of them ranked by how far their input embedding moved since the previous
round. K/V and increments of the corrected tokens are rewritten in the caches, so later rounds see
every earlier correction. Difference from the reference: this tower has no camera / register
tokens (the pose head reads mean-pooled frame features), so there is no attention-derived server
score to rank by; the embedding drift plays that role.

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
        if context.get("vggt_approx_done"):
            # a refinement round: keep the previous embeddings (the drift score) and the tokens
            # this round's patches carry
            prev = sess.extra.get("x_in_prev")
            if prev is None:
                prev = sess.extra["x_in_prev"] = torch.empty_like(sess.x_in)
            prev.copy_(sess.x_in)
            context["vggt_arrived"] = self._arrived_tokens(task, context, config, sess)
        self.engine.prepare_tokens(sess, canvas)
        context["session"] = sess
        return {}

    # ------------------------------------------------------------------ stage walk
    def _engine_layers(self, params) -> tuple:
        """48-stage range [lo, hi) -> engine layer range."""
        pe, total = self.vc.patch_blocks, self.vc.patch_blocks + self.vc.agg_pairs
        lo, hi = params.get("layers", (0, total))
        lo, hi = max(0, int(lo)), min(int(hi), total)

        def layer(s):
            return s if s <= pe else pe + 2 * (s - pe)

        return layer(lo), layer(max(hi, lo))

    def _arrived_tokens(self, task, context, config, sess) -> torch.Tensor:
        """int32 [1, n] canvas token indices covered by this round's residual patches (marked on
        each frame's transmission grid, then resampled to the token grid, as the reference does
        for frames whose transmission grid differs from the model's), or every token."""
        S = int(context["frames"].shape[0])
        g = self.vc.frame // self.vc.patch
        patches = [p for p in (getattr(task, "payload", None) or []) if getattr(p, "group_id", 0) > 0]
        if not patches or not getattr(config, "image_shape", None):
            return torch.arange(sess.N, device=self.device, dtype=torch.int32)[None].contiguous()
        Hi, Wi = int(config.image_shape[0]), int(config.image_shape[1])
        ph, pw = config.patch_size
        mask = np.zeros((S, g, g), dtype=bool)
        centre = (np.arange(g) + 0.5) / g
        for p in patches:
            f = int(p.image_idx)
            if not 0 <= f < S:
                continue
            sc = 2 ** int(p.res_level)
            cw = -(-Wi // (pw * sc))
            r, c = divmod(int(p.spatial_idx), cw)
            y0, y1 = r * ph * sc / Hi, (r + 1) * ph * sc / Hi
            x0, x1 = c * pw * sc / Wi, (c + 1) * pw * sc / Wi
            rows = (centre >= y0) & (centre < y1)
            cols = (centre >= x0) & (centre < x1)
            mask[f][np.ix_(rows, cols)] = True
        idx = np.nonzero(mask.reshape(-1))[0]   # frame-major, raster inside a frame = window order
        if idx.size == 0:
            idx = np.arange(sess.N)
        return torch.from_numpy(idx.astype(np.int32))[None].to(self.device).contiguous()

    def approx_forward(self, params, context, config):
        sess = context["session"]
        l0, l1 = self._engine_layers(params)
        if l1 > l0:
            self.engine.approx(sess, l0, l1, "none")
        context["vggt_approx_done"] = True
        return {"precision": self.engine.precision["approx"]}

    def correct_forward(self, params, context, config):
        if not context.get("vggt_approx_done"):
            raise RuntimeError("CORRECT_FORWARD before APPROX_FORWARD for VGGT")
        from ...common.protocol import normalize_appcorr_kwargs
        from ...ops import kernels as K

        sess = context["session"]
        l0, l1 = self._engine_layers(params)
        if l1 <= l0:
            return {}
        opts = normalize_appcorr_kwargs(config.appcorr_kwargs, config.transmission_kwargs)
        cand = context.get("vggt_arrived")
        if cand is None:
            cand = torch.arange(sess.N, device=self.device, dtype=torch.int32)[None].contiguous()
        score = sess.extra.get("drift")
        if score is None:
            score = sess.extra["drift"] = torch.zeros(1, sess.N, device=self.device)
        prev = sess.extra.get("x_in_prev")
        if prev is not None:
            K.row_sqdist(sess.x_in, prev, score.view(-1))
        pre = torch.zeros(1, 0, device=self.device, dtype=torch.int32)
        self.engine.correct(sess, l0, l1, pre, cand, opts, server=score)
        return {}

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
