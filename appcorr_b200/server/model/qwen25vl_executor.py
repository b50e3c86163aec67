"""Qwen2.5-VL executor: vision tower + causal LLM prefill in approximate / correct mode with a
paged K/V cache rewritten in place for the corrected tokens, then the first generated token.

Reference: offload/server/model/qwen25vl_executor.py:33-339 (preprocess :63-93, prepare_tokens
:128-138, approx_forward :148-172, correct_forward :174-250, head_inference :252-286). Differences
by design: the model is random-init with the configured shape (no checkpoints offline), the
prompt is `n_text` synthetic token ids around the image, the canvas is centre-cropped to a
multiple of 112 px (the reference processor resizes), and only the first token is produced (the
reference falls back to HF generate for the rest).

Rounds: the approximate round runs the whole vision tower on the approximate canvas (keeping
every block's K / V) and the LLM prefill. A correction round recomputes only the merge units
whose pixels changed most (token_keep_ratio of them, ranked by patch drift) through the tower
against the cached K / V of the others, then corrects the prompt text plus exactly those units'
image rows in the LLM (the reference corrects the merge units of the transmission group that
arrived, :174-250).
"""
from __future__ import annotations

from typing import Any, Dict

import torch

from ...common.protocol import normalize_appcorr_kwargs
from ...models.qwen25vl import PRESETS, Qwen25VL
from .base import ModelExecutor
from .dinov3_common import DINOv3BackboneMixin


class Qwen25VLExecutor(ModelExecutor):
    def __init__(self, device):
        super().__init__(device)
        self.engine = None
        self.cfg = None
        self._sessions: Dict = {}

    def load_model(self, model_name: str, config: Any):
        from ...models.qwen_engine import QwenVLEngine

        if self.device.type != "cuda":
            raise RuntimeError("the Qwen2.5-VL executor runs on the sm_100a engine (CUDA device required)")
        profile = config.get_input_profile_config()
        arch = str(profile.get("vlm_arch", "qwen25vl7b"))
        self.cfg = PRESETS[arch]
        seed = int(profile.get("seed", 0))
        self.n_before = int(profile.get("n_text_before", 16))
        self.n_after = int(profile.get("n_text", 128)) - self.n_before
        model = Qwen25VL.random_on(self.cfg, self.device, seed)
        prec = DINOv3BackboneMixin.engine_precision(config)["approx"]
        prec = "fp8" if prec == "nvfp4" else prec  # the LLM engine's low-precision path is e4m3
        tp = int(getattr(config, "tp_size", 1) or 1)
        if tp > 1:
            import torch.distributed as dist

            from ...parallel.comm import TPComm
            from ...parallel.qwen_tp import QwenVLEngineTP

            if not dist.is_initialized() or dist.get_world_size() != tp:
                raise RuntimeError(f"tp_size={tp} needs a torch.distributed group of {tp} ranks, one per GPU")
            self.engine = QwenVLEngineTP(model, TPComm(device=self.device), prec)
        else:
            self.engine = QwenVLEngine(model, self.device, prec)
        del model
        torch.cuda.empty_cache()
        g = torch.Generator().manual_seed(seed + 1)
        self.text_ids = torch.randint(0, self.cfg.vocab, (self.n_before + self.n_after,), generator=g).to(
            self.device, torch.int32)
        self.model = self.engine

    def _crop(self, canvas: torch.Tensor) -> torch.Tensor:
        unit = self.cfg.patch * self.cfg.window
        B, H, W, _ = canvas.shape
        h, w = H // unit * unit, W // unit * unit
        y, x = (H - h) // 2, (W - w) // 2
        return canvas[:1, y:y + h, x:x + w].contiguous()

    def preprocess(self, batch_data, task, context, config):
        canvas = DINOv3BackboneMixin.decode_inputs(self, batch_data, context)
        context["image"] = self._crop(canvas)

    def prepare_tokens(self, task, context, config):
        img = context["image"]
        H, W = img.shape[1:3]
        key = (H, W)
        sess = self._sessions.get(key)
        if sess is None:
            sess = self.engine.new_session(H, W, self.n_before, self.n_after)
            self._sessions = {key: sess}
            self.engine.embed_text(sess, self.text_ids)
        context["session"] = sess
        return {}

    def approx_forward(self, params, context, config):
        sess = context["session"]
        self.engine.vision(sess, context["image"])
        self.engine.approx(sess)
        return {"precision": "fp8" if self.engine.fp8 else "bf16"}

    def correct_forward(self, params, context, config):
        opts = normalize_appcorr_kwargs(config.appcorr_kwargs, config.transmission_kwargs)
        keep = float(opts.get("token_keep_ratio", 0.25))
        sess = context["session"]
        units = self.engine.vision_correct(sess, context["image"], keep)
        self.engine.correct(sess, keep, units=units)
        return {}

    def head_inference(self, task, context, config) -> Dict[str, Any]:
        context["token"] = self.engine.first_token(context["session"])
        return {}

    def full_inference(self, task, context, config):
        sess = context["session"]
        self.engine.vision(sess, context["image"])
        self.engine.approx(sess)
        self.head_inference(task, context, config)

    def get_final_results(self, task, context, config) -> Dict[int, Any]:
        tok = context.get("token")
        if tok is None:
            return {}
        return {0: {"first_token": int(tok.item())}}

    def cache_stats(self, context) -> Dict[str, Any]:
        sess = context.get("session")
        if sess is None:
            return {"total": 0, "breakdown": {}}
        t = sess.tensors
        kv = t["kc"].numel() * 2 + t["vc"].numel() * 2
        inc = t["bos"].numel() * 2
        return {"total": kv + inc, "breakdown": {"kv_pages": kv, "increment": inc}}
