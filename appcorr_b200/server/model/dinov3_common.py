"""Shared DINOv3 backbone handling for the executors (classifier, linear-head segmentor, ...).

On a CUDA device every backbone instruction runs on the sm_100a engine
(appcorr_b200/models/engine.py) with the whole request batch in one session: one GEMM per
projection for all images, where the reference loops over sources one image at a time
(reference dinov3_segmentor_linhead.py:548-575). On the CPU the same instructions run on the fp32
oracle module (config: CPU serving over loopback).
"""
from __future__ import annotations

from typing import Any, Dict, Optional, Tuple

import numpy as np
import torch

from ...common.protocol import normalize_appcorr_kwargs
from ...models.dinov3 import build_vit, create_group_index
from ...models.dinov3.vit import PRESETS
from ...ops import kernels as K
from .base import ModelExecutor, PyramidBatch, to_device_uint8_images

_ARCH_BY_NAME = (("7b", "vit7b16"), ("vitl", "vitl16"), ("vitb", "vitb16"), ("vits", "vits16"))


def arch_for(model_name: str, profile: Dict[str, Any], default: str) -> str:
    arch = profile.get("backbone_arch")
    if arch:
        return arch
    low = model_name.lower()
    for key, preset in _ARCH_BY_NAME:
        if key in low:
            return preset
    return default


class DINOv3BackboneMixin:
    """Backbone state + the APPROX / CORRECT / PREPARE_TOKENS instruction implementations."""

    default_arch = "vit7b16"

    def _init_backbone_state(self) -> None:
        self.backbone = None       # nn.Module (CPU path, and source of weights)
        self.engine = None         # ViTEngine (GPU path)
        self.arch = None
        self._sessions: Dict[Tuple[int, int, int], Any] = {}
        self._group_cache: Dict[Tuple, Tuple[torch.Tensor, torch.Tensor]] = {}

    # ------------------------------------------------------------------ loading
    @staticmethod
    def engine_precision(config: Any) -> Dict[str, str]:
        """Config precision -> engine precision per pass. "auto" picks e4m3 for a pass whose GEMMs
        have at least `fp8_auto_min_rows` rows and bf16 below (dinov3_precision.py:479-488).
        "fp4" / "nvfp4" select the NVFP4 block-scaled GEMMs."""
        m = {"bf16": "bf16", "fp8": "fp8", "auto": "auto", "fp4": "nvfp4", "nvfp4": "nvfp4"}
        ap = m.get(str(getattr(config, "precision", "bf16")).lower(), "bf16")
        cp = m.get(str(getattr(config, "correct_precision", "bf16")).lower(), "bf16")
        return {"approx": ap, "correct": cp}

    def load_backbone(self, model_name: str, config: Any) -> None:
        profile = config.get_input_profile_config()
        self.arch = arch_for(model_name, profile, self.default_arch)
        path = self.weights_path(profile, "backbone_weights_path")
        seed = int(profile.get("seed", 0))
        self._sessions.clear()
        self._group_cache.clear()
        tp = int(getattr(config, "tp_size", 1) or 1)
        prec = self.engine_precision(config)
        self.sr_engine = None
        self._auto_min_rows = int(getattr(config, "fp8_auto_min_rows", 3072) or 3072)
        if self.device.type == "cuda" and hasattr(config, "lowres_sr_enabled") and config.lowres_sr_enabled():
            from ..sr import create_lowres_sr_engine

            self.sr_engine = create_lowres_sr_engine(config.get_lowres_sr_config(), self.device)
        if self.device.type == "cuda" and tp > 1:
            import torch.distributed as dist

            from ...models.engine import weights_from_module
            from ...parallel.comm import TPComm
            from ...parallel.tp import ViTEngineTP

            grp = getattr(self, "tp_group", None)  # set by the serving group after a re-form
            if not dist.is_initialized() or dist.get_world_size(grp) != tp:
                raise RuntimeError(f"tp_size={tp} needs a torch.distributed group of {tp} ranks, one per GPU")
            self.comm = TPComm(group=grp, device=self.device)
            if path is not None:
                m = build_vit(self.arch)
                m.load_state_dict(torch.load(path, map_location="cpu", mmap=True, weights_only=True), strict=True)
                self.engine = ViTEngineTP.from_full(weights_from_module(m.eval(), self.device), self.comm, prec)
            else:
                self.engine = ViTEngineTP.random_tp(PRESETS[self.arch], self.comm, seed=seed, precision=prec)
            self.cfg = self.engine.cfg
            self.engine.auto_min_rows = self._auto_min_rows
        elif self.device.type == "cuda":
            from ...models.engine import ViTEngine

            if path is not None:
                m = build_vit(self.arch)
                m.load_state_dict(torch.load(path, map_location="cpu", mmap=True, weights_only=True), strict=True)
                self.engine = ViTEngine.from_module(m.eval(), self.device, prec)
                self.backbone = None
            else:
                self.engine = ViTEngine.random(PRESETS[self.arch], self.device, seed=seed, precision=prec)
            self.cfg = self.engine.cfg
            self.engine.auto_min_rows = self._auto_min_rows
        else:
            m = build_vit(self.arch)
            if path is not None:
                m.load_state_dict(torch.load(path, map_location="cpu", mmap=True, weights_only=True), strict=True)
            else:
                m.init_weights(seed)
            self.backbone = m.eval().requires_grad_(False)
            self.cfg = m.cfg

    # ------------------------------------------------------------------ inputs
    def decode_inputs(self, batch_data: Any, context: Dict[str, Any]) -> torch.Tensor:
        """LOAD_INPUT: decoded images or a Laplacian PyramidBatch -> uint8 [B, H, W, 3] canvas."""
        dev = self.device
        if isinstance(batch_data, PyramidBatch):
            cur = to_device_uint8_images(batch_data.base, dev)
            steps = batch_data.residual_steps()
            sr = getattr(self, "sr_engine", None)
            if sr is not None and all(r is None for r in steps):
                # approximate pass with super-resolution: the base is upscaled by the network
                # instead of the pyramid's pyrUp chain (reference worker.py:586-614)
                B, h, w, _ = cur.shape
                f = 2 ** len(steps)
                context["canvas"] = sr.upscale(cur, (h * f, w * f))
                context["target_shapes"] = batch_data.target_shapes
                return context["canvas"]
            for i, r in enumerate(steps):
                B, h, w, _ = cur.shape
                if r is not None:
                    r = torch.from_numpy(np.ascontiguousarray(r)) if isinstance(r, np.ndarray) else r
                    if dev.type == "cuda" and not r.is_cuda and not r.is_pinned():
                        r = r.pin_memory()
                    r = r.to(dev, non_blocking=True)
                if dev.type == "cuda":
                    key = f"canvas_l{len(steps) - 1 - i}"
                    nxt = context.get(key)
                    if nxt is None or tuple(nxt.shape) != (B, 2 * h, 2 * w, 3):
                        nxt = torch.empty(B, 2 * h, 2 * w, 3, dtype=torch.uint8, device=dev)
                        context[key] = nxt
                    K.pyrup_add(cur, r, nxt)
                else:
                    from ...policies.transmission.pyramid import pyr_up

                    up = np.stack([pyr_up(b) for b in cur.numpy()]).astype(np.int32)
                    if r is not None:
                        up = up + r.numpy().astype(np.int32)
                    nxt = torch.from_numpy(np.clip(up, 0, 255).astype(np.uint8))
                cur = nxt
            canvas = cur
            context["target_shapes"] = batch_data.target_shapes
        else:
            canvas = to_device_uint8_images(batch_data, dev)
        context["canvas"] = canvas
        return canvas

    def _session(self, B: int, H: int, W: int):
        key = (B, H, W)
        s = self._sessions.get(key)
        if s is None:
            if len(self._sessions) >= 2:
                self._sessions.clear()
                torch.cuda.empty_cache()
            s = self.engine.new_session(B, H, W)
            self._sessions[key] = s
        return s

    # ------------------------------------------------------------------ instructions
    def backbone_prepare_tokens(self, context: Dict[str, Any]) -> None:
        canvas = context["canvas"]
        B, H, W, _ = canvas.shape
        if self.engine is not None:
            sess = self._session(B, H, W)
            self.engine.prepare_tokens(sess, canvas)
            context["session"] = sess
        else:
            mean = torch.tensor(K.IMAGENET_MEAN).view(1, 3, 1, 1)
            std = torch.tensor(K.IMAGENET_STD).view(1, 3, 1, 1)
            img = (canvas.permute(0, 3, 1, 2).float() / 255 - mean) / std
            with torch.no_grad():
                x, (gh, gw) = self.backbone.prepare_tokens_with_masks(img)
            context["x_in"] = x
            context["grid_hw"] = (gh, gw)
            context["rope"] = self.backbone.rope_embed(H=gh, W=gw)
            context.setdefault("cache", {})

    def backbone_approx(self, params: Dict[str, Any], context: Dict[str, Any], config: Any) -> Dict[str, Any]:
        start, end = params.get("layers", (0, self.cfg.depth))
        opts = normalize_appcorr_kwargs(config.appcorr_kwargs, config.transmission_kwargs)
        if self.engine is not None:
            sess, kind = context["session"], opts["server_pscore"]
            self.engine.run_graphed(sess, ("approx", start, end, kind), lambda: self.engine.approx(sess, start, end, kind))
        else:
            x = context["x_in"].clone() if start == 0 or "x" not in context else context["x"]
            with torch.no_grad():
                for l in range(start, end):
                    x, _ = self.backbone.blocks[l].approx(x, context["rope"], context["cache"], f"layer{l}",
                                                          server_pscore=opts["server_pscore"],
                                                          server_pscore_weight=opts["server_pscore_weight"])
            context["x"] = x
        context["approx_frontier"] = max(context.get("approx_frontier", 0), end)
        if self.engine is None:
            return {"precision": "fp32"}
        sess = context["session"]
        return {"precision": sess.extra.get("pass_precision", ("approx", self.engine.precision["approx"]))[1],
                "rows": int(sess.x.shape[0])}

    def group_candidates(self, B: int, grid_hw: Tuple[int, int], group_id: int, config: Any,
                         device) -> Tuple[torch.Tensor, torch.Tensor]:
        """int32 prefix tokens [B, n_prefix] and candidate patch tokens [B, P_g] of a group."""
        tx = config.transmission_kwargs or {}
        ng = max(int(tx.get("num_groups", 1)), 1)
        strategy = str(tx.get("grouping_strategy", "grid"))
        key = (B, grid_hw, group_id, ng, strategy, str(device))
        hit = self._group_cache.get(key)
        if hit is not None:
            return hit
        npre = self.cfg.n_prefix
        P = grid_hw[0] * grid_hw[1]
        if ng > 1 and 1 <= group_id <= ng and strategy in {"grid", "block_grid", "expansion"}:
            gidx = create_group_index(P, ng, strategy, token_hw=grid_hw)
            sel = torch.nonzero(gidx == group_id).flatten() + npre
        else:
            sel = torch.arange(P) + npre
        cand = sel.to(torch.int32).repeat(B, 1).contiguous().to(device)
        pre = torch.arange(npre, dtype=torch.int32).repeat(B, 1).contiguous().to(device)
        self._group_cache[key] = (pre, cand)
        return pre, cand

    def backbone_correct(self, params: Dict[str, Any], context: Dict[str, Any], config: Any) -> Dict[str, Any]:
        start, end = params.get("layers", (0, self.cfg.depth))
        group_id = int(params.get("group_id", 0))
        opts = normalize_appcorr_kwargs(config.appcorr_kwargs, config.transmission_kwargs)
        hint = context.get("mobile_pscore_hint")
        if self.engine is not None:
            sess = context["session"]
            pre, cand = self.group_candidates(sess.B, sess.grid_hw, group_id, config, self.device)
            mobile = None
            if hint is not None and opts["mobile_pscore_weight"] != 0.0:
                mobile = hint.to(self.device, torch.float32).gather(1, (cand - self.cfg.n_prefix).long()).contiguous()
            # replayed as one CUDA graph when every input is static: no per-request mobile score,
            # no random score, no threshold without a cap (that plan needs a host read)
            static = (mobile is None and opts.get("server_pscore") != "random" and
                      not (opts.get("token_keep_thres") is not None and not opts.get("token_keep_cap")))
            if static:
                key = ("correct", start, end, pre.data_ptr(), cand.data_ptr(), tuple(pre.shape), tuple(cand.shape),
                       repr(sorted(opts.items())))
                self.engine.run_graphed(sess, key, lambda: self.engine.correct(sess, start, end, pre, cand, opts))
            else:
                self.engine.correct(sess, start, end, pre, cand, opts, mobile=mobile)
        else:
            x = context["x_in"].clone() if start == 0 or "x" not in context else context["x"]
            B = x.shape[0]
            pre, cand = self.group_candidates(B, context["grid_hw"], group_id, config, "cpu")
            dind = torch.cat([pre, cand], 1).long()
            with torch.no_grad():
                for l in range(start, end):
                    x, _ = self.backbone.blocks[l].correct(x, dind, context["rope"], context["cache"], f"layer{l}",
                                                           mobile_pscore_hint=hint, **opts)
            context["x"] = x
        return {}

    def backbone_full(self, context: Dict[str, Any], config: Any) -> None:
        """FULL_INFERENCE: a stock forward of every layer on the current canvas."""
        self.backbone_prepare_tokens(context)
        self.backbone_approx({"layers": (0, self.cfg.depth)}, context, config)

    def backbone_cache_stats(self, context: Dict[str, Any]) -> Dict[str, Any]:
        sess = context.get("session")
        if sess is None:
            cache = context.get("cache", {})
            tot = {}
            for k, v in cache.items():
                if isinstance(v, torch.Tensor):
                    fam = k.rsplit("_", 1)[-1]
                    tot[fam] = tot.get(fam, 0) + v.numel() * v.element_size()
            return {"total": sum(tot.values()), "breakdown": tot}
        br = {"kv": sess.kc.numel() * 2 * 2, "blocks_out_sum": sess.bos.numel() * 2, "server_pscore": sess.pscore.numel() * 4}
        return {"total": sum(br.values()), "breakdown": br}
