"""DINOv3 backbone + DETR-style detection decoder, with the detector's window wrapper
(reference offload/server/model/dinov3_detector.py:46-1714, PlainDETR head;
appcorr/models/dinov3/eval/detection/models/windows.py:16-80).

Sources. With `detector_windows` = n > 1 (input profile, default 3) the image is split into an
n x n grid of windows whose sides are multiples of the patch size (the last row / column takes the
remainder, windows.py:44-50), and a global source is the whole image resized to the size of the
top-left window. Every source runs the backbone's approximate / correct passes in its own engine
session (batch = the request's images). The head tiles the window features back into the full
token map, resizes the global source's features to that map, concatenates them channel-wise
[global | windows] (windows.py:69-74) and runs the decoder on 2*D channels. n <= 1 runs the whole
image as one source (D channels).

Instructions (offload/policies/scheduling: COCOWindowInterleaved and the global-source modes):
  APPROX_FORWARD  {"layers", "global_only" / "source_kind": "global" | "local"}: the global source,
                  the windows, or (no kind) every source
  CORRECT_FORWARD {"layers", "group_id"}: under a COCO window transmission (one correction group
                  per window, coco_window_trigger.py) group g in 1..n*n corrects window g-1 only;
                  otherwise every source is corrected with all its tokens as candidates.
Results per image: the top-100 (score, label, box[cx, cy, w, h] normalised to the image)
detections. Input-profile keys: backbone_arch (default vitl16), detector_windows (3),
num_queries (300), num_classes (80), decoder_layers (6), decoder_dim (256), decoder_heads (4).
"""
from __future__ import annotations

import math
from typing import Any, Dict, List, Tuple

import numpy as np
import torch
import torch.nn.functional as F

from ...models.detr import DetrDecoder, DetrDecoderGPU, postprocess
from .base import ModelExecutor
from .dinov3_common import DINOv3BackboneMixin


def window_layout(H: int, W: int, n: int, patch: int) -> Tuple[List[int], List[int], int, int]:
    """Window heights / widths of an n x n split (multiples of the patch, remainder last) and the
    top-left window size (windows.py:44-50)."""
    wh = math.ceil((H // n) / patch) * patch
    ww = math.ceil((W // n) / patch) * patch
    hs = [wh] * (n - 1) + [H - wh * (n - 1)]
    ws = [ww] * (n - 1) + [W - ww * (n - 1)]
    return hs, ws, wh, ww


class DINOv3DetectorExecutor(DINOv3BackboneMixin, ModelExecutor):
    default_arch = "vitl16"

    def __init__(self, device):
        super().__init__(device)
        self._init_backbone_state()
        self.decoder = None
        self.decoder_gpu = None
        self.n_windows = 3
        self._src_sessions: Dict[Tuple, Any] = {}

    def load_model(self, model_name: str, config: Any):
        prof = config.get_input_profile_config()
        self.load_backbone(model_name, config)
        self.n_windows = int(prof.get("detector_windows", 3))
        self._src_sessions.clear()
        torch.manual_seed(int(prof.get("seed", 0)))
        in_dim = self.cfg.embed_dim * (2 if self.n_windows > 1 else 1)
        self.decoder = DetrDecoder(in_dim, d_model=int(prof.get("decoder_dim", 256)),
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

    # ------------------------------------------------------------------ sources
    def _sources(self, canvas: torch.Tensor) -> List[Dict[str, Any]]:
        """Window crops (row-major) then the global source, each {"canvas": uint8 [B, h, w, 3]}."""
        B, H, W, _ = canvas.shape
        n, p = self.n_windows, self.cfg.patch_size
        if n <= 1:
            return [{"canvas": canvas, "kind": "whole"}]
        hs, ws, wh, ww = window_layout(H, W, n, p)
        out = []
        y = 0
        for ih in range(n):
            x = 0
            for iw in range(n):
                out.append({"canvas": canvas[:, y:y + hs[ih], x:x + ws[iw]].contiguous(), "kind": "window",
                            "pos": (ih, iw)})
                x += ws[iw]
            y += hs[ih]
        g = F.interpolate(canvas.permute(0, 3, 1, 2).float(), size=(wh, ww), mode="bilinear", align_corners=False,
                          antialias=True)
        out.append({"canvas": g.round().clamp(0, 255).to(torch.uint8).permute(0, 2, 3, 1).contiguous(),
                    "kind": "global"})
        return out

    def prepare_tokens(self, task, context, config):
        canvas = context["canvas"]
        srcs = context.get("det_sources")
        new = self._sources(canvas)
        if srcs is None or len(srcs) != len(new):
            srcs = context["det_sources"] = new
        else:
            for s, ns in zip(srcs, new):
                s["canvas"] = ns["canvas"]
        for i, s in enumerate(srcs):
            if self.engine is not None:
                B, h, w, _ = s["canvas"].shape
                key = (i, B, h, w)
                sess = self._src_sessions.get(key)
                if sess is None:
                    sess = self._src_sessions[key] = self.engine.new_session(B, h, w)
                self.engine.prepare_tokens(sess, s["canvas"])
                s["session"] = sess
            else:
                self.backbone_prepare_tokens(s)
        return {}

    def _selected(self, context, kind):
        srcs = context["det_sources"]
        if kind == "global":
            return [s for s in srcs if s["kind"] in ("global", "whole")]
        if kind == "local":
            return [s for s in srcs if s["kind"] in ("window", "whole")]
        return srcs

    def approx_forward(self, params, context, config):
        kind = "global" if params.get("global_only") else params.get("source_kind")
        out = {}
        for s in self._selected(context, kind):
            out = self.backbone_approx(params, s, config)
        return out

    def _single_window_group(self, config, group_id: int) -> bool:
        n2 = self.n_windows * self.n_windows
        tx = getattr(config, "transmission_policy_name", "") or ""
        return self.n_windows > 1 and 1 <= group_id <= n2 and tx.startswith("COCOWindow")

    def correct_forward(self, params, context, config):
        g = int(params.get("group_id", 0))
        p = dict(params)
        p["group_id"] = 0  # every token of a corrected source is a candidate
        srcs = context["det_sources"]
        if self._single_window_group(config, g):
            self.backbone_correct(p, srcs[g - 1], config)
            return {}
        for s in srcs:
            self.backbone_correct(p, s, config)
        return {}

    # ------------------------------------------------------------------ head
    def _features(self, s) -> Tuple[torch.Tensor, Tuple[int, int]]:
        """Final-normed patch tokens of one source as [B, gh, gw, D] and its grid."""
        B, h, w, _ = s["canvas"].shape
        gh, gw = h // self.cfg.patch_size, w // self.cfg.patch_size
        if self.engine is not None:
            f = self.engine.patch_features(s["session"])
        else:
            with torch.no_grad():
                f = self.backbone.final_norm(s["x"])[:, self.cfg.n_prefix:]
        return f.reshape(B, gh, gw, -1), (gh, gw)

    def memory(self, context) -> Tuple[torch.Tensor, Tuple[int, int]]:
        """Decoder memory [B, Ht*Wt, C] ([global | windows] channels with windows) and its grid."""
        srcs = context["det_sources"]
        if srcs[0]["kind"] == "whole":
            f, hw = self._features(srcs[0])
            return f.reshape(f.shape[0], -1, f.shape[-1]), hw
        n = self.n_windows
        rows = []
        for ih in range(n):
            rows.append(torch.cat([self._features(srcs[ih * n + iw])[0] for iw in range(n)], dim=2))
        win = torch.cat(rows, dim=1)                                   # [B, Ht, Wt, D]
        B, Ht, Wt, D = win.shape
        glob, _ = self._features(srcs[-1])
        glob = F.interpolate(glob.permute(0, 3, 1, 2).float(), size=(Ht, Wt), mode="bilinear",
                             align_corners=False).permute(0, 2, 3, 1).to(win.dtype)
        mem = torch.cat([glob, win], dim=-1)
        return mem.reshape(B, Ht * Wt, 2 * D), (Ht, Wt)

    def head_inference(self, task, context, config) -> Dict[str, Any]:
        mem, hw = self.memory(context)
        B = mem.shape[0]
        if self.decoder_gpu is not None and self.engine is not None:
            out = self.decoder_gpu.forward(mem.reshape(B * hw[0] * hw[1], -1).contiguous(), B, hw)
        else:
            with torch.no_grad():
                out = self.decoder(mem.float(), hw)
        context["detections"] = postprocess(out)
        return {}

    def full_inference(self, task, context, config):
        if "det_sources" not in context or context["det_sources"][0]["canvas"].shape[0] != context["canvas"].shape[0]:
            context.pop("det_sources", None)
        self.prepare_tokens(task, context, config)
        for s in context["det_sources"]:
            self.backbone_approx({"layers": (0, self.cfg.depth)}, s, config)
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
        tot = {"total": 0, "breakdown": {}}
        for s in context.get("det_sources", []):
            st = self.backbone_cache_stats(s)
            tot["total"] += st["total"]
            for k, v in st["breakdown"].items():
                tot["breakdown"][k] = tot["breakdown"].get(k, 0) + v
        return tot
