"""Low-resolution super-resolution engine: upscales the pyramid base for the approximate pass
when `scheduler_kwargs.lowres_sr` is set.

Reference: offload/server/sr/realesrgan.py:102-304 (RRDBNet x4plus: 23 RRDB blocks, 64 features,
growth 32; tiled forward) and its use in the worker's LOAD_INPUT (worker.py:586-614: super-resolve
the low-resolution base, resize to the original size). Here the network is models/conv.py
RRDBNet on the sm_100a convolution path; the result is resized to the target with the bilinear
NHWC kernel and rounded to uint8 on the device. Weights: `<weights_dir>/<model>.pth` in the
Real-ESRGAN key layout (`params_ema` / `params`), else random init.
"""
from __future__ import annotations

import os
import re
from typing import Any, Dict, Optional, Tuple

import torch

from ..models.conv import RRDBNet, RRDBNetGPU, resize

PRESETS = {"realesrgan_x4plus": dict(nf=64, nb=23, gc=32, scale=4),
           "realesrgan_x2plus": dict(nf=64, nb=23, gc=32, scale=2)}


def convert_realesrgan_state(sd: Dict[str, torch.Tensor]) -> Dict[str, torch.Tensor]:
    """Real-ESRGAN key names -> RRDBNet (models/conv.py) names."""
    sd = sd.get("params_ema", sd.get("params", sd))
    out = {}
    for k, v in sd.items():
        m = re.match(r"body\.(\d+)\.rdb(\d)\.conv(\d)\.(weight|bias)", k)
        if m:
            out[f"body.{m[1]}.rdbs.{int(m[2]) - 1}.convs.{int(m[3]) - 1}.{m[4]}"] = v
            continue
        m = re.match(r"conv_up(\d)\.(weight|bias)", k)
        if m:
            out[f"conv_up.{int(m[1]) - 1}.{m[2]}"] = v
            continue
        out[k] = v
    return out


class LowResSR:
    def __init__(self, cfg: Dict[str, Any], device):
        name = str(cfg.get("model", "realesrgan_x4plus"))
        p = PRESETS.get(name, PRESETS["realesrgan_x4plus"])
        self.scale = p["scale"]
        net = RRDBNet(**p)
        path = os.path.join(os.path.expanduser(str(cfg.get("weights_dir") or "")), f"{name}.pth")
        if os.path.exists(path):
            net.load_state_dict(convert_realesrgan_state(torch.load(path, map_location="cpu", weights_only=True)))
        else:
            net.init_weights(int(cfg.get("seed", 0)))
        self.net = net.to(device).eval()
        self.gpu = RRDBNetGPU(self.net, device)

    def upscale(self, base_u8: torch.Tensor, target_hw: Optional[Tuple[int, int]] = None) -> torch.Tensor:
        """uint8 [B, h, w, 3] on the device -> uint8 [B, H, W, 3] (H, W = target or scale * (h, w))."""
        up = self.gpu.forward(base_u8)
        if target_hw is None or tuple(target_hw) == tuple(up.shape[1:3]):
            return up
        # resize through an 8-channel bf16 map (the NHWC kernel works on 8-channel vectors)
        x = torch.zeros(*up.shape[:3], 8, device=up.device, dtype=torch.bfloat16)
        x[..., :3] = up.to(torch.bfloat16)
        y = resize(x, int(target_hw[0]), int(target_hw[1]), False)
        return y[..., :3].float().clamp(0, 255).round().to(torch.uint8).contiguous()


def create_lowres_sr_engine(cfg: Dict[str, Any], device) -> LowResSR:
    return LowResSR(cfg, device)
