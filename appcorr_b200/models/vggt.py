"""VGGT-style multi-view tower: per-frame ViT blocks, then an aggregator alternating frame
attention (inside one frame) and global attention (across all frames of the sequence), with a
DPT depth head on four aggregator layers and a camera-pose head.

Reference: offload/server/model/vggt_omega.py (full inference only in the reference too) and
appcorr/models/vggt_omega/models/aggregator.py:29-451 (24 patch-embed blocks, 24 frame/global
pairs, heads read aggregator blocks 4/11/17/23). Built on the windowed ViT engine: the S frames of
a sequence are stacked into one canvas of S x 1 frames, the window is one frame, so frame
attention is a batched attention over frames and the aggregator's global blocks attend over the
whole sequence; RoPE coordinates are in-frame everywhere. Differences by design: no camera /
register tokens (the pose head reads mean-pooled frame features), random init (no checkpoints).
"""
from __future__ import annotations

from dataclasses import dataclass
from typing import Dict, List, Tuple

import torch
from torch import nn

from .dinov3.vit import ViTConfig


@dataclass
class VGGTConfig:
    frame: int = 512          # frame side in pixels
    patch: int = 16
    dim: int = 1024
    heads: int = 16
    patch_blocks: int = 24
    agg_pairs: int = 24
    mlp_ratio: float = 4.0
    head_layers: Tuple[int, ...] = (4, 11, 17, 23)   # aggregator pairs the depth head reads
    dpt_features: int = 256

    def vit(self) -> ViTConfig:
        g = self.frame // self.patch
        depth = self.patch_blocks + 2 * self.agg_pairs
        glob = tuple(self.patch_blocks + 2 * i + 1 for i in range(self.agg_pairs))
        return ViTConfig(img_size=self.frame, patch_size=self.patch, embed_dim=self.dim, depth=depth,
                         num_heads=self.heads, ffn_ratio=self.mlp_ratio, qkv_bias=True, layerscale_init=1.0,
                         norm_layer="layernorm", ffn_layer="mlp", n_storage_tokens=0, cls_token=False,
                         pos_embed_rope_base=100.0, window_size=g, global_layers=glob, window_rope_everywhere=True)

    def tap_layers(self) -> List[int]:
        """Engine layer index after the global block of each head pair."""
        return [self.patch_blocks + 2 * i + 1 for i in self.head_layers]


VGGT_PRESETS: Dict[str, VGGTConfig] = {
    "vggt_omega_1b": VGGTConfig(),
    "vggt_tiny": VGGTConfig(frame=128, patch=16, dim=256, heads=4, patch_blocks=2, agg_pairs=4,
                            head_layers=(0, 1, 2, 3), dpt_features=64),
}


class PoseHead(nn.Module):
    """Mean-pooled frame features -> 9-D pose encoding (translation 3, quaternion 4, field of view 2)."""

    def __init__(self, dim: int):
        super().__init__()
        self.fc1, self.fc2 = nn.Linear(dim, dim), nn.Linear(dim, 9)

    def forward(self, pooled):
        return self.fc2(torch.nn.functional.gelu(self.fc1(pooled)))
