"""CLIP-style image tower (pre-LN ViT with a learned position embedding and a class token) for
zero-shot classification, run on the approximate / correct ViT engine.

Reference: offload/server/model/openclip_executor.py:40-262 and the OpenCLIP vision forks under
appcorr/models/openclip/vision (approx / correct of the CLIP vision blocks, same recurrences as the
DINOv3 block). The engine (models/engine.py) runs these blocks with LayerScale = 1, no RoPE and
the learned position embedding added to the patch tokens; the pooled output is
LN_post(CLS) @ proj, L2-normalised, and class scores are 100 * cosine against the class text
embeddings (`text_embeds` [C, E], an input: the text tower is not part of this build).
ViT-B/16 and ViT-L/14 use 64-wide heads; bigG/14 (head dim 104, reference
openclip_executor.py:40-262) runs with its heads zero-padded to 128 in the engine: the qkv
weight gets zero rows and the proj weight zero columns per head, so the padded lanes carry zeros
through attention, and the softmax keeps the 1 / sqrt(104) scale.
"""
from __future__ import annotations

import math
from dataclasses import dataclass
from typing import Dict, Optional

import torch
import torch.nn.functional as F
from torch import nn


@dataclass
class CLIPVisionConfig:
    patch_size: int = 14
    image_size: int = 224
    width: int = 1024
    layers: int = 24
    heads: int = 16
    mlp_ratio: float = 4.0
    embed_dim: int = 768           # output projection
    eps: float = 1e-5

    @property
    def head_dim(self) -> int:
        return self.width // self.heads


CLIP_PRESETS: Dict[str, CLIPVisionConfig] = {
    "clip_vitb16": CLIPVisionConfig(patch_size=16, width=768, layers=12, heads=12, embed_dim=512),
    "clip_vitl14": CLIPVisionConfig(),
    "clip_vitbigg14": CLIPVisionConfig(width=1664, layers=48, heads=16, mlp_ratio=8192 / 1664, embed_dim=1280),
    "clip_tiny": CLIPVisionConfig(patch_size=16, width=256, layers=2, heads=4, embed_dim=128),
    # bigG-shaped head width (104) on a small tower, for tests of the padded-head path
    "clip_tiny_hd104": CLIPVisionConfig(patch_size=16, width=416, layers=2, heads=4, mlp_ratio=2.0, embed_dim=128),
}


class CLIPBlock(nn.Module):
    def __init__(self, c: CLIPVisionConfig):
        super().__init__()
        d = c.width
        self.c = c
        self.ln_1, self.ln_2 = nn.LayerNorm(d, eps=c.eps), nn.LayerNorm(d, eps=c.eps)
        self.qkv = nn.Linear(d, 3 * d)
        self.proj = nn.Linear(d, d)
        self.fc1, self.fc2 = nn.Linear(d, int(d * c.mlp_ratio)), nn.Linear(int(d * c.mlp_ratio), d)

    def forward(self, x):
        B, N, D = x.shape
        q, k, v = self.qkv(self.ln_1(x)).view(B, N, 3, self.c.heads, self.c.head_dim).permute(2, 0, 3, 1, 4)
        a = F.scaled_dot_product_attention(q, k, v).transpose(1, 2).reshape(B, N, D)
        x = x + self.proj(a)
        return x + self.fc2(F.gelu(self.fc1(self.ln_2(x))))


class CLIPVision(nn.Module):
    def __init__(self, c: CLIPVisionConfig):
        super().__init__()
        self.c = c
        g = c.image_size // c.patch_size
        self.conv1 = nn.Conv2d(3, c.width, c.patch_size, c.patch_size, bias=False)
        self.class_embedding = nn.Parameter(torch.zeros(c.width))
        self.positional_embedding = nn.Parameter(torch.zeros(1 + g * g, c.width))
        self.ln_pre = nn.LayerNorm(c.width, eps=c.eps)
        self.blocks = nn.ModuleList([CLIPBlock(c) for _ in range(c.layers)])
        self.ln_post = nn.LayerNorm(c.width, eps=c.eps)
        self.proj = nn.Parameter(torch.zeros(c.width, c.embed_dim))

    def init_weights(self, seed: int = 0) -> "CLIPVision":
        g = torch.Generator().manual_seed(seed)
        with torch.no_grad():
            for name, p in self.named_parameters():
                if name.endswith("weight") and p.dim() == 1:
                    p.copy_(1 + 0.05 * torch.randn(p.shape, generator=g))
                elif name.endswith("bias"):
                    p.copy_(0.02 * torch.randn(p.shape, generator=g))
                else:
                    fan = p.shape[-1] if p.dim() > 1 else p.numel()
                    p.copy_(torch.randn(p.shape, generator=g) / math.sqrt(fan))
        return self.eval()

    def tokens(self, img: torch.Tensor) -> torch.Tensor:
        """Normalised float image [B, 3, H, W] at the native grid -> ln_pre(tokens) [B, 1+P, D]."""
        x = self.conv1(img).flatten(2).transpose(1, 2)
        cls = self.class_embedding.expand(x.shape[0], 1, -1)
        return self.ln_pre(torch.cat([cls, x], 1) + self.positional_embedding)

    def forward(self, img: torch.Tensor) -> torch.Tensor:
        x = self.tokens(img)
        for blk in self.blocks:
            x = blk(x)
        return F.normalize(self.ln_post(x[:, 0]) @ self.proj, dim=-1)


def padded_head_dim(head_dim: int) -> int:
    """Attention width the engine runs a head at: 64 or 128 (0: no padding needed)."""
    if head_dim in (64, 128):
        return 0
    if head_dim < 64:
        return 64
    if head_dim < 128:
        return 128
    raise ValueError(f"head dim {head_dim} > 128 is not supported by the engine")


def clip_vit_config(c: CLIPVisionConfig):
    from .dinov3.vit import ViTConfig

    return ViTConfig(img_size=c.image_size, patch_size=c.patch_size, embed_dim=c.width, depth=c.layers,
                     num_heads=c.heads, ffn_ratio=c.mlp_ratio, qkv_bias=True, layerscale_init=None,
                     norm_layer="layernormbf16", ffn_layer="mlp", n_storage_tokens=0,
                     padded_head_dim=padded_head_dim(c.head_dim))


def pad_heads(qkv_w, qkv_b, proj_w, heads: int, hd: int, hp: int):
    """qkv [3*H*hd, D] -> [3*H*hp, D] and its bias, proj [D, H*hd] -> [D, H*hp], zero-filled."""
    D = qkv_w.shape[1]
    w = qkv_w.new_zeros(3, heads, hp, D)
    w[:, :, :hd] = qkv_w.view(3, heads, hd, D)
    b = None
    if qkv_b is not None:
        b = qkv_b.new_zeros(3, heads, hp)
        b[:, :, :hd] = qkv_b.view(3, heads, hd)
        b = b.reshape(-1)
    p = proj_w.new_zeros(proj_w.shape[0], heads, hp)
    p[:, :, :hd] = proj_w.view(proj_w.shape[0], heads, hd)
    return w.reshape(3 * heads * hp, D), b, p.reshape(proj_w.shape[0], heads * hp)


def clip_engine_weights(model: CLIPVision, device):
    """Kernel-layout weights of a CLIP tower for models/engine.py (LayerScale 1, no RoPE,
    learned position embedding, ln_pre before the first block)."""
    from .engine import EngineWeights, LayerW

    c = model.c
    hp = padded_head_dim(c.head_dim)
    bf = lambda t: t.detach().to(device=device, dtype=torch.bfloat16).contiguous()  # noqa: E731
    ones = torch.ones(c.width, device=device, dtype=torch.bfloat16)
    layers = []
    for b in model.blocks:
        qkv_w, qkv_b, proj_w = b.qkv.weight.detach(), b.qkv.bias.detach(), b.proj.weight.detach()
        if hp:
            qkv_w, qkv_b, proj_w = pad_heads(qkv_w, qkv_b, proj_w, c.heads, c.head_dim, hp)
        layers.append(LayerW(norm1_w=bf(b.ln_1.weight), norm1_b=bf(b.ln_1.bias), qkv_w=bf(qkv_w), qkv_b=bf(qkv_b),
                             proj_w=bf(proj_w), proj_b=bf(b.proj.bias), ls1=ones, norm2_w=bf(b.ln_2.weight),
                             norm2_b=bf(b.ln_2.bias), fc1_w=bf(b.fc1.weight), fc1_b=bf(b.fc1.bias),
                             fc2_w=bf(b.fc2.weight), fc2_b=bf(b.fc2.bias), ls2=ones))
    pw = model.conv1.weight.detach()
    return EngineWeights(cfg=clip_vit_config(c), patch_w=bf(pw.reshape(pw.shape[0], -1)),
                         patch_b=torch.zeros(c.width, device=device, dtype=torch.bfloat16),
                         prefix=bf(model.class_embedding[None]), periods=None, layers=layers,
                         norm_w=bf(model.ln_post.weight), norm_b=bf(model.ln_post.bias),
                         pos_embed=bf(model.positional_embedding), pre_norm_w=bf(model.ln_pre.weight),
                         pre_norm_b=bf(model.ln_pre.bias), pixel_mean=CLIP_MEAN, pixel_std=CLIP_STD)


CLIP_MEAN = (0.48145466, 0.4578275, 0.40821073)
CLIP_STD = (0.26862954, 0.26130258, 0.27577711)
