"""DINOv3 vision transformer (module tree + factories) and the token group index.

State-dict compatible with the reference backbone (appcorr/models/dinov3/models/
vision_transformer.py:176-297, hub/backbones.py:201-490). Size presets: ViT-S/16, ViT-B/16,
ViT-L/16, ViT-7B/16.
"""
from __future__ import annotations

from dataclasses import asdict, dataclass, field
from functools import partial
from typing import Any, Dict, List, Optional, Tuple

import torch
from torch import Tensor, nn

from .layers import (
    LayerScale,
    LinearKMaskedBias,
    Mlp,
    PatchEmbed,
    RopePositionEmbedding,
    SelfAttentionBlock,
    SwiGLUFFN,
)

_FFN = {
    "mlp": Mlp,
    "swiglu": SwiGLUFFN,
    "swiglu32": partial(SwiGLUFFN, align_to=32),
    "swiglu64": partial(SwiGLUFFN, align_to=64),
    "swiglu128": partial(SwiGLUFFN, align_to=128),
}
_NORM_EPS = {"layernorm": 1e-6, "layernormbf16": 1e-5}
_DTYPES = {"fp32": torch.float32, "fp16": torch.float16, "bf16": torch.bfloat16}


@dataclass
class ViTConfig:
    img_size: int = 224
    patch_size: int = 16
    in_chans: int = 3
    pos_embed_rope_base: float = 100.0
    pos_embed_rope_normalize_coords: str = "separate"
    pos_embed_rope_rescale_coords: Optional[float] = 2.0
    pos_embed_rope_dtype: str = "fp32"
    embed_dim: int = 768
    depth: int = 12
    num_heads: int = 12
    ffn_ratio: float = 4.0
    qkv_bias: bool = True
    layerscale_init: Optional[float] = 1.0e-5
    norm_layer: str = "layernormbf16"
    ffn_layer: str = "mlp"
    ffn_bias: bool = True
    proj_bias: bool = True
    n_storage_tokens: int = 4
    mask_k_bias: bool = True
    untie_cls_and_patch_norms: bool = False
    untie_global_and_local_cls_norm: bool = False
    # windowed attention (SAM-style towers; engine only): square windows of `window_size` patches,
    # global attention at `global_layers`; window-local RoPE coordinates on windowed layers
    window_size: int = 0
    global_layers: Tuple[int, ...] = ()
    window_rope_everywhere: bool = False  # global layers also use window-local RoPE (multi-frame towers)
    cls_token: bool = True                # False: patch tokens only (SAM- / VGGT-style towers)
    # engine only: attention heads zero-padded to this width (0: head_dim). Lets towers whose
    # head dim is not 64 / 128 (CLIP bigG: 104) run the 64 / 128 attention kernels; the softmax
    # scale stays 1 / sqrt(head_dim)
    padded_head_dim: int = 0

    @property
    def head_dim(self) -> int:
        return self.embed_dim // self.num_heads

    @property
    def n_prefix(self) -> int:
        return int(self.cls_token) + self.n_storage_tokens

    @property
    def norm_eps(self) -> float:
        return _NORM_EPS[self.norm_layer]

    @property
    def ffn_hidden(self) -> int:
        hidden = int(self.embed_dim * self.ffn_ratio)
        if self.ffn_layer.startswith("swiglu"):
            align = int(self.ffn_layer[6:] or 8)
            d = int(hidden * 2 / 3)
            return d + (-d % align)
        return hidden

    @property
    def is_swiglu(self) -> bool:
        return self.ffn_layer.startswith("swiglu")


PRESETS: Dict[str, ViTConfig] = {
    "vits16": ViTConfig(embed_dim=384, depth=12, num_heads=6, ffn_ratio=4, ffn_layer="mlp"),
    "vitb16": ViTConfig(embed_dim=768, depth=12, num_heads=12, ffn_ratio=4, ffn_layer="mlp"),
    "vitl16": ViTConfig(embed_dim=1024, depth=24, num_heads=16, ffn_ratio=4, ffn_layer="mlp"),
    "vit7b16": ViTConfig(embed_dim=4096, depth=40, num_heads=32, ffn_ratio=3, qkv_bias=False, ffn_layer="swiglu64",
                         untie_global_and_local_cls_norm=True),
}


class DinoVisionTransformer(nn.Module):
    def __init__(self, cfg: ViTConfig, device=None):
        super().__init__()
        self.cfg = cfg
        norm = partial(nn.LayerNorm, eps=cfg.norm_eps)
        self.num_features = self.embed_dim = cfg.embed_dim
        self.n_blocks = cfg.depth
        self.num_heads = cfg.num_heads
        self.patch_size = cfg.patch_size
        self.patch_embed = PatchEmbed(cfg.img_size, cfg.patch_size, cfg.in_chans, cfg.embed_dim)
        self.cls_token = nn.Parameter(torch.empty(1, 1, cfg.embed_dim, device=device))
        self.n_storage_tokens = cfg.n_storage_tokens
        if cfg.n_storage_tokens > 0:
            self.storage_tokens = nn.Parameter(torch.empty(1, cfg.n_storage_tokens, cfg.embed_dim, device=device))
        self.rope_embed = RopePositionEmbedding(
            cfg.embed_dim, num_heads=cfg.num_heads, base=cfg.pos_embed_rope_base,
            normalize_coords=cfg.pos_embed_rope_normalize_coords, rescale_coords=cfg.pos_embed_rope_rescale_coords,
            dtype=_DTYPES[cfg.pos_embed_rope_dtype], device=device)
        ffn = _FFN[cfg.ffn_layer]
        self.blocks = nn.ModuleList([
            SelfAttentionBlock(cfg.embed_dim, cfg.num_heads, ffn_ratio=cfg.ffn_ratio, qkv_bias=cfg.qkv_bias,
                               proj_bias=cfg.proj_bias, ffn_bias=cfg.ffn_bias, norm_layer=norm, act_layer=nn.GELU,
                               ffn_layer=ffn, init_values=cfg.layerscale_init, mask_k_bias=cfg.mask_k_bias,
                               device=device)
            for _ in range(cfg.depth)
        ])
        self.chunked_blocks = False
        self.norm = norm(cfg.embed_dim)
        self.untie_cls_and_patch_norms = cfg.untie_cls_and_patch_norms
        self.cls_norm = norm(cfg.embed_dim) if cfg.untie_cls_and_patch_norms else None
        self.untie_global_and_local_cls_norm = cfg.untie_global_and_local_cls_norm
        self.local_cls_norm = norm(cfg.embed_dim) if cfg.untie_global_and_local_cls_norm else None
        self.head = nn.Identity()
        self.mask_token = nn.Parameter(torch.empty(1, cfg.embed_dim, device=device))

    # -- init (random weights for synthetic benchmarks)
    def init_weights(self, seed: Optional[int] = None) -> "DinoVisionTransformer":
        gen = None
        if seed is not None:
            torch.manual_seed(seed)
        self.rope_embed._init_weights()
        nn.init.normal_(self.cls_token, std=0.02)
        if self.n_storage_tokens > 0:
            nn.init.normal_(self.storage_tokens, std=0.02)
        nn.init.zeros_(self.mask_token)
        for m in self.modules():
            if isinstance(m, nn.Linear):
                nn.init.trunc_normal_(m.weight, std=0.02, generator=gen)
                if m.bias is not None:
                    nn.init.zeros_(m.bias)
                if isinstance(m, LinearKMaskedBias) and m.bias is not None:
                    o = m.out_features
                    m.bias_mask.fill_(1)
                    m.bias_mask[o // 3: 2 * o // 3].fill_(0)
            elif isinstance(m, nn.LayerNorm):
                m.reset_parameters()
            elif isinstance(m, (LayerScale, PatchEmbed)):
                m.reset_parameters()
        return self

    # -- tokens
    def prepare_tokens_with_masks(self, x: Tensor, masks: Optional[Tensor] = None) -> Tuple[Tensor, Tuple[int, int]]:
        x = self.patch_embed(x)
        B, H, W, _ = x.shape
        x = x.flatten(1, 2)
        cls = self.cls_token
        if masks is not None:
            x = torch.where(masks.unsqueeze(-1), self.mask_token.to(x.dtype).unsqueeze(0), x)
        else:
            cls = cls + 0 * self.mask_token
        parts = [cls.expand(B, -1, -1)]
        if self.n_storage_tokens > 0:
            parts.append(self.storage_tokens.expand(B, -1, -1))
        parts.append(x)
        return torch.cat(parts, dim=1), (H, W)

    def prefix_tokens(self) -> Tensor:
        """[1 + n_storage, D] rows prepended to every image."""
        rows = [self.cls_token[0]]
        if self.n_storage_tokens > 0:
            rows.append(self.storage_tokens[0])
        return torch.cat(rows, dim=0)

    def final_norm(self, x: Tensor) -> Tensor:
        npre = self.n_storage_tokens + 1
        if self.untie_cls_and_patch_norms:
            return torch.cat([self.cls_norm(x[:, :npre]), self.norm(x[:, npre:])], dim=1)
        return self.norm(x)

    def forward_features(self, x: Tensor, masks: Optional[Tensor] = None) -> Dict[str, Tensor]:
        t, (H, W) = self.prepare_tokens_with_masks(x, masks)
        rope = self.rope_embed(H=H, W=W)
        for blk in self.blocks:
            t = blk(t, rope)
        xn = self.final_norm(t)
        npre = self.n_storage_tokens + 1
        return {"x_norm_clstoken": xn[:, 0], "x_storage_tokens": xn[:, 1:npre], "x_norm_patchtokens": xn[:, npre:],
                "x_prenorm": t, "masks": masks}

    def forward(self, x: Tensor, masks: Optional[Tensor] = None) -> Tensor:
        return self.head(self.forward_features(x, masks)["x_norm_clstoken"])


def build_vit(name: str, device=None, **overrides) -> DinoVisionTransformer:
    """Factory for the size presets (`vits16`, `vitb16`, `vitl16`, `vit7b16`)."""
    if name not in PRESETS:
        raise ValueError(f"unknown ViT preset {name!r}; available: {sorted(PRESETS)}")
    cfg = ViTConfig(**{**asdict(PRESETS[name]), **overrides})
    return DinoVisionTransformer(cfg, device=device)


def dinov3_vits16(pretrained: bool = False, **kw) -> DinoVisionTransformer:
    return build_vit("vits16", **kw).init_weights()


def dinov3_vitl16(pretrained: bool = False, **kw) -> DinoVisionTransformer:
    return build_vit("vitl16", **kw).init_weights()


def dinov3_vit7b16(pretrained: bool = False, **kw) -> DinoVisionTransformer:
    return build_vit("vit7b16", **kw).init_weights()


# ------------------------------------------------------------------------------ group index
def create_group_index(num_tokens: int, num_groups: int, strategy: str, device=None, **kwargs) -> Tensor:
    """Group id (1..num_groups) of each patch token; must agree bit-for-bit with the client's
    assignment of residual patches to groups (vision_transformer.py:59-174 <->
    transmission/progressive.py:245-294)."""
    device = device or "cpu"
    if strategy == "uniform":
        return torch.randint(1, num_groups + 1, (num_tokens,), device=device)
    if strategy in {"grid", "block_grid", "expansion"}:
        hw = kwargs.get("token_hw")
        H, W = (int(num_tokens ** 0.5),) * 2 if hw is None else tuple(map(int, hw))
        if H * W != num_tokens:
            raise ValueError(f"{strategy} grouping requires token_hw whose product matches num_tokens, "
                             f"got token_hw=({H}, {W}) and num_tokens={num_tokens}")
        rows = torch.arange(H, device=device).unsqueeze(1)
        cols = torch.arange(W, device=device).unsqueeze(0)
        if strategy == "grid":
            s = int(num_groups ** 0.5)
            pattern = torch.arange(1, num_groups + 1, device=device).view(s, s)
            return pattern.repeat(-(-H // s), -(-W // s))[:H, :W].flatten()
        if strategy == "block_grid":
            s = int(num_groups ** 0.5)
            if s * s != num_groups:
                raise ValueError(f"block_grid grouping requires a square num_groups, got {num_groups}")
            return ((rows * s // max(H, 1)) * s + (cols * s // max(W, 1)) + 1).flatten()
        if num_groups > num_tokens:
            raise ValueError(f"expansion grouping needs at least one token per group, got num_groups={num_groups} "
                             f"for {num_tokens} tokens")
        # centre-out rings of equal area with an integer-only distance key
        key = ((2 * rows - (H - 1)) ** 2 * max(W - 1, 1) ** 2 + (2 * cols - (W - 1)) ** 2 * max(H - 1, 1) ** 2).flatten()
        order = torch.argsort(key, stable=True)
        rank = torch.empty(num_tokens, dtype=torch.long, device=device)
        rank[order] = torch.arange(num_tokens, device=device)
        return rank * num_groups // num_tokens + 1
    if strategy == "geometric":
        u = torch.rand(num_tokens, device=device)
        return torch.clamp(torch.floor(-torch.log2(1 - u)) + 1, max=num_groups).long()
    if strategy == "uniform_diff":
        diffs = kwargs.get("token_diffs")
        if diffs is None:
            raise ValueError("token_diffs must be provided for 'uniform_diff' grouping strategy.")
        norms = torch.norm(diffs, p=1, dim=-1)
        B, N = norms.shape
        sorted_norms, sorted_idx = torch.sort(norms, dim=1)
        cum = torch.cumsum(sorted_norms.mean(0), 0)
        total = cum[-1]
        if total == 0:
            return torch.randint(1, num_groups + 1, (B * N,), device=device).view(B, N)
        bounds = torch.arange(1, num_groups, device=device, dtype=torch.float32) * (total / num_groups)
        template = torch.bucketize(cum, bounds) + 1
        out = torch.zeros_like(norms, dtype=torch.long)
        out.scatter_(1, sorted_idx, template.unsqueeze(0).expand(B, -1))
        return out
    raise NotImplementedError(f"Unknown grouping strategy: {strategy}")
