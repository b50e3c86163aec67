"""SAM 3-shaped vision tower (windowed-attention ViT) for the approximate / correct engine.

Reference: offload/server/model/sam3_executor.py:41-190 and appcorr/models/sam3/vision/block.py
(approx / correct of the windowed ViT layers: 28 of 32 layers attend inside 24x24-patch windows,
layers 7/15/23/31 globally; RoPE coordinates are window-local on windowed layers; a corrected
query attends only to its own window). Geometry as facebook/sam3: 1008 px, patch 14 (72x72
tokens, 9 windows of 576), hidden 1024, 16 heads, MLP 4736, LayerNorm eps 1e-6, no LayerScale,
no class token, learned absolute position embedding.

The engine keeps tokens window-major, so a windowed layer of the approximate pass is one batched
attention over windows and a corrected query's key range is its window ([q_lo, q_hi] per packed
query in the attention kernel). `SAM3Tower` is the fp32 reference of the same math (token order
window-major as in the engine; RoPE tables from models/engine.py rope_tables).
"""
from __future__ import annotations

import math
from typing import Dict, Optional

import torch
import torch.nn.functional as F
from torch import nn

from .dinov3.layers import RopePositionEmbedding
from .dinov3.vit import ViTConfig
from .qwen25vl import window_order

SAM3_PRESETS: Dict[str, ViTConfig] = {
    "sam3_vitl14": ViTConfig(img_size=1008, patch_size=14, embed_dim=1024, depth=32, num_heads=16,
                             ffn_ratio=4736 / 1024, qkv_bias=True, layerscale_init=None, norm_layer="layernorm",
                             ffn_layer="mlp", n_storage_tokens=0, cls_token=False, pos_embed_rope_base=10000.0,
                             pos_embed_rope_rescale_coords=None, window_size=24, global_layers=(7, 15, 23, 31)),
    "sam3_tiny": ViTConfig(img_size=224, patch_size=14, embed_dim=256, depth=3, num_heads=4, ffn_ratio=4,
                           qkv_bias=True, layerscale_init=None, norm_layer="layernorm", ffn_layer="mlp",
                           n_storage_tokens=0, cls_token=False, pos_embed_rope_base=10000.0, pos_embed_rope_rescale_coords=None,
                           window_size=8, global_layers=(1,)),
}


def _rot(x, sin, cos):
    h = x.shape[-1] // 2
    return x * cos + torch.cat([-x[..., h:], x[..., :h]], -1) * sin


class SAM3Block(nn.Module):
    def __init__(self, c: ViTConfig):
        super().__init__()
        d = c.embed_dim
        self.c = c
        self.norm1, self.norm2 = nn.LayerNorm(d, eps=c.norm_eps), nn.LayerNorm(d, eps=c.norm_eps)
        self.qkv = nn.Linear(d, 3 * d)
        self.proj = nn.Linear(d, d)
        self.fc1, self.fc2 = nn.Linear(d, c.ffn_hidden), nn.Linear(c.ffn_hidden, d)

    def forward(self, x, sin, cos, windows: int):
        """x [B, N, D] window-major; windows = number of attention groups per image (1: global)."""
        B, N, D = x.shape
        H, Dh = self.c.num_heads, self.c.head_dim
        q, k, v = self.qkv(self.norm1(x)).view(B, N, 3, H, Dh).unbind(2)
        q, k = _rot(q, sin[:, None], cos[:, None]), _rot(k, sin[:, None], cos[:, None])
        w = N // windows
        q, k, v = (t.view(B * windows, w, H, Dh).transpose(1, 2) for t in (q, k, v))
        o = F.scaled_dot_product_attention(q, k, v).transpose(1, 2).reshape(B, N, D)
        x = x + self.proj(o)
        return x + self.fc2(F.gelu(self.fc1(self.norm2(x))))


class SAM3Tower(nn.Module):
    def __init__(self, c: ViTConfig):
        super().__init__()
        self.c = c
        g = c.img_size // c.patch_size
        self.patch_embed = nn.Conv2d(3, c.embed_dim, c.patch_size, c.patch_size)
        self.pos_embed = nn.Parameter(torch.zeros(g * g, c.embed_dim))  # window-major token order
        self.rope = RopePositionEmbedding(c.embed_dim, num_heads=c.num_heads, base=c.pos_embed_rope_base,
                                          normalize_coords=c.pos_embed_rope_normalize_coords,
                                          rescale_coords=c.pos_embed_rope_rescale_coords, dtype=torch.float32)
        self.blocks = nn.ModuleList([SAM3Block(c) for _ in range(c.depth)])
        self.norm = nn.LayerNorm(c.embed_dim, eps=c.norm_eps)

    def init_weights(self, seed: int = 0) -> "SAM3Tower":
        g = torch.Generator().manual_seed(seed)
        with torch.no_grad():
            for name, p in self.named_parameters():
                if name.endswith("weight") and p.dim() == 1:
                    p.copy_(1 + 0.05 * torch.randn(p.shape, generator=g))
                elif name.endswith("bias"):
                    p.copy_(0.02 * torch.randn(p.shape, generator=g))
                else:
                    fan = p[0].numel() if p.dim() > 1 else p.numel()
                    p.copy_(torch.randn(p.shape, generator=g) / math.sqrt(fan))
        return self.eval()

    def forward(self, img: torch.Tensor) -> torch.Tensor:
        """Normalised float image [B, 3, H, W] -> final-normed tokens [B, N, D] (window-major)."""
        from .engine import rope_tables

        c = self.c
        B = img.shape[0]
        gh, gw = img.shape[2] // c.patch_size, img.shape[3] // c.patch_size
        order = window_order(gh, gw, c.window_size, 1).to(img.device)
        x = self.patch_embed(img).flatten(2).transpose(1, 2)[:, order] + self.pos_embed
        per = self.rope.periods.to(img.device)
        sg, cg = rope_tables(c, per, gh, gw)
        sg, cg = sg[order], cg[order]
        sw, cw = rope_tables(c, per, c.window_size, c.window_size)
        nw = (gh // c.window_size) * (gw // c.window_size)
        sw, cw = sw.repeat(nw, 1), cw.repeat(nw, 1)
        for i, blk in enumerate(self.blocks):
            glob = i in c.global_layers
            x = blk(x, sg if glob else sw, cg if glob else cw, 1 if glob else nw)
        return self.norm(x)


def sam3_engine_weights(model: SAM3Tower, device):
    from .engine import EngineWeights, LayerW

    c = model.c
    bf = lambda t: t.detach().to(device=device, dtype=torch.bfloat16).contiguous()  # noqa: E731
    ones = torch.ones(c.embed_dim, device=device, dtype=torch.bfloat16)
    layers = [LayerW(norm1_w=bf(b.norm1.weight), norm1_b=bf(b.norm1.bias), qkv_w=bf(b.qkv.weight),
                     qkv_b=bf(b.qkv.bias), proj_w=bf(b.proj.weight), proj_b=bf(b.proj.bias), ls1=ones,
                     norm2_w=bf(b.norm2.weight), norm2_b=bf(b.norm2.bias), fc1_w=bf(b.fc1.weight),
                     fc1_b=bf(b.fc1.bias), fc2_w=bf(b.fc2.weight), fc2_b=bf(b.fc2.bias), ls2=ones)
              for b in model.blocks]
    pw = model.patch_embed.weight.detach()
    return EngineWeights(cfg=c, patch_w=bf(pw.reshape(pw.shape[0], -1)), patch_b=bf(model.patch_embed.bias),
                         prefix=torch.zeros(0, c.embed_dim, device=device, dtype=torch.bfloat16),
                         periods=model.rope.periods.detach().to(device=device, dtype=torch.float32),
                         layers=layers, norm_w=bf(model.norm.weight), norm_b=bf(model.norm.bias),
                         pos_embed=bf(model.pos_embed))


# ----------------------------------------------------------------------------- stock SAM 3 head
# Downstream of the tower the reference runs the stock `transformers` Sam3Model untouched, fed
# with the tower's features through `vision_embeds` (offload/server/model/sam3_executor.py:140-160):
# FPN neck, CLIP text encoder, geometry (box prompt) encoder, DETR encoder / decoder, mask decoder
# and scoring. The same is done here; only the stock model's own ViT backbone is dropped, since the
# features come from this build's tower. Random init (no checkpoints offline).
CLIP_BOS, CLIP_EOS = 49406, 49407


def stock_head_config(c: ViTConfig):
    """Sam3Config whose vision backbone geometry matches tower config `c`. Towers of the
    facebook/sam3 width (1024) take the stock defaults of every downstream part; narrower test
    towers get a proportionally small detector."""
    from transformers.models.sam3 import configuration_sam3 as hf

    g = c.img_size // c.patch_size
    back = dict(hidden_size=c.embed_dim, num_attention_heads=c.num_heads, image_size=c.img_size,
                patch_size=c.patch_size, window_size=c.window_size, global_attn_indexes=list(c.global_layers),
                num_hidden_layers=c.depth)
    if c.embed_dim >= 1024:
        return hf.Sam3Config(vision_config=dict(backbone_config=back))
    small = dict(hidden_size=64, num_attention_heads=2, intermediate_size=128)
    return hf.Sam3Config(
        vision_config=dict(backbone_config=back, fpn_hidden_size=64, backbone_feature_sizes=[[4 * g, 4 * g],
                                                                                            [2 * g, 2 * g], [g, g]]),
        text_config=dict(hidden_size=64, intermediate_size=128, num_hidden_layers=1, num_attention_heads=2,
                         projection_dim=64),
        geometry_encoder_config=dict(num_layers=1, **small),
        detr_encoder_config=dict(num_layers=1, **small),
        detr_decoder_config=dict(num_layers=1, num_queries=20, **small),
        mask_decoder_config=dict(hidden_size=64, num_attention_heads=2))


def build_stock_head(c: ViTConfig, seed: int = 0, device=None, dtype=torch.float32):
    """The stock Sam3Model for tower config `c`, without its own vision backbone (nn.Identity)."""
    from transformers.models.sam3.modeling_sam3 import Sam3Model

    torch.manual_seed(seed)
    m = Sam3Model(stock_head_config(c)).eval()
    m.vision_encoder.backbone = nn.Identity()
    return m.to(device=device, dtype=dtype)


def stock_head_forward(model, feat: torch.Tensor, boxes: Optional[torch.Tensor] = None,
                       input_ids: Optional[torch.Tensor] = None):
    """Tower features in raster order [B, gh, gw, D] -> the stock detector's outputs
    (pred_masks, pred_boxes, pred_logits, ...). boxes: [B, n, 4] normalised (cx, cy, w, h) box
    prompts (default: one whole-image box per image); input_ids: the text prompt (default: the
    empty CLIP prompt, BOS + EOS)."""
    from transformers.models.sam3.modeling_sam3 import Sam3VisionEncoderOutput

    B = feat.shape[0]
    dtype = next(model.parameters()).dtype
    x = feat.to(dtype).permute(0, 3, 1, 2).contiguous()
    fpn, pos = model.vision_encoder.neck(x)
    if boxes is None:
        boxes = torch.tensor([0.5, 0.5, 1.0, 1.0], device=feat.device).repeat(B, 1, 1)
    if input_ids is None:
        input_ids = torch.tensor([[CLIP_BOS, CLIP_EOS]], device=feat.device).repeat(B, 1)
    with torch.no_grad():
        return model(vision_embeds=Sam3VisionEncoderOutput(fpn_hidden_states=fpn, fpn_position_encoding=pos),
                     input_ids=input_ids, input_boxes=boxes.to(dtype))


def raster_features(tokens: torch.Tensor, c: ViTConfig, gh: int, gw: int) -> torch.Tensor:
    """Window-major tower tokens [B, N, D] -> raster feature map [B, gh, gw, D]."""
    order = window_order(gh, gw, c.window_size, 1).to(tokens.device)
    out = torch.empty_like(tokens)
    out[:, order] = tokens
    return out.view(tokens.shape[0], gh, gw, -1)
