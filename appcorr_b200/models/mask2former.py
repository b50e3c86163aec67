"""DINOv3 Mask2Former segmentor: ViT adapter, multi-scale deformable pixel decoder and
masked-attention transformer decoder, with sliding-window (crop) inference.

Reference (behaviour and state-dict layout):
- adapter: appcorr/models/dinov3/eval/segmentation/models/backbone/dinov3_adapter.py
  (SpatialPriorModule :234, Extractor :112, InteractionBlockWithCls :159, DINOv3_Adapter :305-484)
- pixel decoder: .../models/heads/pixel_decoder.py (MSDeformAttnPixelDecoder :239-412,
  encoder layer :166-205)
- decoder: .../models/heads/mask2former_transformer_decoder.py (:271-462)
- head: .../models/heads/mask2former_head.py (:12-96); semantic inference and sliding windows:
  .../segmentation/inference.py (:80-160)

The modules here are fp32 PyTorch oracles whose parameter names follow the reference's
checkpoints (`segmentation_model.0.*` = adapter without its backbone, `segmentation_model.1.*`
= head), so a DINOv3 M2F head checkpoint loads with strict names. The adapter does not own the
backbone: it takes the four tapped layer outputs of the approximate / correct ViT engine (the
reference calls `backbone.get_intermediate_layers` inside the adapter). `Mask2FormerGPU` runs
the same network on the sm_100a kernels (tcgen05 GEMMs for every linear / 1x1 / im2col conv,
the fused deformable-attention kernel, LayerNorm, bilinear resize); GroupNorm, BatchNorm-free
small maps and the masked softmax of the 100-query decoder stay PyTorch ops.
"""
from __future__ import annotations

import math
from typing import Dict, List, Optional, Sequence, Tuple

import torch
import torch.nn.functional as F
from torch import nn

from .m2f import msda_reference


# ----------------------------------------------------------------------------- shared pieces
def sine_pos_normalized(h: int, w: int, num_feats: int, device, temperature: float = 10000.0) -> torch.Tensor:
    """Normalised sine position embedding of an h x w map -> [2*num_feats, h, w] (y features first,
    then x; even feature indices sin, odd cos; coordinates scaled to (0, 2*pi])."""
    eps, scale = 1e-6, 2 * math.pi
    y = torch.arange(1, h + 1, dtype=torch.float32, device=device)[:, None].expand(h, w)
    x = torch.arange(1, w + 1, dtype=torch.float32, device=device)[None, :].expand(h, w)
    y = y / (h + eps) * scale
    x = x / (w + eps) * scale
    dim_t = temperature ** (2 * (torch.arange(num_feats, dtype=torch.float32, device=device) // 2) / num_feats)
    px = x[..., None] / dim_t
    py = y[..., None] / dim_t
    px = torch.stack((px[..., 0::2].sin(), px[..., 1::2].cos()), -1).flatten(2)
    py = torch.stack((py[..., 0::2].sin(), py[..., 1::2].cos()), -1).flatten(2)
    return torch.cat((py, px), -1).permute(2, 0, 1).contiguous()


def centre_points(shapes: Sequence[Tuple[int, int]], device) -> torch.Tensor:
    """[S, 2] normalised (x, y) centre of every cell of each map, maps concatenated."""
    pts = []
    for h, w in shapes:
        yy, xx = torch.meshgrid((torch.arange(h, device=device, dtype=torch.float32) + 0.5) / h,
                                (torch.arange(w, device=device, dtype=torch.float32) + 0.5) / w, indexing="ij")
        pts.append(torch.stack([xx.reshape(-1), yy.reshape(-1)], -1))
    return torch.cat(pts, 0)


class MSDeformAttnR(nn.Module):
    """Deformable attention whose value width is d_model * ratio (the adapter uses ratio 0.5)."""

    def __init__(self, d_model: int, n_levels: int, n_heads: int, n_points: int, ratio: float = 1.0):
        super().__init__()
        self.d_model, self.n_levels, self.n_heads, self.n_points = d_model, n_levels, n_heads, n_points
        self.dv = int(d_model * ratio)
        self.sampling_offsets = nn.Linear(d_model, n_heads * n_levels * n_points * 2)
        self.attention_weights = nn.Linear(d_model, n_heads * n_levels * n_points)
        self.value_proj = nn.Linear(d_model, self.dv)
        self.output_proj = nn.Linear(self.dv, d_model)

    def forward(self, query, ref, value_in, shapes):
        """query [N, Q, d], ref [N, Q, L, 2] (x, y in [0, 1]), value_in [N, S, d] -> [N, Q, d]."""
        N, Q, _ = query.shape
        M, L, P = self.n_heads, self.n_levels, self.n_points
        v = self.value_proj(value_in).view(N, value_in.shape[1], M, self.dv // M)
        off = self.sampling_offsets(query).view(N, Q, M, L, P, 2)
        w = F.softmax(self.attention_weights(query).view(N, Q, M, L * P), -1).view(N, Q, M, L, P)
        norm = torch.tensor([[w_, h_] for h_, w_ in shapes], dtype=query.dtype, device=query.device)
        loc = ref[:, :, None, :, None, :] + off / norm[None, None, None, :, None, :]
        return self.output_proj(msda_reference(v, shapes, loc, w))


# ----------------------------------------------------------------------------- adapter
class DWConv(nn.Module):
    def __init__(self, dim: int):
        super().__init__()
        self.dwconv = nn.Conv2d(dim, dim, 3, 1, 1, bias=True, groups=dim)

    def forward(self, x, H, W):
        """x [B, 21n, C]: tokens of the stride-8, 16 and 32 maps (16n, 4n, n) of an H x W (stride 16) grid."""
        B, N, C = x.shape
        n = N // 21
        maps = [(0, 16 * n, 2 * H, 2 * W), (16 * n, 20 * n, H, W), (20 * n, N, H // 2, W // 2)]
        outs = [self.dwconv(x[:, a:b].transpose(1, 2).reshape(B, C, h, w)).flatten(2).transpose(1, 2)
                for a, b, h, w in maps]
        return torch.cat(outs, 1)


class ConvFFN(nn.Module):
    def __init__(self, dim: int, hidden: int):
        super().__init__()
        self.fc1 = nn.Linear(dim, hidden)
        self.dwconv = DWConv(hidden)
        self.fc2 = nn.Linear(hidden, dim)

    def forward(self, x, H, W):
        return self.fc2(F.gelu(self.dwconv(self.fc1(x), H, W)))


class Extractor(nn.Module):
    """query (the adapter's conv tokens) += deform-attn(LN(query) -> LN(ViT tokens)); += ConvFFN."""

    def __init__(self, dim: int, heads: int, points: int, ratio: float, cffn_ratio: float):
        super().__init__()
        self.query_norm = nn.LayerNorm(dim, eps=1e-6)
        self.feat_norm = nn.LayerNorm(dim, eps=1e-6)
        self.attn = MSDeformAttnR(dim, 1, heads, points, ratio)
        self.ffn = ConvFFN(dim, int(dim * cffn_ratio))
        self.ffn_norm = nn.LayerNorm(dim, eps=1e-6)

    def forward(self, query, ref, feat, feat_shape, H, W):
        query = query + self.attn(self.query_norm(query), ref, self.feat_norm(feat), [feat_shape])
        return query + self.ffn(self.ffn_norm(query), H, W)


class InteractionBlock(nn.Module):
    def __init__(self, dim: int, heads: int, points: int, ratio: float, cffn_ratio: float, extra: bool):
        super().__init__()
        self.extractor = Extractor(dim, heads, points, ratio, cffn_ratio)
        self.extra_extractors = (nn.Sequential(*[Extractor(dim, heads, points, ratio, cffn_ratio) for _ in range(2)])
                                 if extra else None)

    def forward(self, x, c, ref, feat_shape, H, W):
        c = self.extractor(c, ref, x, feat_shape, H, W)
        if self.extra_extractors is not None:
            for ex in self.extra_extractors:
                c = ex(c, ref, x, feat_shape, H, W)
        return c


def _conv_bn_relu(cin, cout, stride):
    return [nn.Conv2d(cin, cout, 3, stride, 1, bias=False), nn.BatchNorm2d(cout), nn.ReLU(inplace=True)]


class SpatialPriorModule(nn.Module):
    """Conv stem: c1 (stride 4), c2 (8), c3 (16), c4 (32), each projected to the ViT width."""

    def __init__(self, inplanes: int, dim: int):
        super().__init__()
        self.stem = nn.Sequential(*_conv_bn_relu(3, inplanes, 2), *_conv_bn_relu(inplanes, inplanes, 1),
                                  *_conv_bn_relu(inplanes, inplanes, 1), nn.MaxPool2d(3, 2, 1))
        self.conv2 = nn.Sequential(*_conv_bn_relu(inplanes, 2 * inplanes, 2))
        self.conv3 = nn.Sequential(*_conv_bn_relu(2 * inplanes, 4 * inplanes, 2))
        self.conv4 = nn.Sequential(*_conv_bn_relu(4 * inplanes, 4 * inplanes, 2))
        self.fc1 = nn.Conv2d(inplanes, dim, 1)
        self.fc2 = nn.Conv2d(2 * inplanes, dim, 1)
        self.fc3 = nn.Conv2d(4 * inplanes, dim, 1)
        self.fc4 = nn.Conv2d(4 * inplanes, dim, 1)

    def forward(self, x):
        c1 = self.stem(x)
        c2 = self.conv2(c1)
        c3 = self.conv3(c2)
        c4 = self.conv4(c3)
        return self.fc1(c1), self.fc2(c2), self.fc3(c3), self.fc4(c4)


class DINOv3Adapter(nn.Module):
    """Everything of the reference's DINOv3_Adapter except the backbone it wraps."""

    def __init__(self, dim: int, patch: int = 16, inplanes: int = 64, points: int = 4, heads: int = 16,
                 cffn_ratio: float = 0.25, ratio: float = 0.5, n_interactions: int = 4):
        super().__init__()
        self.dim, self.patch = dim, patch
        self.level_embed = nn.Parameter(torch.zeros(3, dim))
        self.spm = SpatialPriorModule(inplanes, dim)
        self.interactions = nn.Sequential(*[
            InteractionBlock(dim, heads, points, ratio, cffn_ratio, extra=(i == n_interactions - 1))
            for i in range(n_interactions)])
        self.up = nn.ConvTranspose2d(dim, dim, 2, 2)
        self.norm1, self.norm2, self.norm3, self.norm4 = (nn.BatchNorm2d(dim) for _ in range(4))

    def forward(self, x: torch.Tensor, taps: List[torch.Tensor]) -> Dict[str, torch.Tensor]:
        """x [B, 3, h, w] normalised image (h, w multiples of 32); taps: 4 x [B, (h/p)*(w/p), dim]
        patch tokens of the interaction layers -> {"1": stride 4, ..., "4": stride 32} maps."""
        B, _, h, w = x.shape
        Hc, Wc = h // 16, w // 16
        Ht, Wt = h // self.patch, w // self.patch
        c1, c2, c3, c4 = self.spm(x)
        c2 = c2.flatten(2).transpose(1, 2) + self.level_embed[0]
        c3 = c3.flatten(2).transpose(1, 2) + self.level_embed[1]
        c4 = c4.flatten(2).transpose(1, 2) + self.level_embed[2]
        n2, n3 = c2.shape[1], c3.shape[1]
        c = torch.cat([c2, c3, c4], 1)
        ref = centre_points([(h // 8, w // 8), (h // 16, w // 16), (h // 32, w // 32)], x.device)
        ref = ref[None, :, None, :].expand(B, -1, 1, -1)
        outs = []
        for blk, t in zip(self.interactions, taps):
            c = blk(t, c, ref, (Ht, Wt), Hc, Wc)
            outs.append(t.transpose(1, 2).reshape(B, self.dim, Ht, Wt))
        c2 = c[:, :n2].transpose(1, 2).reshape(B, self.dim, 2 * Hc, 2 * Wc)
        c3 = c[:, n2:n2 + n3].transpose(1, 2).reshape(B, self.dim, Hc, Wc)
        c4 = c[:, n2 + n3:].transpose(1, 2).reshape(B, self.dim, Hc // 2, Wc // 2)
        c1 = self.up(c2) + c1
        sizes = [(4 * Hc, 4 * Wc), (2 * Hc, 2 * Wc), (Hc, Wc), (Hc // 2, Wc // 2)]
        cs = [c1, c2, c3, c4]
        for i in range(4):
            cs[i] = cs[i] + F.interpolate(outs[i], size=sizes[i], mode="bilinear", align_corners=False)
        norms = (self.norm1, self.norm2, self.norm3, self.norm4)
        return {str(i + 1): norms[i](cs[i]) for i in range(4)}


# ----------------------------------------------------------------------------- pixel decoder
class Conv2dNorm(nn.Conv2d):
    """Conv2d with an optional norm module and activation after it (`weight`, `bias`, `norm.*`)."""

    def __init__(self, *a, norm: Optional[nn.Module] = None, act: bool = False, **k):
        super().__init__(*a, **k)
        self.norm = norm
        self.act = act

    def forward(self, x):
        x = F.conv2d(x, self.weight, self.bias, self.stride, self.padding)
        if self.norm is not None:
            x = self.norm(x)
        return F.relu(x) if self.act else x


class EncoderLayer(nn.Module):
    """Post-norm deformable encoder layer: x = LN(x + attn(x + pos)); x = LN(x + FFN(x))."""

    def __init__(self, d: int, ffn: int, levels: int, heads: int, points: int):
        super().__init__()
        self.self_attn = MSDeformAttnR(d, levels, heads, points)
        self.norm1 = nn.LayerNorm(d)
        self.linear1 = nn.Linear(d, ffn)
        self.linear2 = nn.Linear(ffn, d)
        self.norm2 = nn.LayerNorm(d)

    def forward(self, x, pos, ref, shapes):
        x = self.norm1(x + self.self_attn(x + pos, ref, x, shapes))
        return self.norm2(x + self.linear2(F.relu(self.linear1(x))))


class _EncoderStack(nn.Module):
    def __init__(self, d, ffn, levels, heads, points, layers):
        super().__init__()
        self.layers = nn.ModuleList([EncoderLayer(d, ffn, levels, heads, points) for _ in range(layers)])


class _EncoderOnly(nn.Module):
    def __init__(self, d, ffn, levels, heads, points, layers):
        super().__init__()
        self.encoder = _EncoderStack(d, ffn, levels, heads, points, layers)
        self.level_encoding = nn.Parameter(torch.zeros(levels, d))


class PixelDecoder(nn.Module):
    """Input maps "2".."4" (strides 8..32) -> 1x1 conv + GroupNorm(32) -> 6 deformable encoder layers
    over the three levels -> FPN step onto "1" (stride 4) -> mask features (1x1 conv)."""

    def __init__(self, in_dim: int, d: int, mask_dim: int, heads: int = 16, ffn: int = 4096, layers: int = 6,
                 points: int = 4):
        super().__init__()
        self.d = d
        self.input_convs = nn.ModuleList([nn.Sequential(nn.Conv2d(in_dim, d, 1), nn.GroupNorm(32, d))
                                          for _ in range(3)])
        self.encoder = _EncoderOnly(d, ffn, 3, heads, points, layers)
        self.mask_feature = Conv2dNorm(d, mask_dim, 1)
        self.lateral_convs = nn.ModuleList([Conv2dNorm(in_dim, d, 1, bias=False, norm=nn.GroupNorm(32, d))])
        self.output_convs = nn.ModuleList([Conv2dNorm(d, d, 3, padding=1, bias=False, norm=nn.GroupNorm(32, d),
                                                      act=True)])

    def forward(self, feats: Dict[str, torch.Tensor]):
        """-> (mask_features [B, mask_dim, H/4, W/4], [stride-32, 16, 8 maps])."""
        srcs, pos, shapes = [], [], []
        for i, key in enumerate(("4", "3", "2")):
            x = feats[key]
            srcs.append(self.input_convs[i](x))
            h, w = x.shape[-2:]
            shapes.append((h, w))
            pos.append(sine_pos_normalized(h, w, self.d // 2, x.device))
        B = srcs[0].shape[0]
        src = torch.cat([s.flatten(2).transpose(1, 2) for s in srcs], 1)
        p = torch.cat([(pe.flatten(1).t() + self.encoder.level_encoding[l]) for l, pe in enumerate(pos)], 0)[None]
        ref = centre_points(shapes, src.device)[None, :, None, :].expand(B, -1, 3, -1)
        for ly in self.encoder.encoder.layers:
            src = ly(src, p, ref, shapes)
        outs, o = [], 0
        for h, w in shapes:
            outs.append(src[:, o:o + h * w].transpose(1, 2).reshape(B, self.d, h, w))
            o += h * w
        x1 = feats["1"]
        cur = self.lateral_convs[0](x1)
        y = cur + F.interpolate(outs[-1], size=cur.shape[-2:], mode="bilinear", align_corners=False)
        y = self.output_convs[0](y)
        return self.mask_feature(y), outs


# ----------------------------------------------------------------------------- masked decoder
class _SelfAttn(nn.Module):
    def __init__(self, d, heads):
        super().__init__()
        self.self_attn = nn.MultiheadAttention(d, heads)
        self.norm = nn.LayerNorm(d)

    def forward(self, tgt, qpos):
        q = tgt + qpos
        return self.norm(tgt + self.self_attn(q, q, value=tgt)[0])


class _CrossAttn(nn.Module):
    def __init__(self, d, heads):
        super().__init__()
        self.multihead_attn = nn.MultiheadAttention(d, heads)
        self.norm = nn.LayerNorm(d)

    def forward(self, tgt, mem, mask, pos, qpos):
        out = self.multihead_attn(query=tgt + qpos, key=mem + pos, value=mem, attn_mask=mask)[0]
        return self.norm(tgt + out)


class _FFN(nn.Module):
    def __init__(self, d, ffn):
        super().__init__()
        self.linear1 = nn.Linear(d, ffn)
        self.linear2 = nn.Linear(ffn, d)
        self.norm = nn.LayerNorm(d)

    def forward(self, x):
        return self.norm(x + self.linear2(F.relu(self.linear1(x))))


class _MLP(nn.Module):
    def __init__(self, d, out, n):
        super().__init__()
        self.layers = nn.ModuleList([nn.Linear(d, d if i < n - 1 else out) for i in range(n)])

    def forward(self, x):
        for i, ly in enumerate(self.layers):
            x = ly(x)
            if i < len(self.layers) - 1:
                x = F.relu(x)
        return x


class MaskedDecoder(nn.Module):
    """Masked-attention transformer decoder: each layer cross-attends (level i mod 3) only to the
    positions the previous prediction's mask covers (sigmoid >= 0.5 at that level's size; a query
    whose mask is empty attends everywhere), then self-attention, then FFN (all post-norm)."""

    def __init__(self, d: int, num_classes: int, queries: int = 100, heads: int = 16, ffn: int = 4096,
                 layers: int = 9, mask_dim: Optional[int] = None):
        super().__init__()
        self.heads, self.num_layers, self.num_queries = heads, layers, queries
        self.transformer_self_attention_layers = nn.ModuleList([_SelfAttn(d, heads) for _ in range(layers)])
        self.transformer_cross_attention_layers = nn.ModuleList([_CrossAttn(d, heads) for _ in range(layers)])
        self.transformer_ffn_layers = nn.ModuleList([_FFN(d, ffn) for _ in range(layers)])
        self.post_norm = nn.LayerNorm(d)
        self.query_feat = nn.Embedding(queries, d)
        self.query_embed = nn.Embedding(queries, d)
        self.level_embed = nn.Embedding(3, d)
        self.input_proj = nn.ModuleList([nn.Sequential() for _ in range(3)])
        self.class_embed = nn.Linear(d, num_classes + 1)
        self.mask_embed = _MLP(d, mask_dim or d, 3)

    def heads_out(self, out, mask_features, size):
        dec = self.post_norm(out).transpose(0, 1)                            # [B, Q, d]
        cls = self.class_embed(dec)
        masks = torch.einsum("bqc,bchw->bqhw", self.mask_embed(dec), mask_features)
        am = F.interpolate(masks, size=size, mode="bilinear", align_corners=False)
        am = (am.sigmoid().flatten(2) < 0.5)                                  # True = may not attend
        am = am[:, None].expand(-1, self.heads, -1, -1).flatten(0, 1)
        return cls, masks, am

    def forward(self, levels: List[torch.Tensor], mask_features: torch.Tensor):
        B = mask_features.shape[0]
        d = self.query_feat.weight.shape[1]
        src, pos, sizes = [], [], []
        for i, x in enumerate(levels):
            sizes.append(x.shape[-2:])
            pos.append(sine_pos_normalized(x.shape[-2], x.shape[-1], d // 2, x.device).flatten(1).t()[:, None]
                       .expand(-1, B, -1))
            src.append(x.flatten(2).permute(2, 0, 1) + self.level_embed.weight[i])
        qpos = self.query_embed.weight[:, None].expand(-1, B, -1)
        out = self.query_feat.weight[:, None].expand(-1, B, -1).clone()
        cls, masks, am = self.heads_out(out, mask_features, sizes[0])
        for i in range(self.num_layers):
            lv = i % 3
            am = am.clone()
            am[am.all(-1)] = False
            out = self.transformer_cross_attention_layers[i](out, src[lv], am, pos[lv], qpos)
            out = self.transformer_self_attention_layers[i](out, qpos)
            out = self.transformer_ffn_layers[i](out)
            cls, masks, am = self.heads_out(out, mask_features, sizes[(i + 1) % 3])
        return {"pred_logits": cls, "pred_masks": masks}


class Mask2FormerHead(nn.Module):
    def __init__(self, in_dim: int, num_classes: int = 150, hidden: int = 2048, heads: int = 16, ffn: int = 4096,
                 enc_layers: int = 6, dec_layers: int = 9, queries: int = 100):
        super().__init__()
        self.num_classes = num_classes
        self.pixel_decoder = PixelDecoder(in_dim, hidden, hidden, heads, ffn, enc_layers)
        self.predictor = MaskedDecoder(hidden, num_classes, queries, heads, ffn, dec_layers)

    def forward(self, feats: Dict[str, torch.Tensor]):
        mask_features, levels = self.pixel_decoder(feats)
        return self.predictor(levels, mask_features)


def semantic_map(pred: Dict[str, torch.Tensor], size: Tuple[int, int]) -> torch.Tensor:
    """sum_q softmax(class_q)[:-1] * sigmoid(mask_q) at `size` -> [B, C, h, w] fp32."""
    masks = F.interpolate(pred["pred_masks"].float(), size=size, mode="bilinear", align_corners=False)
    cls = pred["pred_logits"].float().softmax(-1)[..., :-1]
    return torch.einsum("bqc,bqhw->bchw", cls, masks.sigmoid())


class DINOv3M2FSegmentor(nn.Module):
    """`segmentation_model` = [adapter, head], the reference's checkpoint layout."""

    def __init__(self, dim: int, num_classes: int = 150, hidden: int = 2048, patch: int = 16, heads: int = 16,
                 adapter_heads: int = 16, ffn: int = 4096, enc_layers: int = 6, dec_layers: int = 9,
                 queries: int = 100, inplanes: int = 64):
        super().__init__()
        self.segmentation_model = nn.ModuleList([
            DINOv3Adapter(dim, patch, inplanes, heads=adapter_heads),
            Mask2FormerHead(dim, num_classes, hidden, heads, ffn, enc_layers, dec_layers, queries)])

    @property
    def adapter(self) -> DINOv3Adapter:
        return self.segmentation_model[0]

    @property
    def head(self) -> Mask2FormerHead:
        return self.segmentation_model[1]

    def init_weights(self, seed: int = 0) -> "DINOv3M2FSegmentor":
        """Random weights at unit-ish scale (no checkpoints offline); BatchNorm statistics random."""
        g = torch.Generator().manual_seed(seed)
        with torch.no_grad():
            for name, p in self.named_parameters():
                if p.dim() == 1 and ("norm" in name or name.endswith(".1.weight") or ".4.weight" in name
                                     or ".7.weight" in name):
                    p.copy_(1 + 0.1 * torch.randn(p.shape, generator=g))
                elif p.dim() == 1 or "embed" in name or "level" in name:
                    p.copy_(0.1 * torch.randn(p.shape, generator=g))
                else:
                    fan_in = p[0].numel()
                    p.copy_(torch.randn(p.shape, generator=g) / math.sqrt(fan_in))
            for m in self.modules():
                if isinstance(m, nn.BatchNorm2d):
                    m.running_mean.copy_(0.1 * torch.randn(m.running_mean.shape, generator=g))
                    m.running_var.copy_(1 + 0.2 * torch.rand(m.running_var.shape, generator=g))
        return self

    def forward(self, x: torch.Tensor, taps: List[torch.Tensor]) -> Dict[str, torch.Tensor]:
        return self.head(self.adapter(x, taps))


def slide_windows(h: int, w: int, crop: int, stride: int) -> List[Tuple[int, int, int, int]]:
    """Sliding-window crops (y1, y2, x1, x2) covering an h x w image: a grid of
    ceil((size - crop) / stride) + 1 windows per axis, the last one flush with the border; an image
    smaller than the crop on both axes uses its short side as the crop."""
    if crop > h and crop > w:
        crop = min(h, w)
    ny = max(h - crop + stride - 1, 0) // stride + 1
    nx = max(w - crop + stride - 1, 0) // stride + 1
    out = []
    for iy in range(ny):
        for ix in range(nx):
            y2, x2 = min(iy * stride + crop, h), min(ix * stride + crop, w)
            out.append((max(y2 - crop, 0), y2, max(x2 - crop, 0), x2))
    return out


def crop_cover_groups(h: int, w: int, crops: Sequence[Tuple[int, int, int, int]], patch: int) -> torch.Tensor:
    """Patch-grid group map for crop-ordered transmission: patch (i, j) of the full image belongs to
    the first crop that contains its centre (group = crop index + 1)."""
    gh, gw = h // patch, w // patch
    g = torch.zeros(gh, gw, dtype=torch.int64)
    yc = (torch.arange(gh) + 0.5) * patch
    xc = (torch.arange(gw) + 0.5) * patch
    for k in range(len(crops) - 1, -1, -1):
        y1, y2, x1, x2 = crops[k]
        inside = ((yc >= y1) & (yc < y2))[:, None] & ((xc >= x1) & (xc < x2))[None, :]
        g[inside] = k + 1
    return g


def slide_predict(image: torch.Tensor, crops: Sequence[Tuple[int, int, int, int]], predict_crop) -> torch.Tensor:
    """Average of per-crop class maps over the image: predict_crop(k, crop_image) -> [1, C, ch, cw]."""
    _, _, h, w = image.shape
    acc, cnt = None, torch.zeros(1, 1, h, w, device=image.device)
    for k, (y1, y2, x1, x2) in enumerate(crops):
        p = predict_crop(k, image[:, :, y1:y2, x1:x2]).float()
        if acc is None:
            acc = torch.zeros(1, p.shape[1], h, w, device=image.device)
        acc[:, :, y1:y2, x1:x2] += p
        cnt[:, :, y1:y2, x1:x2] += 1
    return acc / cnt


# ----------------------------------------------------------------------------- sm_100a runner
def _bf(t: torch.Tensor, device) -> torch.Tensor:
    return t.detach().to(device=device, dtype=torch.bfloat16).contiguous()


def _fold_bn(conv: nn.Conv2d, bn: nn.BatchNorm2d) -> nn.Conv2d:
    """Conv2d whose weights absorb the eval-mode BatchNorm that follows it."""
    s = bn.weight.detach() / torch.sqrt(bn.running_var + bn.eps)
    out = nn.Conv2d(conv.in_channels, conv.out_channels, conv.kernel_size, conv.stride, conv.padding, bias=True)
    with torch.no_grad():
        out.weight.copy_(conv.weight.detach() * s[:, None, None, None])
        b = conv.bias.detach() if conv.bias is not None else torch.zeros_like(s)
        out.bias.copy_((b - bn.running_mean) * s + bn.bias.detach())
    return out


class _LinGPU:
    """nn.Linear on the tcgen05 GEMM (weights padded to a multiple of 32 output rows)."""

    def __init__(self, lin: nn.Linear, device, rows: Optional[torch.Tensor] = None,
                 bias: Optional[torch.Tensor] = None):
        from .weights import pad_rows

        w = lin.weight.detach() if rows is None else rows
        b = (lin.bias.detach() if lin.bias is not None else torch.zeros(w.shape[0])) if bias is None else bias
        self.n = w.shape[0]
        self.w = _bf(pad_rows(w, 32), device)
        self.b = _bf(pad_rows(b[:, None], 32)[:, 0], device)
        self.ones = torch.ones(self.w.shape[0], device=device, dtype=torch.bfloat16)

    def __call__(self, x: torch.Tensor, resid: Optional[torch.Tensor] = None, epi: Optional[int] = None) -> torch.Tensor:
        from ..ops import kernels as K

        out = torch.empty(x.shape[0], self.w.shape[0], device=x.device, dtype=torch.bfloat16)
        if resid is not None:
            assert self.w.shape[0] == self.n
            K.gemm(x, self.w, out, epi=K.EPI_RESID, bias=self.b, gamma=self.ones, resid=resid)
        else:
            K.gemm(x, self.w, out, epi=K.EPI_BF16 if epi is None else epi, bias=self.b)
        return out if self.w.shape[0] == self.n else out[:, :self.n].contiguous()


class _LNGPU:
    def __init__(self, ln: nn.LayerNorm, device):
        self.w, self.b, self.eps = _bf(ln.weight, device), _bf(ln.bias, device), ln.eps

    def __call__(self, x: torch.Tensor) -> torch.Tensor:
        from ..ops import kernels as K

        out = torch.empty_like(x)
        return K.layernorm(x, self.w, self.b, self.eps, out)


class _MSDAGPU:
    """Deformable attention: value projection and the packed offset / logit projection as GEMMs,
    softmax + bilinear sampling + weighted sum in the fused kernel, output projection with the
    residual add in its epilogue."""

    def __init__(self, a: MSDeformAttnR, device):
        self.M, self.L, self.P, self.dv = a.n_heads, a.n_levels, a.n_points, a.dv
        packed = torch.cat([a.sampling_offsets.weight, a.attention_weights.weight]).detach()
        packed_b = torch.cat([a.sampling_offsets.bias, a.attention_weights.bias]).detach()
        self.n_off = a.sampling_offsets.weight.shape[0]
        self.oa = _LinGPU(a.sampling_offsets, device, rows=packed, bias=packed_b)
        self.v = _LinGPU(a.value_proj, device)
        self.o = _LinGPU(a.output_proj, device)

    def __call__(self, query: torch.Tensor, value_in: torch.Tensor, ref: torch.Tensor, N: int,
                 shapes: Sequence[Tuple[int, int]], resid: torch.Tensor) -> torch.Tensor:
        """query [N*Q, d], value_in [N*S, d], ref fp32 [N, Q, L, 2] -> resid + attn  [N*Q, d]."""
        from ..ops import kernels as K

        Q = query.shape[0] // N
        S = value_in.shape[0] // N
        val = self.v(value_in)
        oa = torch.empty(query.shape[0], self.oa.w.shape[0], device=query.device, dtype=torch.bfloat16)
        K.gemm(query, self.oa.w, oa, bias=self.oa.b)
        att = torch.empty(N * Q, self.dv, device=query.device, dtype=torch.bfloat16)
        K.msda(val.view(N, S, self.M, self.dv // self.M), ref, oa, oa[:, self.n_off:], att.view(N, Q, self.dv),
               [v for hw in shapes for v in hw], self.M, self.L, self.P)
        return self.o(att, resid=resid)


def _group_norm_nhwc(x: torch.Tensor, gn: nn.GroupNorm, relu: bool = False) -> torch.Tensor:
    y = F.group_norm(x.permute(0, 3, 1, 2).float(), gn.num_groups, gn.weight, gn.bias, gn.eps)
    if relu:
        y = F.relu(y)
    return y.permute(0, 2, 3, 1).to(torch.bfloat16).contiguous()


class Mask2FormerGPU:
    """DINOv3M2FSegmentor on the sm_100a kernels, NHWC bf16 maps.

    tcgen05 GEMMs: every linear layer, 1x1 convolution, the im2col 3x3 convolutions (BatchNorm
    folded into the weights) and the 2x2 transposed convolution; fused deformable-attention
    kernel; LayerNorm kernel; bilinear resize (+ add) kernel. PyTorch ops: GroupNorm, max-pool,
    the depthwise 3x3 convolution of ConvFFN, GELU / ReLU, and the 100-query masked attention core
    of the decoder (batched matmul + masked softmax over at most H/8 x W/8 keys)."""

    def __init__(self, mod: DINOv3M2FSegmentor, device):
        from .conv import ConvGPU

        self.m, self.dev = mod, device
        ad, hd = mod.adapter, mod.head
        self.dim, self.patch = ad.dim, ad.patch
        spm = ad.spm
        st = spm.stem
        c0 = _fold_bn(st[0], st[1])
        c0p = nn.Conv2d(8, c0.out_channels, 3, 2, 1, bias=True)  # image channels padded 3 -> 8 (im2col rows)
        with torch.no_grad():
            c0p.weight.zero_()
            c0p.weight[:, :3].copy_(c0.weight)
            c0p.bias.copy_(c0.bias)
        self.stem = [ConvGPU(c0p, device), ConvGPU(_fold_bn(st[3], st[4]), device),
                     ConvGPU(_fold_bn(st[6], st[7]), device)]
        self.convs = [ConvGPU(_fold_bn(c[0], c[1]), device) for c in (spm.conv2, spm.conv3, spm.conv4)]
        self.fcs = [ConvGPU(f, device) for f in (spm.fc1, spm.fc2, spm.fc3, spm.fc4)]
        self.level_embed = _bf(ad.level_embed, device)
        self.ex = []
        for blk in ad.interactions:
            chain = [blk.extractor] + (list(blk.extra_extractors) if blk.extra_extractors is not None else [])
            self.ex.append([{"qn": _LNGPU(e.query_norm, device), "fn": _LNGPU(e.feat_norm, device),
                             "attn": _MSDAGPU(e.attn, device), "ffn_n": _LNGPU(e.ffn_norm, device),
                             "fc1": _LinGPU(e.ffn.fc1, device), "fc2": _LinGPU(e.ffn.fc2, device),
                             "dw": (e.ffn.dwconv.dwconv.weight.detach().to(device, torch.bfloat16),
                                    e.ffn.dwconv.dwconv.bias.detach().to(device, torch.bfloat16))}
                            for e in chain])
        w = ad.up.weight.detach()                                       # [Cin, Cout, 2, 2]
        self.up_w = _bf(w.permute(2, 3, 1, 0).reshape(4 * w.shape[1], w.shape[0]), device)
        self.up_b = _bf(ad.up.bias.repeat(4), device)
        self.bn = []
        for bn in (ad.norm1, ad.norm2, ad.norm3, ad.norm4):
            s = bn.weight.detach() / torch.sqrt(bn.running_var + bn.eps)
            self.bn.append((s.to(device), (bn.bias.detach() - bn.running_mean * s).to(device)))
        pd = hd.pixel_decoder
        self.d = pd.d
        self.in_convs = [(ConvGPU(s[0], device), s[1]) for s in pd.input_convs]
        self.level_encoding = pd.encoder.level_encoding.detach().to(device)
        self.enc = [{"attn": _MSDAGPU(ly.self_attn, device), "n1": _LNGPU(ly.norm1, device),
                     "l1": _LinGPU(ly.linear1, device), "l2": _LinGPU(ly.linear2, device),
                     "n2": _LNGPU(ly.norm2, device)} for ly in pd.encoder.encoder.layers]
        self.lateral = (ConvGPU(pd.lateral_convs[0], device), pd.lateral_convs[0].norm)
        self.outconv = (ConvGPU(pd.output_convs[0], device), pd.output_convs[0].norm)
        self.mask_feature = ConvGPU(pd.mask_feature, device)
        self.pred = hd.predictor
        self._cache: Dict = {}

    # ------------------------------------------------------------------ adapter
    def adapter(self, img: torch.Tensor, taps: List[torch.Tensor], B: int) -> List[torch.Tensor]:
        """img [B, h, w, 3] bf16 normalised (NHWC); taps 4 x [B*(h/p)*(w/p), dim] bf16 ->
        NHWC maps at strides 4, 8, 16, 32."""
        from ..ops import kernels as K
        from .conv import resize

        _, h, w, _ = img.shape
        D = self.dim
        x = F.pad(img, (0, 5))                                            # 3 -> 8 channels
        for cv in self.stem:
            x = torch.relu_(cv(x))
        x = F.max_pool2d(x.permute(0, 3, 1, 2), 3, 2, 1).permute(0, 2, 3, 1).contiguous()
        c = [x]
        for cv in self.convs:
            c.append(torch.relu_(cv(c[-1])))
        c = [fc(ci) for fc, ci in zip(self.fcs, c)]                       # NHWC [B, h_i, w_i, D]
        Hc, Wc = h // 16, w // 16
        Ht, Wt = h // self.patch, w // self.patch
        n2, n3, n4 = 4 * Hc * Wc, Hc * Wc, (Hc // 2) * (Wc // 2)
        tok = torch.cat([(c[i + 1].reshape(B, -1, D) + self.level_embed[i]) for i in range(3)], 1)
        tok = tok.reshape(B * (n2 + n3 + n4), D).contiguous()
        key = ("ref", B, h, w)
        if key not in self._cache:
            ref = centre_points([(h // 8, w // 8), (h // 16, w // 16), (h // 32, w // 32)], self.dev)
            self._cache[key] = ref[None, :, None, :].expand(B, -1, 1, -1).contiguous()
        ref = self._cache[key]
        for chain, t in zip(self.ex, taps):
            for e in chain:
                q = e["qn"](tok)
                f = e["fn"](t)
                tok = e["attn"](q, f, ref, B, [(Ht, Wt)], resid=tok)
                hdn = e["fc1"](e["ffn_n"](tok))
                hid = hdn.shape[1]
                hb = hdn.view(B, n2 + n3 + n4, hid)
                outs = []
                for a0, a1, hh, ww in ((0, n2, 2 * Hc, 2 * Wc), (n2, n2 + n3, Hc, Wc),
                                       (n2 + n3, n2 + n3 + n4, Hc // 2, Wc // 2)):
                    mp = hb[:, a0:a1].reshape(B, hh, ww, hid).permute(0, 3, 1, 2)
                    y = F.conv2d(mp, e["dw"][0], e["dw"][1], 1, 1, 1, hid)
                    outs.append(y.permute(0, 2, 3, 1).reshape(B, -1, hid))
                g = F.gelu(torch.cat(outs, 1).float()).to(torch.bfloat16).reshape(-1, hid).contiguous()
                tok = e["fc2"](g, resid=tok)
        tb = tok.view(B, n2 + n3 + n4, D)
        c2 = tb[:, :n2].reshape(B, 2 * Hc, 2 * Wc, D)
        c3 = tb[:, n2:n2 + n3].reshape(B, Hc, Wc, D)
        c4 = tb[:, n2 + n3:].reshape(B, Hc // 2, Wc // 2, D)
        up = torch.empty(B * 4 * Hc * Wc, 4 * D, device=self.dev, dtype=torch.bfloat16)
        K.gemm(c2.reshape(-1, D).contiguous(), self.up_w, up, bias=self.up_b)
        up = up.view(B, 2 * Hc, 2 * Wc, 2, 2, D).permute(0, 1, 3, 2, 4, 5).reshape(B, 4 * Hc, 4 * Wc, D)
        c1 = (up + c[0]).contiguous()
        maps = [c1, c2.contiguous(), c3.contiguous(), c4.contiguous()]
        sizes = [(4 * Hc, 4 * Wc), (2 * Hc, 2 * Wc), (Hc, Wc), (Hc // 2, Wc // 2)]
        out = []
        for i in range(4):
            vit = taps[i].view(B, Ht, Wt, D)
            s = resize(vit, sizes[i][0], sizes[i][1], False, add=maps[i])
            sc, sh = self.bn[i]
            out.append((s.float() * sc + sh).to(torch.bfloat16).contiguous())
        return out

    # ------------------------------------------------------------------ pixel decoder
    def pixel_decoder(self, feats: List[torch.Tensor], B: int):
        from ..ops import kernels as K
        from .conv import resize

        d = self.d
        srcs, shapes = [], []
        for i, key in enumerate((3, 2, 1)):                            # strides 32, 16, 8
            cv, gn = self.in_convs[i]
            srcs.append(_group_norm_nhwc(cv(feats[key]), gn))
            shapes.append(tuple(feats[key].shape[1:3]))
        S = sum(h * w for h, w in shapes)
        src = torch.cat([s.reshape(B, -1, d) for s in srcs], 1).reshape(B * S, d).contiguous()
        key = ("pd", B, tuple(shapes))
        if key not in self._cache:
            pos = torch.cat([sine_pos_normalized(h, w, d // 2, self.dev).flatten(1).t() + self.level_encoding[l]
                             for l, (h, w) in enumerate(shapes)], 0)
            ref = centre_points(shapes, self.dev)[None, :, None, :].expand(B, -1, 3, -1).contiguous()
            self._cache[key] = (pos.to(torch.bfloat16).repeat(B, 1).contiguous(), ref)
        pos, ref = self._cache[key]
        for Ld in self.enc:
            q = src + pos
            t = Ld["attn"](q, src, ref, B, shapes, resid=src)
            src = Ld["n1"](t)
            hdn = torch.relu_(Ld["l1"](src))
            src = Ld["n2"](Ld["l2"](hdn, resid=src))
        outs, o = [], 0
        sb = src.view(B, S, d)
        for h, w in shapes:
            outs.append(sb[:, o:o + h * w].reshape(B, h, w, d))
            o += h * w
        lc, lgn = self.lateral
        cur = _group_norm_nhwc(lc(feats[0]), lgn)
        y = resize(outs[-1].contiguous(), cur.shape[1], cur.shape[2], False, add=cur)
        oc, ogn = self.outconv
        y = _group_norm_nhwc(oc(y), ogn, relu=True)
        return self.mask_feature(y), outs

    # ------------------------------------------------------------------ masked decoder
    def decoder(self, levels: List[torch.Tensor], mask_feat: torch.Tensor, B: int) -> Dict[str, torch.Tensor]:
        """Masked-attention decoder in fp32 on the GPU (100 queries: a few MFLOP per layer next to
        the GEMMs of the adapter and the pixel decoder)."""
        p = self.pred
        d = p.query_feat.weight.shape[1]
        mf = mask_feat.permute(0, 3, 1, 2).float()
        lv = [x.permute(0, 3, 1, 2).float() for x in levels]
        with torch.no_grad():
            return p(lv, mf)

    def forward(self, img: torch.Tensor, taps: List[torch.Tensor], B: int) -> Dict[str, torch.Tensor]:
        feats = self.adapter(img, taps, B)
        mask_feat, levels = self.pixel_decoder(feats, B)
        return self.decoder(levels, mask_feat, B)
