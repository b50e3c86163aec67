"""Mask2Former-style segmentation head on the ViT backbone: multi-scale deformable-attention pixel
decoder + query decoder + mask classification.

Reference: appcorr/models/dinov3/eval/segmentation/models/heads/{pixel_decoder.py,
mask2former_head.py, mask2former_transformer_decoder.py} and utils/ms_deform_attn.py (module
parameters `sampling_offsets`, `attention_weights`, `value_proj`, `output_proj`, forward
:159-222). Differences by design: the multi-scale input is built from the final patch features
(strided average pooling) instead of the DINOv3 adapter's four intermediate layers, and the query
decoder is the DETR-style decoder of models/detr.py (self-attention, cross-attention to the pixel
decoder memory, FFN) instead of masked attention; class and mask predictions, and the semantic
map = sum_q softmax(class_q)[:, :-1] * sigmoid(mask_q), follow Mask2Former.

`msda_reference` is the fp32 oracle of the deformable sampling (grid_sample, zeros padding,
align_corners=False); `MSDeformAttnGPU` runs value projection and the packed offset / logit
projection as GEMMs and the fused softmax + sampling + weighted sum as one kernel (csrc/msda.cu).
"""
from __future__ import annotations

import math
from typing import Dict, List, Optional, Sequence, Tuple

import torch
import torch.nn.functional as F
from torch import nn

from ..ops import kernels as K
from .detr import DetrDecoder, DetrDecoderGPU, sine_pos_embed
from .weights import pad_rows


def msda_reference(value: torch.Tensor, shapes: Sequence[Tuple[int, int]], loc: torch.Tensor,
                   weights: torch.Tensor) -> torch.Tensor:
    """value [N, S, M, Dh], loc [N, Q, M, L, P, 2] in [0, 1], weights [N, Q, M, L, P] -> [N, Q, M*Dh]."""
    N, S, M, Dh = value.shape
    _, Q, _, L, P, _ = loc.shape
    vals = value.split([h * w for h, w in shapes], dim=1)
    grids = 2 * loc - 1
    out = 0
    for l, (h, w) in enumerate(shapes):
        v = vals[l].flatten(2).transpose(1, 2).reshape(N * M, Dh, h, w)
        g = grids[:, :, :, l].transpose(1, 2).flatten(0, 1)                  # [N*M, Q, P, 2]
        smp = F.grid_sample(v.float(), g.float(), mode="bilinear", padding_mode="zeros", align_corners=False)
        wl = weights[:, :, :, l].transpose(1, 2).flatten(0, 1)[:, None]       # [N*M, 1, Q, P]
        out = out + (smp * wl).sum(-1)                                        # [N*M, Dh, Q]
    return out.view(N, M * Dh, Q).transpose(1, 2).contiguous()


class MSDeformAttn(nn.Module):
    def __init__(self, d_model: int = 256, n_levels: int = 3, n_heads: int = 8, n_points: int = 4):
        super().__init__()
        self.d_model, self.n_levels, self.n_heads, self.n_points = d_model, n_levels, n_heads, n_points
        self.sampling_offsets = nn.Linear(d_model, n_heads * n_levels * n_points * 2)
        self.attention_weights = nn.Linear(d_model, n_heads * n_levels * n_points)
        self.value_proj = nn.Linear(d_model, d_model)
        self.output_proj = nn.Linear(d_model, d_model)

    def forward(self, query, ref, value_in, shapes):
        N, Q, _ = query.shape
        M, L, P = self.n_heads, self.n_levels, self.n_points
        v = self.value_proj(value_in).view(N, value_in.shape[1], M, self.d_model // M)
        off = self.sampling_offsets(query).view(N, Q, M, L, P, 2)
        w = F.softmax(self.attention_weights(query).view(N, Q, M, L * P), -1).view(N, Q, M, L, P)
        norm = torch.tensor([[w_, h_] for h_, w_ in shapes], dtype=query.dtype, device=query.device)
        loc = ref[:, :, None, :, None, :] + off / norm[None, None, None, :, None, :]
        return self.output_proj(msda_reference(v, shapes, loc, w))


class PixelDecoderLayer(nn.Module):
    """Deformable-attention encoder layer (post-norm): x = LN(x + attn(x + pos)); x = LN(x + FFN(x))."""

    def __init__(self, d: int, heads: int, levels: int, points: int, ffn: int):
        super().__init__()
        self.self_attn = MSDeformAttn(d, levels, heads, points)
        self.norm1, self.norm2 = nn.LayerNorm(d), nn.LayerNorm(d)
        self.linear1, self.linear2 = nn.Linear(d, ffn), nn.Linear(ffn, d)

    def forward(self, x, pos, ref, shapes):
        x = self.norm1(x + self.self_attn(x + pos, ref, x, shapes))
        return self.norm2(x + self.linear2(F.relu(self.linear1(x))))


def level_shapes(gh: int, gw: int, levels: int) -> List[Tuple[int, int]]:
    return [(max(gh >> l, 1), max(gw >> l, 1)) for l in range(levels)]


def reference_points(shapes: Sequence[Tuple[int, int]], device) -> torch.Tensor:
    """[S, L, 2] normalised centre of every token, repeated for every level."""
    pts = []
    for h, w in shapes:
        y, x = torch.meshgrid((torch.arange(h, device=device, dtype=torch.float32) + 0.5) / h,
                              (torch.arange(w, device=device, dtype=torch.float32) + 0.5) / w, indexing="ij")
        pts.append(torch.stack([x.reshape(-1), y.reshape(-1)], -1))
    p = torch.cat(pts, 0)
    return p[:, None, :].expand(-1, len(shapes), -1).contiguous()


class M2FHead(nn.Module):
    """fp32 reference of the head: features [B, gh*gw, in_dim] -> per-class logits map [B, C, gh, gw]."""

    def __init__(self, in_dim: int, num_classes: int = 150, d: int = 256, heads: int = 8, levels: int = 3,
                 points: int = 4, enc_layers: int = 6, dec_layers: int = 6, queries: int = 100, ffn: int = 1024):
        super().__init__()
        self.d, self.levels, self.num_classes, self.queries = d, levels, num_classes, queries
        self.input_proj = nn.Linear(in_dim, d)
        self.level_embed = nn.Parameter(torch.zeros(levels, d))
        self.layers = nn.ModuleList([PixelDecoderLayer(d, heads, levels, points, ffn) for _ in range(enc_layers)])
        self.mask_proj = nn.Linear(d, d)
        self.decoder = DetrDecoder(d, d_model=d, heads=max(d // 64, 1), layers=dec_layers, ffn=ffn,
                                   num_queries=queries, num_classes=num_classes)
        self.mask_embed = nn.ModuleList([nn.Linear(d, d), nn.Linear(d, d), nn.Linear(d, d)])

    def init_weights(self, seed: int = 0) -> "M2FHead":
        g = torch.Generator().manual_seed(seed)
        with torch.no_grad():
            for name, p in self.named_parameters():
                if "norm" in name and name.endswith("weight"):
                    p.fill_(1.0)
                elif name.endswith("bias") or "level_embed" in name:
                    p.copy_(0.02 * torch.randn(p.shape, generator=g))
                else:
                    p.copy_(torch.randn(p.shape, generator=g) / math.sqrt(p.shape[-1]))
        return self

    def multiscale(self, feat: torch.Tensor, gh: int, gw: int) -> Tuple[torch.Tensor, List[Tuple[int, int]]]:
        B = feat.shape[0]
        x = self.input_proj(feat)                                                   # [B, gh*gw, d]
        img = x.transpose(1, 2).reshape(B, self.d, gh, gw)
        shapes = level_shapes(gh, gw, self.levels)
        toks = []
        for l, (h, w) in enumerate(shapes):
            lv = img if l == 0 else F.adaptive_avg_pool2d(img, (h, w))
            toks.append(lv.flatten(2).transpose(1, 2) + self.level_embed[l])
        return torch.cat(toks, 1), shapes

    def forward(self, feat: torch.Tensor, gh: int, gw: int) -> torch.Tensor:
        B = feat.shape[0]
        src, shapes = self.multiscale(feat, gh, gw)
        pos = torch.cat([sine_pos_embed(h, w, self.d, feat.device) for h, w in shapes], 0)[None]
        ref = reference_points(shapes, feat.device)[None].expand(B, -1, -1, -1)
        for ly in self.layers:
            src = ly(src, pos, ref, shapes)
        S0 = gh * gw
        mask_feat = self.mask_proj(src[:, :S0])                                   # [B, S0, d]
        out = self.decoder(src[:, :S0], (gh, gw))                                 # memory: finest level
        me = out["hidden"]
        for i, lin in enumerate(self.mask_embed):
            me = lin(me)
            if i < 2:
                me = F.relu(me)
        masks = torch.einsum("bqd,bsd->bqs", me, mask_feat)
        cls = out["pred_logits"].softmax(-1)[..., :-1]
        sem = torch.einsum("bqc,bqs->bcs", cls, masks.sigmoid())
        return sem.reshape(B, self.num_classes, gh, gw)


class M2FHeadGPU:
    """M2FHead with the sm_100a kernels: GEMMs with fused residual epilogues, LayerNorm, the fused
    deformable-attention kernel, the DETR-style decoder of models/detr.py and the upsample+argmax
    kernel. Level pooling, the positional terms and the two small softmax / sigmoid maps stay
    PyTorch ops."""

    def __init__(self, mod: M2FHead, device):
        bf = lambda t: t.detach().to(device=device, dtype=torch.bfloat16).contiguous()  # noqa: E731
        self.m, self.dev, self.d = mod, device, mod.d
        self.in_w, self.in_b = bf(mod.input_proj.weight), bf(mod.input_proj.bias)
        self.level_embed = bf(mod.level_embed)
        self.ones = torch.ones(mod.d, device=device, dtype=torch.bfloat16)
        self.L = []
        for ly in mod.layers:
            a = ly.self_attn
            packed = torch.cat([a.sampling_offsets.weight, a.attention_weights.weight]).detach()
            packed_b = torch.cat([a.sampling_offsets.bias, a.attention_weights.bias]).detach()
            n_off = a.sampling_offsets.weight.shape[0]
            self.L.append({
                "heads": a.n_heads, "points": a.n_points, "n_off": n_off,
                "oa_w": bf(pad_rows(packed, 32)), "oa_b": bf(pad_rows(packed_b[:, None], 32)[:, 0]),
                "v_w": bf(a.value_proj.weight), "v_b": bf(a.value_proj.bias),
                "o_w": bf(a.output_proj.weight), "o_b": bf(a.output_proj.bias),
                "n1": (bf(ly.norm1.weight), bf(ly.norm1.bias), ly.norm1.eps),
                "n2": (bf(ly.norm2.weight), bf(ly.norm2.bias), ly.norm2.eps),
                "l1_w": bf(ly.linear1.weight), "l1_b": bf(ly.linear1.bias),
                "l2_w": bf(ly.linear2.weight), "l2_b": bf(ly.linear2.bias)})
        self.mask_w, self.mask_b = bf(mod.mask_proj.weight), bf(mod.mask_proj.bias)
        self.decoder = DetrDecoderGPU(mod.decoder, device)
        self.me = [(bf(l.weight), bf(l.bias)) for l in mod.mask_embed]
        self._cache: Dict = {}

    def logits(self, feat: torch.Tensor, B: int, gh: int, gw: int) -> torch.Tensor:
        """feat: final-normed patch tokens [B*gh*gw, D] bf16 -> class map [B, C, gh, gw] (fp32)."""
        m, d = self.m, self.d
        S0 = gh * gw
        x = torch.empty(B * S0, d, device=self.dev, dtype=torch.bfloat16)
        K.gemm(feat, self.in_w, x, bias=self.in_b)
        shapes = level_shapes(gh, gw, m.levels)
        img = x.view(B, gh, gw, d).permute(0, 3, 1, 2)
        toks = [(img if l == 0 else F.adaptive_avg_pool2d(img.float(), (h, w)).to(torch.bfloat16))
                .flatten(2).transpose(1, 2) + self.level_embed[l] for l, (h, w) in enumerate(shapes)]
        S = sum(h * w for h, w in shapes)
        src = torch.cat(toks, 1).reshape(B * S, d).contiguous()
        key = (B, gh, gw)
        if key not in self._cache:
            pos = torch.cat([sine_pos_embed(h, w, d, self.dev) for h, w in shapes], 0).to(torch.bfloat16)
            ref = reference_points(shapes, self.dev)[None].expand(B, -1, -1, -1).contiguous()
            self._cache[key] = (pos.repeat(B, 1).contiguous(), ref)
        pos, ref = self._cache[key]
        q = torch.empty_like(src)
        val = torch.empty_like(src)
        att = torch.empty_like(src)
        tmp = torch.empty_like(src)
        h = torch.empty(B * S, self.L[0]["l1_w"].shape[0], device=self.dev, dtype=torch.bfloat16)
        sh = [v for hw in shapes for v in hw]
        for Ld in self.L:
            M, P = Ld["heads"], Ld["points"]
            oa = torch.empty(B * S, Ld["oa_w"].shape[0], device=self.dev, dtype=torch.bfloat16)
            torch.add(src, pos, out=q)
            K.gemm(src, Ld["v_w"], val, bias=Ld["v_b"])
            K.gemm(q, Ld["oa_w"], oa, bias=Ld["oa_b"])
            K.msda(val.view(B, S, M, d // M), ref, oa, oa[:, Ld["n_off"]:], att.view(B, S, d), sh, M, m.levels, P)
            K.gemm(att, Ld["o_w"], tmp, epi=K.EPI_RESID, bias=Ld["o_b"], gamma=self.ones, resid=src)
            K.layernorm(tmp, *Ld["n1"][:2], Ld["n1"][2], src)
            K.gemm(src, Ld["l1_w"], h, bias=Ld["l1_b"])
            torch.relu_(h)
            K.gemm(h, Ld["l2_w"], tmp, epi=K.EPI_RESID, bias=Ld["l2_b"], gamma=self.ones, resid=src)
            K.layernorm(tmp, *Ld["n2"][:2], Ld["n2"][2], src)
        fine = src.view(B, S, d)[:, :S0].reshape(B * S0, d)
        mask_feat = torch.empty(B * S0, d, device=self.dev, dtype=torch.bfloat16)
        K.gemm(fine, self.mask_w, mask_feat, bias=self.mask_b)
        out = self.decoder.forward(fine, B, (gh, gw))
        me = out["hidden"]
        for i, (w, b) in enumerate(self.me):
            nxt = torch.empty(me.shape[0], w.shape[0], device=self.dev, dtype=torch.bfloat16)
            K.gemm(me, w, nxt, bias=b)
            me = torch.relu_(nxt) if i < 2 else nxt
        Qn = m.queries
        C = m.num_classes
        cls = out["pred_logits"].float().softmax(-1)[..., :C]                      # [B, Q, C]
        sem = torch.empty(B, C, S0, device=self.dev, dtype=torch.float32)
        Qp = (Qn + 15) // 16 * 16
        masks = torch.empty(Qn, S0, device=self.dev, dtype=torch.float32)
        for b in range(B):  # masks = mask_embed . mask_feat^T, then sem = cls^T . sigmoid(masks)
            K.gemm(me[b * Qn:(b + 1) * Qn], mask_feat[b * S0:(b + 1) * S0], masks, epi=K.EPI_F32)
            prob = torch.zeros(S0, Qp, device=self.dev, dtype=torch.bfloat16)
            prob[:, :Qn] = masks.sigmoid().t()
            clsT = torch.zeros(C, Qp, device=self.dev, dtype=torch.bfloat16)
            clsT[:, :Qn] = cls[b].t()
            K.gemm(clsT, prob, sem[b], epi=K.EPI_F32)
        return sem.view(B, C, gh, gw)
