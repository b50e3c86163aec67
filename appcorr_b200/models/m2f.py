"""Multi-scale deformable attention: fp32 oracle and a plain module (the Mask2Former pixel decoder
and ViT adapter in models/mask2former.py build on them; the fused kernel is csrc/msda.cu).

Reference: appcorr/models/dinov3/eval/segmentation/models/utils/ms_deform_attn.py (module
parameters `sampling_offsets`, `attention_weights`, `value_proj`, `output_proj`, forward
:159-222; `ms_deform_attn_core_pytorch` is the same arithmetic as `msda_reference`).

`msda_reference` samples with grid_sample (zeros padding, align_corners=False).
"""
from __future__ import annotations

import math
from typing import Dict, List, Optional, Sequence, Tuple

import torch
import torch.nn.functional as F
from torch import nn



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
