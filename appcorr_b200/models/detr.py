"""DETR-style detection decoder on top of the ViT backbone.

Reference: the reference detector is PlainDETR (two-stage, 1500 queries, 91 classes;
appcorr/models/dinov3/hub/detectors.py:40-117). The configuration benchmarked here is the
DETR-style decoder of the build's BASELINE (6 layers, 300 queries, 80 classes), built from the
same pieces: a linear projection of the backbone's patch tokens to the decoder width (+ 2-D sine
position embedding), then per layer post-norm self-attention over the queries, cross-attention
from the queries to the memory tokens, and a ReLU FFN; class logits (num_classes + 1 for "no
object") and sigmoid (cx, cy, w, h) boxes from a 3-layer MLP.

`DetrDecoder` is the fp32 module (state dict / oracle); `DetrDecoderGPU` runs the same math with
the sm_100a GEMM, attention and LayerNorm kernels (head dim 64, BTHD layout).
"""
from __future__ import annotations

import math
from typing import Dict, Optional, Tuple

import torch
import torch.nn.functional as F
from torch import nn

from ..ops import kernels as K


def sine_pos_embed(h: int, w: int, dim: int, device=None, temperature: float = 10000.0) -> torch.Tensor:
    """[h*w, dim] 2-D sine embedding (half the channels for y, half for x)."""
    npf = dim // 4
    y, x = torch.meshgrid(torch.arange(h, device=device, dtype=torch.float32),
                          torch.arange(w, device=device, dtype=torch.float32), indexing="ij")
    y = (y + 0.5) / h * 2 * math.pi
    x = (x + 0.5) / w * 2 * math.pi
    t = temperature ** (torch.arange(npf, device=device, dtype=torch.float32) / npf)
    py, px = y.flatten()[:, None] / t, x.flatten()[:, None] / t
    return torch.cat([py.sin(), py.cos(), px.sin(), px.cos()], dim=1)


class DecoderLayer(nn.Module):
    def __init__(self, d: int, heads: int, ffn: int):
        super().__init__()
        self.self_attn = nn.MultiheadAttention(d, heads, batch_first=True)
        self.cross_attn = nn.MultiheadAttention(d, heads, batch_first=True)
        self.norm1, self.norm2, self.norm3 = nn.LayerNorm(d), nn.LayerNorm(d), nn.LayerNorm(d)
        self.linear1, self.linear2 = nn.Linear(d, ffn), nn.Linear(ffn, d)

    def forward(self, tgt, query_pos, memory, memory_pos):
        q = k = tgt + query_pos
        tgt = self.norm1(tgt + self.self_attn(q, k, tgt, need_weights=False)[0])
        tgt = self.norm2(tgt + self.cross_attn(tgt + query_pos, memory + memory_pos, memory, need_weights=False)[0])
        return self.norm3(tgt + self.linear2(F.relu(self.linear1(tgt))))


class DetrDecoder(nn.Module):
    def __init__(self, in_dim: int, d_model: int = 256, heads: int = 4, layers: int = 6, ffn: int = 1024,
                 num_queries: int = 300, num_classes: int = 80):
        super().__init__()
        self.d_model, self.heads, self.num_queries, self.num_classes = d_model, heads, num_queries, num_classes
        self.input_proj = nn.Linear(in_dim, d_model)
        self.query_embed = nn.Embedding(num_queries, 2 * d_model)  # [query_pos | tgt init]
        self.layers = nn.ModuleList([DecoderLayer(d_model, heads, ffn) for _ in range(layers)])
        self.class_embed = nn.Linear(d_model, num_classes + 1)
        self.bbox_embed = nn.ModuleList([nn.Linear(d_model, d_model), nn.Linear(d_model, d_model), nn.Linear(d_model, 4)])

    def forward(self, patch_tokens: torch.Tensor, hw: Tuple[int, int]) -> Dict[str, torch.Tensor]:
        B = patch_tokens.shape[0]
        mem = self.input_proj(patch_tokens.float())
        pos = sine_pos_embed(hw[0], hw[1], self.d_model, mem.device)[None].expand(B, -1, -1)
        qp, tgt = self.query_embed.weight.split(self.d_model, dim=1)
        qp, tgt = qp[None].expand(B, -1, -1), tgt[None].expand(B, -1, -1)
        for layer in self.layers:
            tgt = layer(tgt, qp, mem, pos)
        logits = self.class_embed(tgt)
        h = tgt
        for i, lin in enumerate(self.bbox_embed):
            h = lin(h)
            if i < 2:
                h = F.relu(h)
        return {"pred_logits": logits, "pred_boxes": h.sigmoid(), "hidden": tgt}


def postprocess(out: Dict[str, torch.Tensor], top_k: int = 100):
    """Top-k (score, label, box) per image over all queries x classes (sigmoid-free softmax
    scores excluding the no-object class)."""
    prob = out["pred_logits"].float().softmax(-1)[..., :-1]
    B, Q, C = prob.shape
    scores, idx = prob.reshape(B, -1).topk(min(top_k, Q * C), dim=1)
    q, labels = idx // C, idx % C
    boxes = out["pred_boxes"].float().gather(1, q[..., None].expand(-1, -1, 4))
    return scores, labels, boxes


class DetrDecoderGPU:
    """DetrDecoder forward with the sm_100a kernels. Attention projections are packed so each
    step is one GEMM; residual + post-norm use the resid epilogue (gamma = 1) + LayerNorm."""

    def __init__(self, mod: DetrDecoder, device):
        bf = lambda t: t.detach().to(device=device, dtype=torch.bfloat16).contiguous()  # noqa: E731
        d = mod.d_model
        if d % mod.heads or d // mod.heads not in (64, 128):
            raise ValueError("DetrDecoderGPU needs a head dim of 64 or 128")
        self.m, self.d, self.H, self.dev = mod, d, mod.heads, device
        self.in_w, self.in_b = bf(mod.input_proj.weight), bf(mod.input_proj.bias)
        self.qpos, self.tgt0 = (bf(t) for t in mod.query_embed.weight.split(d, dim=1))
        self.ones = torch.ones(d, device=device, dtype=torch.bfloat16)
        self.L = []
        for ly in mod.layers:
            sa, ca = ly.self_attn, ly.cross_attn
            self.L.append({
                "sa_qk_w": bf(sa.in_proj_weight[: 2 * d]), "sa_qk_b": bf(sa.in_proj_bias[: 2 * d]),
                "sa_v_w": bf(sa.in_proj_weight[2 * d:]), "sa_v_b": bf(sa.in_proj_bias[2 * d:]),
                "sa_o_w": bf(sa.out_proj.weight), "sa_o_b": bf(sa.out_proj.bias),
                "ca_q_w": bf(ca.in_proj_weight[:d]), "ca_q_b": bf(ca.in_proj_bias[:d]),
                "ca_k_w": bf(ca.in_proj_weight[d:2 * d]), "ca_k_b": bf(ca.in_proj_bias[d:2 * d]),
                "ca_v_w": bf(ca.in_proj_weight[2 * d:]), "ca_v_b": bf(ca.in_proj_bias[2 * d:]),
                "ca_o_w": bf(ca.out_proj.weight), "ca_o_b": bf(ca.out_proj.bias),
                "n": [(bf(n.weight), bf(n.bias), n.eps) for n in (ly.norm1, ly.norm2, ly.norm3)],
                "l1_w": bf(ly.linear1.weight), "l1_b": bf(ly.linear1.bias),
                "l2_w": bf(ly.linear2.weight), "l2_b": bf(ly.linear2.bias)})
        from .weights import pad_rows

        self.cls_w = bf(pad_rows(mod.class_embed.weight.detach(), 32))
        self.cls_b = bf(pad_rows(mod.class_embed.bias.detach()[:, None], 32)[:, 0])
        self.box = [(bf(l.weight), bf(l.bias)) for l in mod.bbox_embed[:2]]
        self.box_w3 = bf(pad_rows(mod.bbox_embed[2].weight.detach(), 32))
        self.box_b3 = bf(pad_rows(mod.bbox_embed[2].bias.detach()[:, None], 32)[:, 0])
        self._pos_cache: Dict = {}

    def _e(self, *shape, dtype=torch.bfloat16):
        return torch.empty(*shape, device=self.dev, dtype=dtype)

    def forward(self, patch_feat: torch.Tensor, B: int, hw: Tuple[int, int]) -> Dict[str, torch.Tensor]:
        """patch_feat: final-normed patch tokens [B*P, D_backbone] (bf16)."""
        d, H, Q = self.d, self.H, self.m.num_queries
        P = hw[0] * hw[1]
        mem = self._e(B * P, d)
        K.gemm(patch_feat, self.in_w, mem, bias=self.in_b)
        key = (B, hw)
        if key not in self._pos_cache:
            pos = sine_pos_embed(hw[0], hw[1], d, self.dev).to(torch.bfloat16).repeat(B, 1).contiguous()
            qpos = self.qpos.repeat(B, 1).contiguous()
            self._pos_cache[key] = (pos, qpos)
        pos, qpos = self._pos_cache[key]
        mem_pos = mem + pos  # keys of cross attention see memory + position
        tgt = self.tgt0.repeat(B, 1).contiguous()
        qk, v, q, o = self._e(B * Q, 2 * d), self._e(B * Q, d), self._e(B * Q, d), self._e(B * Q, d)
        kmem, vmem = self._e(B * P, d), self._e(B * P, d)
        tmp, h = self._e(B * Q, d), self._e(B * Q, self.L[0]["l1_w"].shape[0])
        for L in self.L:
            n1, n2, n3 = L["n"]
            tq = tgt + qpos
            K.gemm(tq, L["sa_qk_w"], qk, bias=L["sa_qk_b"])
            K.gemm(tgt, L["sa_v_w"], v, bias=L["sa_v_b"])
            K.attention(qk[:, :d], qk[:, d:], v, o, B=B, Tq=Q, Tk=Q, H=H, Dh=d // H)
            K.gemm(o, L["sa_o_w"], tmp, epi=K.EPI_RESID, bias=L["sa_o_b"], gamma=self.ones, resid=tgt)
            K.layernorm(tmp, n1[0], n1[1], n1[2], tgt)
            K.gemm(tgt + qpos, L["ca_q_w"], q, bias=L["ca_q_b"])
            K.gemm(mem_pos, L["ca_k_w"], kmem, bias=L["ca_k_b"])
            K.gemm(mem, L["ca_v_w"], vmem, bias=L["ca_v_b"])
            K.attention(q, kmem, vmem, o, B=B, Tq=Q, Tk=P, H=H, Dh=d // H)
            K.gemm(o, L["ca_o_w"], tmp, epi=K.EPI_RESID, bias=L["ca_o_b"], gamma=self.ones, resid=tgt)
            K.layernorm(tmp, n2[0], n2[1], n2[2], tgt)
            K.gemm(tgt, L["l1_w"], h, bias=L["l1_b"])
            h = torch.relu_(h)
            K.gemm(h, L["l2_w"], tmp, epi=K.EPI_RESID, bias=L["l2_b"], gamma=self.ones, resid=tgt)
            K.layernorm(tmp, n3[0], n3[1], n3[2], tgt)
        logits = self._e(B * Q, self.cls_w.shape[0], dtype=torch.float32)
        K.gemm(tgt, self.cls_w, logits, epi=K.EPI_F32, bias=self.cls_b)
        hb = tgt
        for w, b in self.box:
            nxt = self._e(B * Q, d)
            K.gemm(hb, w, nxt, bias=b)
            hb = torch.relu_(nxt)
        boxes = self._e(B * Q, self.box_w3.shape[0], dtype=torch.float32)
        K.gemm(hb, self.box_w3, boxes, epi=K.EPI_F32, bias=self.box_b3)
        C = self.m.num_classes + 1
        return {"pred_logits": logits[:, :C].view(B, Q, C), "pred_boxes": boxes[:, :4].sigmoid().view(B, Q, 4),
                "hidden": tgt}
