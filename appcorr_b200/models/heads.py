"""Task heads on top of the DINOv3 backbone, with their sm_100a execution paths.

* LinearSegHead  BatchNorm2d(D) + Conv2d(D, C, 1) on the final-normed patch grid
  (reference offload/server/model/dinov3_segmentor_linhead.py:186-246,749-851). On the GPU the
  eval-mode BN is folded into the 1x1 conv, which becomes one GEMM with an fp32 epilogue, and the
  bilinear upsample + argmax to pixel labels is one kernel.
* LinearClassifierHead  Linear(D * (1 + use_avgpool), num_classes) on [CLS | mean(patches)]
  (reference appcorr/models/dinov3/hub/classifiers.py:35,96; dinov3_classifier.py:665).
"""
from __future__ import annotations

from typing import Optional

import torch
from torch import nn

from ..ops import kernels as K
from .weights import fold_batchnorm_conv1x1, pad_rows


class LinearSegHead(nn.Module):
    def __init__(self, embed_dim: int, num_classes: int = 150):
        super().__init__()
        self.batchnorm_layer = nn.BatchNorm2d(embed_dim)
        self.conv = nn.Conv2d(embed_dim, num_classes, kernel_size=1)
        self.num_classes = num_classes

    def forward(self, patch_spatial: torch.Tensor) -> torch.Tensor:
        """[B, D, h, w] -> logits [B, C, h, w] (fp32)."""
        return self.conv(self.batchnorm_layer(patch_spatial.float()))

    def random_init(self, seed: int = 0) -> "LinearSegHead":
        g = torch.Generator().manual_seed(seed)
        with torch.no_grad():
            self.batchnorm_layer.weight.copy_(1.0 + 0.1 * torch.randn(self.batchnorm_layer.weight.shape, generator=g))
            self.batchnorm_layer.bias.copy_(0.1 * torch.randn(self.batchnorm_layer.bias.shape, generator=g))
            self.batchnorm_layer.running_mean.copy_(0.1 * torch.randn(self.batchnorm_layer.running_mean.shape, generator=g))
            self.batchnorm_layer.running_var.copy_(1.0 + 0.1 * torch.rand(self.batchnorm_layer.running_var.shape, generator=g))
            nn.init.normal_(self.conv.weight, std=0.02, generator=g)
            nn.init.zeros_(self.conv.bias)
        return self.eval()


class SegHeadGPU:
    """Fused GPU path of LinearSegHead: folded GEMM -> fp32 logits -> upsample + argmax."""

    def __init__(self, head: LinearSegHead, device):
        bn = head.batchnorm_layer
        w, b = fold_batchnorm_conv1x1(head.conv.weight, head.conv.bias, bn.weight, bn.bias, bn.running_mean,
                                      bn.running_var, bn.eps)
        self.num_classes = head.num_classes
        self.w = pad_rows(w, 32).to(device=device, dtype=torch.bfloat16).contiguous()
        self.b = pad_rows(b[:, None], 32)[:, 0].to(device=device, dtype=torch.bfloat16).contiguous()
        self.cpad = self.w.shape[0]
        self._logits: Optional[torch.Tensor] = None

    def logits(self, patch_feat: torch.Tensor, B: int, gh: int, gw: int) -> torch.Tensor:
        n = patch_feat.shape[0]
        if self._logits is None or self._logits.shape[0] != n:
            self._logits = torch.empty(n, self.cpad, device=patch_feat.device, dtype=torch.float32)
        K.gemm(patch_feat, self.w, self._logits, epi=K.EPI_F32, bias=self.b)
        return self._logits.view(B, gh, gw, self.cpad)

    def labels(self, patch_feat: torch.Tensor, B: int, gh: int, gw: int, H: int, W: int,
               out: Optional[torch.Tensor] = None) -> torch.Tensor:
        lg = self.logits(patch_feat, B, gh, gw)
        if out is None:
            out = torch.empty(B, H, W, device=patch_feat.device, dtype=torch.uint8)
        K.upsample_argmax(lg, self.num_classes, H, W, out)
        return out


class LinearClassifierHead(nn.Module):
    def __init__(self, embed_dim: int, num_classes: int = 1000, use_avgpool: bool = True):
        super().__init__()
        self.use_avgpool = use_avgpool
        self.linear = nn.Linear(embed_dim * (2 if use_avgpool else 1), num_classes)

    def forward(self, cls_tok: torch.Tensor, patch_tok: torch.Tensor) -> torch.Tensor:
        feat = torch.cat([cls_tok, patch_tok.mean(1)], dim=-1) if self.use_avgpool else cls_tok
        return self.linear(feat.float())


class ClassifierHeadGPU:
    def __init__(self, head: LinearClassifierHead, device):
        self.use_avgpool = head.use_avgpool
        self.num_classes = head.linear.out_features
        self.w = pad_rows(head.linear.weight.detach(), 32).to(device=device, dtype=torch.bfloat16).contiguous()
        self.b = pad_rows(head.linear.bias.detach()[:, None], 32)[:, 0].to(device=device, dtype=torch.bfloat16).contiguous()

    def logits(self, normed_tokens: torch.Tensor, B: int, N: int, n_prefix: int) -> torch.Tensor:
        """normed_tokens: final-normed [B*N, D] -> fp32 [B, num_classes]."""
        D = normed_tokens.shape[1]
        feat = torch.empty(B, D * (2 if self.use_avgpool else 1), device=normed_tokens.device, dtype=torch.bfloat16)
        rows = (torch.arange(B, device=normed_tokens.device, dtype=torch.int32) * N).contiguous()
        K.gather_rows(normed_tokens, rows, feat[:, :D])
        if self.use_avgpool:
            K.mean_rows(normed_tokens, B, N, n_prefix, feat[:, D:])
        out = torch.empty(B, self.w.shape[0], device=normed_tokens.device, dtype=torch.float32)
        K.gemm(feat, self.w, out, epi=K.EPI_F32, bias=self.b)
        return out[:, : self.num_classes]
