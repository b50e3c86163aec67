"""Weight re-layouts done once at load time for the fused kernels.

The state dict keeps the DINOv3 key names and shapes (appcorr/models/dinov3/layers/block.py:
102-126, attention.py:107-111, ffn_layers.py:77-79); the runtime derives kernel-friendly copies:
  * SwiGLU w1 / w2 are interleaved in 128-row blocks so one GEMM tile holds matching rows of
    both and its epilogue can emit silu(x1) * x2 directly.
  * qkv bias is multiplied by its k-mask (LinearKMaskedBias, attention.py:39-49) once.
  * The linear segmentation head's BatchNorm (eval statistics) is folded into the 1x1 conv.
"""
from __future__ import annotations

from typing import Optional, Tuple

import torch

SWIGLU_BLOCK = 128


def pack_swiglu(w1: torch.Tensor, w2: torch.Tensor, b1: Optional[torch.Tensor], b2: Optional[torch.Tensor],
                block: int = SWIGLU_BLOCK) -> Tuple[torch.Tensor, Optional[torch.Tensor]]:
    """Interleave w1 / w2 rows in `block`-row blocks: a GEMM tile of 2 * block columns then holds
    matching gate and up columns (128 for the 256-wide bf16 / e4m3 tiles, 64 for NVFP4's 128)."""
    hd, k = w1.shape
    assert w2.shape == (hd, k) and hd % block == 0, f"SwiGLU hidden size must be a multiple of {block}"
    nb = hd // block
    w = torch.stack([w1.view(nb, block, k), w2.view(nb, block, k)], dim=1).reshape(2 * hd, k)
    b = None
    if b1 is not None:
        b = torch.stack([b1.view(nb, block), b2.view(nb, block)], dim=1).reshape(2 * hd)
    return w.contiguous(), (b.contiguous() if b is not None else None)


def unpack_swiglu(w: torch.Tensor, block: int = SWIGLU_BLOCK) -> Tuple[torch.Tensor, torch.Tensor]:
    two_hd = w.shape[0]
    rest = tuple(w.shape[1:])
    nb = two_hd // (2 * block)
    v = w.reshape((nb, 2, block) + rest)
    return v[:, 0].reshape((-1,) + rest), v[:, 1].reshape((-1,) + rest)


def repack_swiglu(w: torch.Tensor, b: Optional[torch.Tensor], block_from: int = SWIGLU_BLOCK,
                  block_to: int = 64) -> Tuple[torch.Tensor, Optional[torch.Tensor]]:
    """Change the w1 / w2 interleave block of a packed SwiGLU weight (and bias)."""
    w1, w2 = unpack_swiglu(w, block_from)
    b1 = b2 = None
    if b is not None:
        b1, b2 = unpack_swiglu(b, block_from)
    return pack_swiglu(w1, w2, b1, b2, block_to)


def fold_batchnorm_conv1x1(conv_w: torch.Tensor, conv_b: Optional[torch.Tensor], bn_w: torch.Tensor,
                           bn_b: torch.Tensor, bn_mean: torch.Tensor, bn_var: torch.Tensor, eps: float
                           ) -> Tuple[torch.Tensor, torch.Tensor]:
    """conv(BN(x)) == x @ W'^T + b' for eval-mode BN followed by a 1x1 conv."""
    w = conv_w.reshape(conv_w.shape[0], -1).float()
    s = bn_w.float() / torch.sqrt(bn_var.float() + eps)
    shift = bn_b.float() - bn_mean.float() * s
    w_f = w * s[None, :]
    b_f = w @ shift
    if conv_b is not None:
        b_f = b_f + conv_b.float()
    return w_f, b_f


def pad_rows(w: torch.Tensor, multiple: int) -> torch.Tensor:
    n = w.shape[0]
    pad = (-n) % multiple
    if pad == 0:
        return w
    return torch.cat([w, w.new_zeros((pad,) + tuple(w.shape[1:]))], dim=0)
