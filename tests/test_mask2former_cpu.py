"""Mask2Former segmentor (adapter + pixel decoder + masked-attention decoder): fp32 oracle on CPU.

When the reference package is installed next to the repository (baseline/_ref), its own modules
are built at a small width, their weights are loaded into ours by name (strict), and the outputs
are compared: this pins both the checkpoint layout and the arithmetic.
"""
import os
import sys

import pytest
import torch

from appcorr_b200.models.mask2former import (DINOv3M2FSegmentor, crop_cover_groups, semantic_map,
                                             slide_windows)

REF = os.path.join(os.path.dirname(os.path.dirname(os.path.abspath(__file__))), "baseline", "_ref",
                   "appcorr", "models")


def _small(seed=0):
    torch.manual_seed(seed)
    return DINOv3M2FSegmentor(dim=64, num_classes=7, hidden=64, heads=4, adapter_heads=4, ffn=96, enc_layers=2,
                              dec_layers=3, queries=10, inplanes=16).init_weights(seed).eval()


def _inputs(B=1, h=64, w=96, dim=64, patch=16, seed=1):
    g = torch.Generator().manual_seed(seed)
    x = torch.randn(B, 3, h, w, generator=g)
    taps = [torch.randn(B, (h // patch) * (w // patch), dim, generator=g) for _ in range(4)]
    return x, taps


def test_oracle_shapes():
    m = _small()
    x, taps = _inputs()
    with torch.no_grad():
        feats = m.adapter(x, taps)
        assert feats["1"].shape == (1, 64, 16, 24) and feats["4"].shape == (1, 64, 2, 3)
        out = m.head(feats)
        assert out["pred_logits"].shape == (1, 10, 8) and out["pred_masks"].shape == (1, 10, 16, 24)
        sem = semantic_map(out, (64, 96))
    assert sem.shape == (1, 7, 64, 96) and torch.isfinite(sem).all()


def test_slide_windows_cover():
    crops = slide_windows(896, 1200, 896, 596)
    assert crops == [(0, 896, 0, 896), (0, 896, 304, 1200)]
    crops = slide_windows(1000, 1300, 896, 596)
    assert len(crops) == 4 and crops[-1] == (104, 1000, 404, 1300)
    g = crop_cover_groups(1000, 1296, crops, 16)
    assert g.min() >= 1 and g.max() == len(crops)
    assert slide_windows(300, 400, 896, 596) == [(0, 300, 0, 300), (0, 300, 100, 400)]


def _ref_modules(dim, hidden, classes, patch):
    if not os.path.isdir(REF):
        pytest.skip("reference package not installed")
    if REF not in sys.path:
        sys.path.insert(0, REF)
    from dinov3.eval.segmentation.models.backbone.dinov3_adapter import DINOv3_Adapter
    from dinov3.eval.segmentation.models.heads.mask2former_head import Mask2FormerHead

    class FakeBackbone(torch.nn.Module):
        def __init__(self):
            super().__init__()
            self.embed_dim, self.patch_size, self.taps = dim, patch, None

        def get_intermediate_layers(self, x, n, return_class_token=True):
            return [(t, t[:, :1]) for t in self.taps]

    return FakeBackbone, DINOv3_Adapter, Mask2FormerHead


def test_matches_reference_modules():
    """Same weights, same inputs: our adapter + head reproduce the reference's modules."""
    dim, hidden, C, patch = 64, 64, 7, 16
    FakeBackbone, Adapter, Head = _ref_modules(dim, hidden, C, patch)
    import torch.nn as nn

    torch.manual_seed(0)
    bb = FakeBackbone()
    ra = Adapter(bb, interaction_indexes=[0, 1, 2, 3], conv_inplane=16, deform_num_heads=4, with_cp=False).eval()
    rh = Head({"1": [dim, 0, 0, 4], "2": [dim, 0, 0, 8], "3": [dim, 0, 0, 16], "4": [dim, 0, 0, 32]},
              hidden_dim=hidden, num_classes=C).eval()
    # the reference head's widths are fixed (16 heads, FFN 4096, 6 + 9 layers, 100 queries)
    m = DINOv3M2FSegmentor(dim=dim, num_classes=C, hidden=hidden, heads=16, adapter_heads=4, ffn=4096,
                           enc_layers=6, dec_layers=9, queries=100, inplanes=16).init_weights(3).eval()
    # SyncBatchNorm -> BatchNorm2d so the reference runs on CPU (same parameters and buffers)
    for mod in list(ra.modules()):
        for name, ch in list(mod.named_children()):
            if isinstance(ch, nn.SyncBatchNorm):
                bn = nn.BatchNorm2d(ch.num_features, eps=ch.eps)
                bn.load_state_dict(ch.state_dict())
                bn.eval()
                setattr(mod, name, bn)
    ours = m.state_dict()
    ref_sd = {k: v for k, v in ra.state_dict().items() if not k.startswith("backbone.")}
    ref_sd = {**{f"segmentation_model.0.{k}": v for k, v in ref_sd.items()},
              **{f"segmentation_model.1.{k}": v for k, v in rh.state_dict().items()}}
    assert set(ref_sd) == set(ours), (sorted(set(ref_sd) ^ set(ours)))[:10]
    for k in ours:
        assert ref_sd[k].shape == ours[k].shape, k
    # random (non-degenerate) weights into the reference, then ours <- reference
    g = torch.Generator().manual_seed(5)
    with torch.no_grad():
        for k, v in ref_sd.items():
            if v.dtype.is_floating_point:
                if "running_var" in k:
                    v.copy_(1 + 0.2 * torch.rand(v.shape, generator=g))
                elif v.dim() == 1:
                    v.copy_((1 if ("norm" in k and k.endswith("weight")) else 0) + 0.1 * torch.randn(v.shape, generator=g))
                else:
                    v.copy_(torch.randn(v.shape, generator=g) / max(v[0].numel(), 1) ** 0.5)
    m.load_state_dict(ref_sd, strict=True)
    x, taps = _inputs(h=64, w=64, dim=dim)
    bb.taps = taps
    with torch.no_grad():
        rf = ra(x)
        of = m.adapter(x, taps)
        for key in ("1", "2", "3", "4"):
            err = (rf[key] - of[key]).abs().max().item() / rf[key].abs().max().item()
            assert err < 1e-4, (key, err)
        ro = rh(rf)
        oo = m.head(of)
    for key in ("pred_logits", "pred_masks"):
        err = (ro[key] - oo[key]).abs().max().item() / ro[key].abs().max().item()
        assert err < 1e-3, (key, err)
