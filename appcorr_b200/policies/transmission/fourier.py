"""DCT-based transmission (reference offload/policies/transmission/fourier_progressive.py:38-490,
fourier_laplacian_hybrid.py:30-284, fourier_laplacian_progressive.py:13-250).

* FourierLaplacianProgressivePolicy: group 0 is a whole-image DCT low-pass base (the top-left
  keep_h x keep_w coefficients per channel, int16 with a per-payload scale); groups 1..N are
  pixel-domain int16 residual crops against the decoder's own reconstruction of that base (closed
  loop, so sending every group is lossless), grouped with the progressive strategies. The
  "Hybrid" and window-layout registry names use this class with their default grouping.
* FourierProgressiveTransmissionPolicy: per-crop 2-D DCT. Group 0 sends each crop's low-frequency
  block; groups 1..N send the remaining coefficients of each crop, grouped by crop.
"""
from __future__ import annotations

import math
import struct
import zlib
from typing import Dict, List, Tuple

import numpy as np

from ...common.protocol import ExperimentConfig, Patch
from .laplacian import as_image_list, cut_crops, place_patch
from .progressive import ProgressiveLPyramidPolicy, assign_groups, balanced_rank_groups, crop_energy

try:
    import cv2  # type: ignore
except Exception:  # pragma: no cover
    cv2 = None

_BASE_HDR = struct.Struct("<5if")   # c, h, w, keep_h, keep_w, scale


def dct_keep(config: ExperimentConfig, native_hw=None) -> Tuple[int, int]:
    levels = sorted(config.transmission_kwargs.get("pyramid_levels", [2, 0]), reverse=True)
    H, W = config.image_shape[:2]
    explicit = config.transmission_kwargs.get("dct_keep")
    ref_h, ref_w = native_hw if native_hw is not None else (H, W)
    if explicit == "window":
        f = int(config.transmission_kwargs.get("global_base_downscale", 3))
        return min(max(math.ceil(ref_h / f), 1), H), min(max(math.ceil(ref_w / f), 1), W)
    if explicit:
        return (int(explicit[0]), int(explicit[1])) if isinstance(explicit, (list, tuple)) else (int(explicit),) * 2
    s = 2 ** levels[0]
    return min(max(math.ceil(ref_h / s), 1), H), min(max(math.ceil(ref_w / s), 1), W)


def dct_base_encode(image: np.ndarray, kh: int, kw: int) -> Tuple[bytes, np.ndarray]:
    """-> (payload, uint8 reconstruction the decoder will compute from that payload)."""
    H, W, C = image.shape
    coef = np.stack([cv2.dct(np.ascontiguousarray(image[:, :, c], dtype=np.float32))[:kh, :kw] for c in range(C)])
    scale = float(np.abs(coef).max() / 32767.0) or 1.0
    q = np.clip(np.rint(coef / scale), -32768, 32767).astype(np.int16)
    payload = _BASE_HDR.pack(C, H, W, kh, kw, scale) + q.tobytes()
    return payload, dct_base_decode(payload)


def dct_base_decode(payload: bytes) -> np.ndarray:
    C, H, W, kh, kw, scale = _BASE_HDR.unpack(payload[:_BASE_HDR.size])
    q = np.frombuffer(payload[_BASE_HDR.size:], np.int16).reshape(C, kh, kw).astype(np.float32) * scale
    out = np.empty((H, W, C), np.float32)
    for c in range(C):
        full = np.zeros((H, W), np.float32)
        full[:kh, :kw] = q[c]
        out[:, :, c] = cv2.idct(full)
    return np.clip(np.rint(out), 0, 255).astype(np.uint8)


class FourierLaplacianProgressivePolicy(ProgressiveLPyramidPolicy):
    BASE_LEVEL = 99            # res_level tag of the DCT base patch
    default_strategy = "grid"

    def encode(self, images, config: ExperimentConfig):
        imgs = as_image_list(images)
        comp = config.transmission_kwargs.get("compression_level", 1)
        kh, kw = dct_keep(config, tuple(imgs[0].shape[:2]) if imgs else None)
        ph, pw = config.patch_size
        kind = self.mobile_pscore(config)
        base, preds = [], []
        for b, im in enumerate(imgs):
            payload, pred = dct_base_encode(im, kh, kw)
            preds.append(pred)
            base.append(Patch(b, 0, zlib.compress(payload, comp), self.BASE_LEVEL, 0))
        for p in base:
            p.batch_group_total = len(base)
        yield base
        if config.transmission_kwargs.get("base_only", False):
            return
        ng = self.num_groups(config, imgs)
        strategy = config.transmission_kwargs.get("grouping_strategy", self.default_strategy)
        crops = []
        for im, pred in zip(imgs, preds):
            res = im.astype(np.int16) - pred.astype(np.int16)
            gh, gw = res.shape[0] // ph, res.shape[1] // pw
            crops.append([{"spatial_idx": i, "res_level": 0, "grid_hw": (gh, gw), "row": i // gw, "col": i % gw,
                           "crop": c, "pscore": crop_energy(c)} for i, c in enumerate(cut_crops(res, ph, pw))])
        if strategy in ("energy_asc", "energy_desc", "uniform_diff"):
            vals = np.asarray([[it["pscore"] for it in items] for items in crops])
            gid = balanced_rank_groups(vals, ng, descending=strategy == "energy_desc")
        else:
            gid = [assign_groups(strategy, items, ng, config) for items in crops]
        groups: Dict[int, List[Patch]] = {}
        for b, items in enumerate(crops):
            for it, g in zip(items, gid[b]):
                if g > 0:
                    groups.setdefault(int(g), []).append(self._make_patch(b, it, g, config, kind, ()))
        for g in sorted(groups):
            for p in groups[g]:
                p.batch_group_total = len(groups[g])
            yield groups[g]

    def decode(self, patches: List[Patch], config: ExperimentConfig, canvas=None):
        B = config.batch_size
        H, W, C = config.image_shape
        ph, pw = config.patch_size
        out = np.zeros((B, H, W, C), np.uint8)
        res = np.zeros((B, H, W, C), np.int16)
        for p in patches:
            if p.res_level == self.BASE_LEVEL:
                rec = getattr(p, "_base_rec", None)
                if rec is None:
                    rec = p._base_rec = dct_base_decode(zlib.decompress(p.data))
                out[p.image_idx] = rec
            else:
                place_patch(res[p.image_idx], p, ph, pw, np.int16)
        return np.clip(out.astype(np.int16) + res, 0, 255).astype(np.uint8)

    def decode_lowres(self, patches, config):
        B = config.batch_size
        H, W, C = config.image_shape
        out = np.zeros((B, H, W, C), np.uint8)
        for p in patches:
            if p.res_level == self.BASE_LEVEL:
                out[p.image_idx] = dct_base_decode(zlib.decompress(p.data))
        return out


class FourierProgressiveTransmissionPolicy(ProgressiveLPyramidPolicy):
    """Per-crop DCT split into a low block (group 0) and the rest (groups >= 1)."""

    _HDR = struct.Struct("<3if")      # lo_h, lo_w, part(0 low / 1 high), scale

    def _low_hw(self, config):
        levels = sorted(config.transmission_kwargs.get("pyramid_levels", [2, 0]), reverse=True)
        ph, pw = config.patch_size
        s = 2 ** levels[0]
        return max(1, math.ceil(ph / s)), max(1, math.ceil(pw / s))

    @staticmethod
    def _q(a: np.ndarray) -> Tuple[np.ndarray, float]:
        scale = float(np.abs(a).max() / 32767.0) or 1.0
        return np.clip(np.rint(a / scale), -32768, 32767).astype(np.int16), scale

    def encode(self, images, config: ExperimentConfig):
        imgs = as_image_list(images)
        ph, pw = config.patch_size
        lh, lw = self._low_hw(config)
        comp = config.transmission_kwargs.get("compression_level", 1)
        ng = self.num_groups(config, imgs)
        strategy = config.transmission_kwargs.get("grouping_strategy", "grid")
        low, high = [], []
        for b, im in enumerate(imgs):
            cr = cut_crops(im, ph, pw).astype(np.float32)
            gw = im.shape[1] // pw
            items = []
            for i, c in enumerate(cr):
                coef = np.stack([cv2.dct(np.ascontiguousarray(c[:, :, ch])) for ch in range(c.shape[2])])
                lo, ls = self._q(coef[:, :lh, :lw])
                hi_mask = np.ones(coef.shape[1:], bool)
                hi_mask[:lh, :lw] = False
                hi, hs = self._q(coef[:, hi_mask])
                low.append(Patch(b, i, zlib.compress(self._HDR.pack(lh, lw, 0, ls) + lo.tobytes(), comp), 0, 0))
                items.append({"spatial_idx": i, "row": i // gw, "col": i % gw, "grid_hw": (im.shape[0] // ph, gw),
                              "payload": self._HDR.pack(lh, lw, 1, hs) + hi.tobytes(), "pscore": float((hi.astype(np.float32) ** 2).sum())})
            high.append(items)
        for p in low:
            p.batch_group_total = len(low)
        yield low
        groups: Dict[int, List[Patch]] = {}
        for b, items in enumerate(high):
            gid = assign_groups(strategy, items, ng, config)
            for it, g in zip(items, gid):
                if g > 0:
                    groups.setdefault(int(g), []).append(
                        Patch(b, it["spatial_idx"], zlib.compress(it["payload"], comp), 0, int(g), pscore_hint=it["pscore"]))
        for g in sorted(groups):
            for p in groups[g]:
                p.batch_group_total = len(groups[g])
            yield groups[g]

    def decode(self, patches: List[Patch], config: ExperimentConfig, canvas=None):
        B = config.batch_size
        H, W, C = config.image_shape
        ph, pw = config.patch_size
        coefs: Dict[Tuple[int, int], np.ndarray] = {}
        for p in patches:
            raw = zlib.decompress(p.data)
            lh, lw, part, scale = self._HDR.unpack(raw[:self._HDR.size])
            vals = np.frombuffer(raw[self._HDR.size:], np.int16).astype(np.float32) * scale
            coef = coefs.setdefault((p.image_idx, p.spatial_idx), np.zeros((C, ph, pw), np.float32))
            if part == 0:
                coef[:, :lh, :lw] = vals.reshape(C, lh, lw)
            else:
                m = np.ones((ph, pw), bool)
                m[:lh, :lw] = False
                coef[:, m] = vals.reshape(C, -1)
        out = np.zeros((B, H, W, C), np.uint8)
        gw = W // pw
        for (b, i), coef in coefs.items():
            r, c = divmod(i, gw)
            block = np.stack([cv2.idct(coef[ch]) for ch in range(C)], -1)
            out[b, r * ph:(r + 1) * ph, c * pw:(c + 1) * pw] = np.clip(np.rint(block), 0, 255).astype(np.uint8)
        return out
