"""Window-aligned progressive Laplacian variants (reference coco_window_progressive.py:13-318,
ade20k_window_progressive.py:9-123, nyu_appcorr_progressive.py:15-205, vggt_laplacian.py:58-271).

* COCOWindowProgressiveLaplacianPolicy: residual groups are the 3x3 detector windows
  (`block_grid` with 9 groups), so each group corrects exactly one window.
* ADE20KWindowProgressiveLaplacianPolicy ("crop_cover"): each residual crop goes to the first
  sliding segmentation crop (server_crop_size / server_stride of the input profile) that covers
  it; the group count is the per-image crop count, carried in `num_correction_groups`.
* NYUAppCorr* and VGGTLaplacian: the progressive policy on the model's canvas; VGGT's group
  count is `correction_groups`.
"""
from __future__ import annotations

from typing import List

import numpy as np

from ...common.protocol import ExperimentConfig
from .progressive import ProgressiveLPyramidPolicy, assign_groups


def slide_crops(h: int, w: int, crop: int, stride: int) -> List[tuple]:
    """(y1, y2, x1, x2) sliding windows in the order the segmentor visits them."""
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


class COCOWindowProgressiveLaplacianPolicy(ProgressiveLPyramidPolicy):
    def num_groups(self, config, images) -> int:
        return int(config.transmission_kwargs.get("num_window_groups", 9))

    def encode(self, images, config: ExperimentConfig):
        tk = dict(config.transmission_kwargs)
        tk.setdefault("grouping_strategy", "block_grid")
        tk["num_groups"] = self.num_groups(config, images)
        cfg = _with_tx(config, tk)
        yield from super().encode(images, cfg)


class ADE20KWindowProgressiveLaplacianPolicy(ProgressiveLPyramidPolicy):
    def encode(self, images, config: ExperimentConfig):
        prof = config.get_input_profile_config()
        crop = int(prof.get("server_crop_size", 512))
        stride = int(prof.get("server_stride", 341))
        H, W = config.image_shape[:2]
        crops = slide_crops(H, W, crop, stride)
        n = len(crops)
        tk = dict(config.transmission_kwargs)
        tk["grouping_strategy"] = "crop_cover"
        tk["num_groups"] = n
        cfg = _with_tx(config, tk)
        self._crops = crops
        for group in super().encode(images, cfg):
            for p in group:
                p.num_correction_groups = n
            yield group


def _crop_cover_groups(items, crops, ph, pw, level_scale):
    out = np.zeros(len(items), dtype=int)
    for k, it in enumerate(items):
        cy = (it["row"] * ph + ph // 2) * level_scale
        cx = (it["col"] * pw + pw // 2) * level_scale
        for g, (y1, y2, x1, x2) in enumerate(crops, start=1):
            if y1 <= cy < y2 and x1 <= cx < x2:
                out[k] = g
                break
    return out


def _assign_with_crop_cover(strategy, items, num_groups, config=None, rng=None):
    if strategy == "crop_cover":
        prof = config.get_input_profile_config()
        H, W = config.image_shape[:2]
        crops = slide_crops(H, W, int(prof.get("server_crop_size", 512)), int(prof.get("server_stride", 341)))
        ph, pw = config.patch_size
        scale = 2 ** int(items[0]["res_level"]) if items else 1
        return _crop_cover_groups(items, crops, ph, pw, scale)
    return assign_groups(strategy, items, num_groups, config, rng)


class FixedModelGridMixin:
    """NYU depther transmission on the depther's fixed model grid (reference
    nyu_appcorr_progressive.py:15-84): input-shape preservation is always off, so every pyramid
    level is cut on config.image_shape / 2**level, and whatever a decode produces is resized to
    config.image_shape (area interpolation when shrinking, bilinear when enlarging)."""

    @staticmethod
    def preserve_shape(config: ExperimentConfig) -> bool:
        return False

    @staticmethod
    def model_hw(config: ExperimentConfig):
        return int(config.image_shape[0]), int(config.image_shape[1])

    @staticmethod
    def to_model_grid(image: np.ndarray, h: int, w: int) -> np.ndarray:
        import cv2

        image = np.ascontiguousarray(image)
        if image.shape[:2] == (h, w):
            return image
        interp = cv2.INTER_LINEAR if (h > image.shape[0] or w > image.shape[1]) else cv2.INTER_AREA
        return np.ascontiguousarray(cv2.resize(image, (w, h), interpolation=interp))

    def fit_decoded(self, decoded, config: ExperimentConfig):
        h, w = self.model_hw(config)
        if isinstance(decoded, list):
            out = []
            for item in decoded:
                if isinstance(item, dict) and item.get("image") is not None:
                    item = dict(item)
                    item["image"] = self.to_model_grid(item["image"], h, w)
                elif isinstance(item, np.ndarray):
                    item = self.to_model_grid(item, h, w)
                out.append(item)
            return out
        if isinstance(decoded, np.ndarray) and decoded.ndim == 4 and decoded.shape[1:3] != (h, w):
            return np.stack([self.to_model_grid(im, h, w) for im in decoded])
        return decoded

    def decode(self, patches, config: ExperimentConfig, canvas=None):
        return self.fit_decoded(super().decode(patches, config, canvas=canvas), config)


class NYUAppCorrProgressiveLaplacianPolicy(FixedModelGridMixin, ProgressiveLPyramidPolicy):
    """Progressive Laplacian NYU transmission decoded onto the fixed model grid."""


class VGGTLaplacianPolicy(ProgressiveLPyramidPolicy):
    def num_groups(self, config, images) -> int:
        return max(1, int(config.transmission_kwargs.get("correction_groups", 1)))


def _with_tx(config: ExperimentConfig, tk: dict) -> ExperimentConfig:
    import copy

    cfg = copy.copy(config)
    cfg.transmission_kwargs = tk
    return cfg
