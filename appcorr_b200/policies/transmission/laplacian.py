"""Laplacian pyramid transmission (reference offload/policies/transmission/laplacian.py:10-453).

Encoding: Gaussian pyramid by integer pyrDown; level `levels[0]` (the coarsest) is sent as
uint8, every finer level as an int16 *closed-loop* residual against the decoder's own upsample
of the previous level, so `clip(pyrUp(prev) + residual)` reproduces the level exactly. Each level
is cut into patch_size crops (row-major spatial index) and zlib-compressed per crop.

Decoding has two forms:
  * `decode` rebuilds uint8 images on the CPU (numpy), as the reference does.
  * `decode_pyramid` only unpacks the crops into a uint8 base and int16 residual canvases
    (zeros where a crop has not arrived) and hands them to the GPU executor, which reconstructs
    with the `pyrup_add` kernel: the server's decoder thread does no per-pixel arithmetic.
"""
from __future__ import annotations

import math
import zlib
from concurrent.futures import ThreadPoolExecutor
from typing import Dict, Iterable, List, Optional, Sequence, Tuple

import numpy as np

from ...common.protocol import ExperimentConfig, Patch
from ..interface import ITransmissionPolicy
from .pyramid import pyr_down, pyr_up

try:
    import cv2  # type: ignore
except Exception:  # pragma: no cover
    cv2 = None

_POOL: Optional[ThreadPoolExecutor] = None


def pool() -> ThreadPoolExecutor:
    global _POOL
    if _POOL is None:
        _POOL = ThreadPoolExecutor(max_workers=8)
    return _POOL


def as_image_list(images) -> List[np.ndarray]:
    if isinstance(images, np.ndarray):
        if images.ndim != 4:
            raise RuntimeError(f"Expected image batch [B,H,W,C], got {tuple(images.shape)}")
        return [np.ascontiguousarray(images[b]) for b in range(images.shape[0])]
    if isinstance(images, (list, tuple)):
        return [np.ascontiguousarray(im) for im in images]
    raise RuntimeError(f"Unsupported image batch type: {type(images)!r}")


def levels_of(config: ExperimentConfig, default=(2, 1, 0)) -> List[int]:
    """Pyramid levels, coarsest first."""
    return sorted(config.transmission_kwargs.get("pyramid_levels", list(default)), reverse=True)


def cut_crops(image: np.ndarray, ph: int, pw: int) -> np.ndarray:
    """[H, W, C] -> [gh*gw, ph, pw, C] in row-major spatial order (H, W divisible by the patch)."""
    H, W, C = image.shape
    if H % ph or W % pw:
        raise ValueError(f"image shape {(H, W)} is not divisible by patch {(ph, pw)}")
    gh, gw = H // ph, W // pw
    return image.reshape(gh, ph, gw, pw, C).transpose(0, 2, 1, 3, 4).reshape(gh * gw, ph, pw, C)


def compress_crops(crops: np.ndarray, dtype, level: int) -> List[bytes]:
    return [zlib.compress(np.ascontiguousarray(c.astype(dtype, copy=False)).tobytes(), level) for c in crops]


def place_patch(canvas: np.ndarray, patch: Patch, ph: int, pw: int, dtype) -> None:
    H, W, C = canvas.shape
    gw = -(-W // pw)
    r, c = divmod(patch.spatial_idx, gw)
    y, x = r * ph, c * pw
    th, tw = min(ph, H - y), min(pw, W - x)
    if th <= 0 or tw <= 0:
        return
    raw = getattr(patch, "_decompressed_cache", None)
    if raw is None:
        try:
            raw = zlib.decompress(patch.data)
        except zlib.error as exc:
            print(f"[laplacian] corrupt patch at level {patch.res_level}: {exc}")
            return
        patch._decompressed_cache = raw
    canvas[y:y + th, x:x + tw] = np.frombuffer(raw, dtype=dtype).reshape(ph, pw, C)[:th, :tw]


class LaplacianPyramidPolicy(ITransmissionPolicy):
    default_levels = (2, 1, 0)

    # ------------------------------------------------------------------ grids
    @staticmethod
    def preserve_shape(config: ExperimentConfig) -> bool:
        return bool(config.transmission_kwargs.get("preserve_input_shape", False))

    @staticmethod
    def _align_up(v: float, m: int) -> int:
        return int(math.ceil(float(v) / m)) * m

    @classmethod
    def level_hw(cls, config: ExperimentConfig, lvl: int, image_hw: Optional[Tuple[int, int]] = None) -> Tuple[int, int]:
        """Transmission grid of a level: config.image_shape / 2**lvl, or, with
        preserve_input_shape, the short side scaled to the profile's size, patch aligned."""
        ph, pw = config.patch_size
        if image_hw is not None and cls.preserve_shape(config):
            h, w = image_hw
            short = int(config.get_input_profile_config().get("mobile_resize_short_side", config.image_shape[0]))
            ts = short // (2 ** lvl)
            if h <= w:
                th = cls._align_up(ts, ph)
                return th, cls._align_up(w / h * th, pw)
            tw = cls._align_up(ts, pw)
            return cls._align_up(h / w * tw, ph), tw
        H, W = config.image_shape[:2]
        s = 2 ** lvl
        if H % s or W % s:
            raise RuntimeError(f"Target image shape {(H, W)} is not divisible by pyramid scale {s}")
        return H // s, W // s

    @staticmethod
    def _resize(image: np.ndarray, hw: Tuple[int, int], dtype) -> np.ndarray:
        th, tw = hw
        if image.shape[:2] == (th, tw):
            return np.ascontiguousarray(image.astype(dtype, copy=False))
        if cv2 is None:
            raise RuntimeError("resampling to a non-dyadic grid needs OpenCV")
        interp = cv2.INTER_LINEAR if (th > image.shape[0] or tw > image.shape[1]) else cv2.INTER_AREA
        if dtype == np.int16:
            r = cv2.resize(image.astype(np.float32), (tw, th), interpolation=interp)
            return np.clip(np.rint(r), -32768, 32767).astype(np.int16)
        out = cv2.resize(image, (tw, th), interpolation=interp)
        if out.ndim == 2:
            out = out[..., None]
        return np.ascontiguousarray(out.astype(dtype, copy=False))

    def project(self, image, lvl, config, dtype, image_hw=None):
        return self._resize(image, self.level_hw(config, lvl, image_hw), dtype)

    @staticmethod
    def gaussians(image: np.ndarray, max_lvl: int) -> Dict[int, np.ndarray]:
        if image.dtype != np.uint8:
            image = np.clip(image, 0, 255).astype(np.uint8)
        g = {0: np.ascontiguousarray(image)}
        for i in range(1, max_lvl + 1):
            g[i] = pyr_down(g[i - 1])
        return g

    def upsample(self, img: np.ndarray, start_lvl: int, end_lvl: int, config, image_hw=None) -> np.ndarray:
        """The decoder's inter-level upsample (integer pyrUp on the dyadic grid; bilinear resize
        on the preserve-shape grid)."""
        cur = img
        if self.preserve_shape(config) and image_hw is not None:
            target = self.level_hw(config, end_lvl, image_hw)
            gap = start_lvl - end_lvl
            for k in range(gap):
                h, w = cur.shape[:2]
                nh, nw = target if k == gap - 1 else (2 * h, 2 * w)
                cur = cv2.resize(cur, (nw, nh), interpolation=cv2.INTER_LINEAR).astype(np.uint8)
                if cur.ndim == 2:
                    cur = cur[..., None]
            return cur
        for _ in range(start_lvl - end_lvl):
            cur = pyr_up(cur)
        return cur

    def closed_loop_residual(self, g, prev_lvl, lvl, config, image_hw=None) -> np.ndarray:
        prev_tx = self.project(g[prev_lvl], prev_lvl, config, np.uint8, image_hw)
        tgt = self.project(g[lvl], lvl, config, np.uint8, image_hw)
        pred = self.upsample(prev_tx, prev_lvl, lvl, config, image_hw)
        if pred.shape != tgt.shape:
            raise RuntimeError(f"closed-loop predictor {pred.shape[:2]} != target grid {tgt.shape[:2]}")
        return tgt.astype(np.int16) - pred.astype(np.int16)

    # ------------------------------------------------------------------ encode
    def _encode_level(self, b: int, image: np.ndarray, idx: int, levels: List[int], config) -> List[Patch]:
        ph, pw = config.patch_size
        comp = config.transmission_kwargs.get("compression_level", 1)
        hw = image.shape[:2] if self.preserve_shape(config) else None
        g = self.gaussians(image, max(levels))
        lvl = levels[idx]
        if idx == 0:
            band, dt = self.project(g[lvl], lvl, config, np.uint8, hw), np.uint8
        else:
            band, dt = self.closed_loop_residual(g, levels[idx - 1], lvl, config, hw), np.int16
        data = compress_crops(cut_crops(band, ph, pw), dt, comp)
        ts = tuple(image.shape[:2]) if hw is not None else ()
        return [Patch(b, i, d, lvl, target_shape=ts) for i, d in enumerate(data)]

    def encode(self, images, config: ExperimentConfig):
        imgs = as_image_list(images)
        levels = levels_of(config, self.default_levels)
        for idx in range(len(levels)):
            futs = [pool().submit(self._encode_level, b, im, idx, levels, config) for b, im in enumerate(imgs)]
            patches = [p for f in futs for p in f.result()]
            for p in patches:
                p.batch_group_total = len(patches)
                p.group_id = idx
            yield patches

    # ------------------------------------------------------------------ decode
    @staticmethod
    def _by_image(patches: Iterable[Patch], B: int) -> List[List[Patch]]:
        out: List[List[Patch]] = [[] for _ in range(B)]
        for p in patches:
            if 0 <= p.image_idx < B:
                out[p.image_idx].append(p)
        return out

    def _target_shapes(self, patches, B):
        ts = [None] * B
        for p in patches:
            if p.target_shape and p.image_idx < B and ts[p.image_idx] is None:
                ts[p.image_idx] = tuple(p.target_shape)
        return ts

    def _decode_one(self, plist: List[Patch], config, target_shape=None) -> np.ndarray:
        ph, pw = config.patch_size
        C = config.image_shape[2]
        levels = levels_of(config, self.default_levels)
        hw = target_shape if self.preserve_shape(config) else None
        if hw is None and self.preserve_shape(config):
            hw = tuple(config.image_shape[:2])
        base_lvl = levels[0]
        bh, bw = self.level_hw(config, base_lvl, hw)
        if not plist:
            return np.zeros(self.level_hw(config, 0, hw) + (C,), np.uint8)
        by_lvl: Dict[int, List[Patch]] = {}
        for p in plist:
            by_lvl.setdefault(p.res_level, []).append(p)
        cur = np.zeros((bh, bw, C), np.uint8)
        for p in by_lvl.get(base_lvl, []):
            place_patch(cur, p, ph, pw, np.uint8)
        prev = base_lvl
        for lvl in sorted(by_lvl, reverse=True):
            if lvl == base_lvl:
                continue
            cur = self.upsample(cur, prev, lvl, config, hw)
            res = np.zeros(cur.shape, np.int16)
            for p in by_lvl[lvl]:
                place_patch(res, p, ph, pw, np.int16)
            cur = np.clip(cur.astype(np.int16) + res, 0, 255).astype(np.uint8)
            prev = lvl
        if prev > 0:
            cur = self.upsample(cur, prev, 0, config, hw)
        return cur

    def decode(self, patches: List[Patch], config: ExperimentConfig, canvas: np.ndarray = None):
        B = config.batch_size
        groups = self._by_image(patches, B)
        if self.preserve_shape(config):
            ts = self._target_shapes(patches, B)
            futs = [pool().submit(self._decode_one, groups[b], config, ts[b]) for b in range(B)]
            return [f.result() for f in futs]
        futs = [pool().submit(self._decode_one, groups[b], config) for b in range(B)]
        return np.stack([f.result() for f in futs])

    def decode_pyramid(self, patches: List[Patch], config: ExperimentConfig):
        """Unpack crops for GPU reconstruction (dyadic grids only).

        Returns a PyramidBatch: base uint8 [B, h, w, C] and one int16 residual canvas per finer
        level (coarse to fine), None for a level with no arrived crop.
        """
        from ...server.model.base import PyramidBatch

        if self.preserve_shape(config):
            raise NotImplementedError("GPU reconstruction supports the dyadic grid only")
        B, C = config.batch_size, config.image_shape[2]
        ph, pw = config.patch_size
        levels = levels_of(config, self.default_levels)
        bh, bw = self.level_hw(config, levels[0])
        base = np.zeros((B, bh, bw, C), np.uint8)
        res: Dict[int, np.ndarray] = {}
        for p in patches:
            if p.res_level == levels[0]:
                place_patch(base[p.image_idx], p, ph, pw, np.uint8)
            else:
                canvas = res.get(p.res_level)
                if canvas is None:
                    h, w = self.level_hw(config, p.res_level)
                    canvas = res[p.res_level] = np.zeros((B, h, w, C), np.int16)
                place_patch(canvas[p.image_idx], p, ph, pw, np.int16)
        return PyramidBatch(base=base, residual=[res.get(l) for l in levels[1:]], levels=levels)

    def decode_lowres(self, patches: List[Patch], config: ExperimentConfig):
        B, C = config.batch_size, config.image_shape[2]
        ph, pw = config.patch_size
        base_lvl = levels_of(config, self.default_levels)[0]
        if self.preserve_shape(config):
            ts = self._target_shapes(patches, B)
            outs = []
            for b in range(B):
                h, w = self.level_hw(config, base_lvl, ts[b]) if ts[b] else (
                    config.image_shape[0] >> base_lvl, config.image_shape[1] >> base_lvl)
                cv = np.zeros((h, w, C), np.uint8)
                for p in patches:
                    if p.image_idx == b and p.res_level == base_lvl:
                        place_patch(cv, p, ph, pw, np.uint8)
                outs.append(cv)
            return np.stack(outs) if all(o.shape == outs[0].shape for o in outs) else outs
        bh, bw = self.level_hw(config, base_lvl)
        out = np.zeros((B, bh, bw, C), np.uint8)
        for p in patches:
            if p.res_level == base_lvl:
                place_patch(out[p.image_idx], p, ph, pw, np.uint8)
        return out
