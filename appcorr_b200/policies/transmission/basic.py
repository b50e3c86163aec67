"""Single-shot transmission: raw crops, zlib crops, one compressed image
(reference offload/policies/transmission/raw.py:8-122, zlib.py:8-65, full_image.py:8-184)."""
from __future__ import annotations

import math
import struct
import zlib
from typing import Any, List

import numpy as np

from ...common.protocol import ExperimentConfig, Patch
from ..interface import ITransmissionPolicy
from .laplacian import cut_crops, pool

try:
    import cv2  # type: ignore
except Exception:  # pragma: no cover
    cv2 = None

_HDR = struct.Struct("<5i")  # h, w, c, target_h, target_w


def _short_side(config: ExperimentConfig) -> int:
    return int(config.get_input_profile_config().get("mobile_resize_short_side", min(config.image_shape[:2])))


def resize_short_side(image: np.ndarray, short: int, patch) -> np.ndarray:
    """Scale so the short side is `short` (patch aligned) keeping the aspect ratio."""
    h, w = image.shape[:2]
    ph, pw = patch
    up = lambda v, m: int(math.ceil(float(v) / m)) * m  # noqa: E731
    if h <= w:
        th = up(short, ph)
        tw = up(w / h * th, pw)
    else:
        tw = up(short, pw)
        th = up(h / w * tw, ph)
    if (h, w) == (th, tw):
        return np.ascontiguousarray(image)
    return np.ascontiguousarray(cv2.resize(image, (tw, th), interpolation=cv2.INTER_LINEAR))


def _split_item(item):
    if isinstance(item, dict):
        return item.get("image"), dict(item.get("metadata") or {})
    return item, {}


def _place(canvas: np.ndarray, idx: int, chunk: np.ndarray, ph: int, pw: int) -> None:
    gw = canvas.shape[1] // pw
    r, c = divmod(idx, gw)
    canvas[r * ph:(r + 1) * ph, c * pw:(c + 1) * pw] = chunk


class RawTransmissionPolicy(ITransmissionPolicy):
    def encode(self, images: Any, config: ExperimentConfig):
        if bool(config.transmission_kwargs.get("preserve_input_shape", False)):
            items = [images[b] for b in range(images.shape[0])] if isinstance(images, np.ndarray) else list(images)
            out = []
            for b, item in enumerate(items):
                img, meta = _split_item(item)
                img = resize_short_side(img, _short_side(config), config.patch_size)
                ts = meta.get("target_shape") or (0, 0)
                out.append(Patch(image_idx=b, spatial_idx=0, data=_HDR.pack(*img.shape, *ts) + img.tobytes()))
            yield out
            return
        ph, pw = config.patch_size
        out = []
        for b in range(images.shape[0]):
            for i, crop in enumerate(cut_crops(images[b], ph, pw)):
                out.append(Patch(image_idx=b, spatial_idx=i, data=crop.tobytes()))
        yield out

    def decode(self, patches: List[Patch], config: ExperimentConfig, canvas: np.ndarray = None):
        B = config.batch_size
        H, W, C = config.image_shape
        if bool(config.transmission_kwargs.get("preserve_input_shape", False)):
            outs = list(canvas) if isinstance(canvas, list) else [None] * B
            for p in patches:
                if p.spatial_idx != 0 or not p.data:
                    continue
                h, w, c, th, tw = _HDR.unpack(p.data[:_HDR.size])
                item = {"image": np.frombuffer(p.data[_HDR.size:], np.uint8).reshape(h, w, c).copy()}
                if th > 0 and tw > 0:
                    item["target_shape"] = (th, tw)
                outs[p.image_idx] = item
            return outs
        ph, pw = config.patch_size
        out = np.zeros((B, H, W, C), np.uint8) if canvas is None else canvas
        for p in patches:
            _place(out[p.image_idx], p.spatial_idx, np.frombuffer(p.data, np.uint8).reshape(ph, pw, C), ph, pw)
        return out


class ZlibTransmissionPolicy(ITransmissionPolicy):
    def encode(self, images: np.ndarray, config: ExperimentConfig):
        ph, pw = config.patch_size
        lvl = config.transmission_kwargs.get("compression_level", 1)
        out = []
        for b in range(images.shape[0]):
            for i, crop in enumerate(cut_crops(images[b], ph, pw)):
                out.append(Patch(image_idx=b, spatial_idx=i, data=zlib.compress(crop.tobytes(), lvl)))
        yield out

    def decode(self, patches: List[Patch], config: ExperimentConfig, canvas: np.ndarray = None):
        B = config.batch_size
        H, W, C = config.image_shape
        ph, pw = config.patch_size
        out = np.zeros((B, H, W, C), np.uint8) if canvas is None else canvas

        def one(p):
            try:
                _place(out[p.image_idx], p.spatial_idx,
                       np.frombuffer(zlib.decompress(p.data), np.uint8).reshape(ph, pw, C), ph, pw)
            except zlib.error as exc:
                print(f"[zlib] corrupt patch {p.spatial_idx}: {exc}")

        list(pool().map(one, patches))
        return out


class FullImageCompressionPolicy(ITransmissionPolicy):
    """JPEG (default, quality 95) or PNG (compression 3) of the whole image in crop 0; the other
    crop slots are sent empty so patch counting stays per-crop."""

    @staticmethod
    def _params(config: ExperimentConfig):
        fmt = str(config.transmission_kwargs.get("format", "jpg")).lower()
        q = config.transmission_kwargs.get("quality", 95 if fmt == "jpg" else 3)
        if fmt == "jpg":
            return ".jpg", [cv2.IMWRITE_JPEG_QUALITY, int(q)]
        return ".png", [cv2.IMWRITE_PNG_COMPRESSION, int(q)]

    def encode(self, images: Any, config: ExperimentConfig):
        preserve = bool(config.transmission_kwargs.get("preserve_input_shape", False))
        ext, params = self._params(config)
        if preserve:
            items = [(images[b], {}) for b in range(images.shape[0])] if isinstance(images, np.ndarray) else \
                [_split_item(it) for it in images]
            n = 1
        else:
            B, H, W, _ = images.shape
            items = [(images[b], {}) for b in range(B)]
            n = (H // config.patch_size[0]) * (W // config.patch_size[1])
        out = []
        for b, (img, meta) in enumerate(items):
            if preserve:
                img = resize_short_side(img, _short_side(config), config.patch_size)
            ok, enc = cv2.imencode(ext, np.ascontiguousarray(img), params)
            if not ok:
                raise RuntimeError(f"failed to encode image {b} as {ext}")
            data = enc.tobytes()
            if preserve:
                ts = meta.get("target_shape") or (0, 0)
                data = struct.pack("<2i", *ts) + data
            out.append(Patch(image_idx=b, spatial_idx=0, data=data))
            out += [Patch(image_idx=b, spatial_idx=i, data=b"") for i in range(1, n)]
        yield out

    def decode(self, patches: List[Patch], config: ExperimentConfig, canvas: np.ndarray = None):
        B = config.batch_size
        H, W, C = config.image_shape
        preserve = bool(config.transmission_kwargs.get("preserve_input_shape", False))
        outs = [None] * B if preserve else (np.zeros((B, H, W, C), np.uint8) if canvas is None else canvas)
        for p in patches:
            if p.spatial_idx != 0 or not p.data:
                continue
            data = p.data
            ts = None
            if preserve:
                th, tw = struct.unpack("<2i", data[:8])
                data = data[8:]
                ts = (th, tw) if th > 0 and tw > 0 else None
            img = cv2.imdecode(np.frombuffer(data, np.uint8), cv2.IMREAD_COLOR)
            if img is None:
                raise ValueError(f"imdecode returned None for image {p.image_idx}")
            if preserve:
                outs[p.image_idx] = {"image": img, **({"target_shape": ts} if ts else {})}
            else:
                outs[p.image_idx] = img if img.shape[:2] == (H, W) else cv2.resize(img, (W, H))
        return outs
