"""Request sources and task metrics for the mobile client (reference offload/mobile/dataset.py:8-849,
co3d_loader.py:38-171).

Loaders (`get_dataset_loader(name, root, batch_size, image_shape, ...)`), all reading local files
in the datasets' standard layouts (no network, no fiftyone / HF datasets / pycocotools):
  imagenet-1k        <root>/<class>/<image>                      top-1 / top-5 accuracy
  coco2017           <root>/annotations/instances_val2017.json,  COCO box mAP (own evaluator:
                     <root>/val2017/<file>                       IoU 0.50:0.95, 101-point AP)
  ade20k             <root>/images/validation/*.jpg,             mIoU / aAcc / dice / fscore from
                     <root>/annotations/validation/*.png         intersect-and-union areas
  nyu_depth          <root>/nyu_test.txt: "rgb depth_png [focal]" abs_rel, sq_rel, rmse, rmse_log,
                                                                 delta 1.25^k after least-squares
                                                                 scale/shift alignment, Eigen crop
  co3d / co3dv2      <root>/<category>/frame_annotations.jgz    median-aligned depth abs_rel,
                                                                 relative rotation error / RRA@15
  synthetic          deterministic images of the configured shape (pixels ~ clipped N(128, 60^2))
                     with random labels; also used when `root` does not exist
Loaders iterate as (images, labels); those with metrics expose evaluate_batch(preds, labels) and
get_summary().
"""
from __future__ import annotations

import os
from typing import Iterator, List, Optional, Tuple

import numpy as np

try:
    import cv2  # type: ignore
except Exception:  # pragma: no cover
    cv2 = None


class SyntheticLoader:
    def __init__(self, batch_size: int, image_shape, num_batches: int = 8, num_classes: int = 1000, seed: int = 0,
                 mean: float = 128.0, std: float = 60.0, **_):
        self.batch_size, self.shape = batch_size, tuple(image_shape)
        self.num_batches, self.num_classes, self.seed = num_batches, num_classes, seed
        self.mean, self.std = mean, std

    def __len__(self) -> int:
        return self.num_batches

    def __iter__(self) -> Iterator[Tuple[np.ndarray, np.ndarray]]:
        rng = np.random.default_rng(self.seed)
        for _ in range(self.num_batches):
            imgs = np.clip(rng.normal(self.mean, self.std, size=(self.batch_size,) + self.shape), 0, 255).astype(np.uint8)
            yield imgs, rng.integers(0, self.num_classes, size=self.batch_size)

    def get_loader(self):
        return self


class ImageFolderLoader:
    EXT = (".jpg", ".jpeg", ".png", ".bmp", ".webp")

    def __init__(self, root: str, batch_size: int, image_shape, limit: Optional[int] = None, **_):
        root = os.path.expanduser(root)
        classes = sorted(d for d in os.listdir(root) if os.path.isdir(os.path.join(root, d)))
        self.items: List[Tuple[str, int]] = []
        for ci, c in enumerate(classes):
            for f in sorted(os.listdir(os.path.join(root, c))):
                if f.lower().endswith(self.EXT):
                    self.items.append((os.path.join(root, c, f), ci))
        if limit:
            self.items = self.items[:limit]
        self.batch_size, self.shape = batch_size, tuple(image_shape)

    def __len__(self) -> int:
        return -(-len(self.items) // self.batch_size)

    def _load(self, path: str) -> np.ndarray:
        img = cv2.cvtColor(cv2.imread(path, cv2.IMREAD_COLOR), cv2.COLOR_BGR2RGB)
        h, w = self.shape[:2]
        s = max(h / img.shape[0], w / img.shape[1])
        img = cv2.resize(img, (max(w, round(img.shape[1] * s)), max(h, round(img.shape[0] * s))),
                         interpolation=cv2.INTER_AREA)
        y, x = (img.shape[0] - h) // 2, (img.shape[1] - w) // 2
        return np.ascontiguousarray(img[y:y + h, x:x + w])

    def __iter__(self):
        for i in range(0, len(self.items), self.batch_size):
            chunk = self.items[i:i + self.batch_size]
            yield np.stack([self._load(p) for p, _ in chunk]), np.asarray([c for _, c in chunk])

    def get_loader(self):
        return self


def get_dataset_loader(name: str, data_root: Optional[str], batch_size: int, image_shape, **kwargs):
    if name == "synthetic" or data_root is None or not os.path.isdir(os.path.expanduser(str(data_root))):
        return SyntheticLoader(batch_size, image_shape, **kwargs)
    from . import datasets as D

    n = str(name).lower()
    if n in ("imagenet-1k", "imagenet", "image_folder"):
        return D.ImageNetLoader(data_root, batch_size, image_shape, **kwargs)
    if n == "coco2017":
        return D.COCO2017Loader(data_root, batch_size, image_shape, **kwargs)
    if n in ("ade20k", "scene_parse_150"):
        return D.ADE20KLoader(data_root, batch_size, image_shape, **kwargs)
    if n == "nyu_depth":
        return D.NYUDepthLoader(data_root, batch_size, image_shape, **kwargs)
    if n in ("co3d", "co3dv2"):
        return D.CO3DSequenceLoader(data_root, batch_size, image_shape, **kwargs)
    return ImageFolderLoader(data_root, batch_size, image_shape, **kwargs)


# ------------------------------------------------------------------ metrics
def topk_correct(preds, labels, k: int) -> int:
    n = 0
    for p, y in zip(preds, labels):
        top = p.get("topk", []) if isinstance(p, dict) else list(p)
        n += int(int(y) in [int(t) for t in top[:k]])
    return n


def confusion(pred: np.ndarray, gt: np.ndarray, num_classes: int, ignore: int = 255) -> np.ndarray:
    m = gt != ignore
    return np.bincount(num_classes * gt[m].astype(int) + pred[m].astype(int), minlength=num_classes ** 2).reshape(
        num_classes, num_classes)


def miou(conf: np.ndarray) -> Tuple[float, float]:
    inter = np.diag(conf).astype(float)
    union = conf.sum(0) + conf.sum(1) - inter
    valid = union > 0
    return float((inter[valid] / union[valid]).mean()) if valid.any() else 0.0, float(inter.sum() / max(conf.sum(), 1))


def depth_metrics(pred: np.ndarray, gt: np.ndarray) -> dict:
    m = gt > 0
    p, g = pred[m], gt[m]
    ratio = np.maximum(p / g, g / p)
    return {"abs_rel": float(np.mean(np.abs(p - g) / g)), "delta1": float(np.mean(ratio < 1.25))}
