"""Dataset loaders and task metrics on local files (reference offload/mobile/dataset.py:41-835 and
co3d_loader.py:38-171; see appcorr_b200/mobile/dataset.py for the layouts).

Every loader iterates as (images, labels) batches of `batch_size` (Co3D: one sequence per batch)
and keeps running metrics through evaluate_batch(preds, labels) / get_summary(). Images are
uint8 RGB; classification and detection images are resized to the configured shape, ADE20K and
NYU keep their native size (the server's sliding / fixed-grid inference handles the geometry).
"""
from __future__ import annotations

import gzip
import json
import os
from typing import Any, Dict, Iterator, List, Optional, Tuple

import numpy as np

try:
    import cv2  # type: ignore
except Exception:  # pragma: no cover
    cv2 = None

IMG_EXT = (".jpg", ".jpeg", ".png", ".bmp", ".webp")


def _read_rgb(path: str) -> np.ndarray:
    img = cv2.imread(path, cv2.IMREAD_COLOR)
    if img is None:
        raise FileNotFoundError(path)
    return np.ascontiguousarray(cv2.cvtColor(img, cv2.COLOR_BGR2RGB))


def resize_center_crop(img: np.ndarray, h: int, w: int) -> np.ndarray:
    """Resize so the image covers (h, w), then take the centre crop (torchvision Resize +
    CenterCrop for a square target)."""
    s = max(h / img.shape[0], w / img.shape[1])
    nh, nw = max(h, round(img.shape[0] * s)), max(w, round(img.shape[1] * s))
    interp = cv2.INTER_AREA if s < 1 else cv2.INTER_LINEAR
    img = cv2.resize(img, (nw, nh), interpolation=interp)
    y, x = (nh - h) // 2, (nw - w) // 2
    return np.ascontiguousarray(img[y:y + h, x:x + w])


class _Base:
    def __init__(self, root: str, batch_size: int, image_shape, **kwargs):
        self.root = os.path.expanduser(str(root))
        self.batch_size = int(batch_size)
        self.shape = tuple(image_shape)
        self.kwargs = kwargs

    def get_loader(self):
        return self

    def get_pbar_desc(self) -> str:
        return ", ".join(f"{k}: {v:.4g}" if isinstance(v, float) else f"{k}: {v}" for k, v in self.get_summary().items())


# ---------------------------------------------------------------------------------- ImageNet
class ImageNetLoader(_Base):
    """<root>/<class>/<image>, classes in sorted order; `sample_stride` takes an evenly spaced
    subset across all classes (dataset.py:56-63)."""

    def __init__(self, root: str, batch_size: int, image_shape, sample_stride: Optional[int] = None,
                 limit: Optional[int] = None, **kwargs):
        super().__init__(root, batch_size, image_shape, **kwargs)
        classes = sorted(d for d in os.listdir(self.root) if os.path.isdir(os.path.join(self.root, d)))
        items = []
        for ci, c in enumerate(classes):
            for f in sorted(os.listdir(os.path.join(self.root, c))):
                if f.lower().endswith(IMG_EXT):
                    items.append((os.path.join(self.root, c, f), ci))
        if sample_stride:
            items = items[:: int(sample_stride)]
        if limit:
            items = items[: int(limit)]
        self.items = items
        self.total_top1 = self.total_top5 = self.total_samples = 0

    def __len__(self) -> int:
        return -(-len(self.items) // self.batch_size)

    def __iter__(self) -> Iterator[Tuple[np.ndarray, np.ndarray]]:
        h, w = self.shape[:2]
        for i in range(0, len(self.items), self.batch_size):
            chunk = self.items[i:i + self.batch_size]
            yield (np.stack([resize_center_crop(_read_rgb(p), h, w) for p, _ in chunk]),
                   np.asarray([c for _, c in chunk]))

    def evaluate_batch(self, preds: List[Any], labels, **_) -> Dict[str, Any]:
        t1 = t5 = 0
        for p, y in zip(preds, labels):
            top = p.get("topk", []) if isinstance(p, dict) else list(p or [])
            top = [int(t) for t in top]
            if not top:
                continue
            t1 += int(top[0] == int(y))
            t5 += int(int(y) in top[:5])
        n = len(labels)
        self.total_top1 += t1
        self.total_top5 += t5
        self.total_samples += n
        return {"top1": t1, "top5": t5, "total": n}

    def get_summary(self) -> Dict[str, Any]:
        n = max(self.total_samples, 1)
        return {"total_samples": self.total_samples, "top1_acc": 100.0 * self.total_top1 / n,
                "top5_acc": 100.0 * self.total_top5 / n}


# ---------------------------------------------------------------------------------- COCO
def box_iou_xywh(d: np.ndarray, g: np.ndarray, crowd: Optional[np.ndarray] = None) -> np.ndarray:
    """IoU matrix of [n, 4] and [m, 4] boxes in (x, y, w, h); against a crowd region the overlap
    is measured over the detection's own area (the COCO convention)."""
    if len(d) == 0 or len(g) == 0:
        return np.zeros((len(d), len(g)))
    dx2, dy2 = d[:, 0] + d[:, 2], d[:, 1] + d[:, 3]
    gx2, gy2 = g[:, 0] + g[:, 2], g[:, 1] + g[:, 3]
    iw = np.clip(np.minimum(dx2[:, None], gx2[None]) - np.maximum(d[:, 0:1], g[None, :, 0]), 0, None)
    ih = np.clip(np.minimum(dy2[:, None], gy2[None]) - np.maximum(d[:, 1:2], g[None, :, 1]), 0, None)
    inter = iw * ih
    union = (d[:, 2] * d[:, 3])[:, None] + (g[:, 2] * g[:, 3])[None] - inter
    if crowd is not None and crowd.any():
        union = np.where(crowd[None, :], (d[:, 2] * d[:, 3])[:, None], union)
    return inter / np.maximum(union, 1e-12)


def coco_box_map(gts: Dict[int, List[dict]], dets: List[dict], img_ids: List[int],
                 iou_thrs=np.linspace(0.5, 0.95, 10), max_dets: int = 100) -> Dict[str, float]:
    """COCO-style box AP over all areas: per category and IoU threshold, detections (top
    `max_dets` per image by score) are matched greedily in score order to the unmatched
    non-crowd ground truth of highest IoU above the threshold; matches to crowd boxes are ignored;
    precision is made monotone and sampled at 101 recall points. mAP averages over IoU thresholds
    and categories that have ground truth; AP50 / AP75 at those thresholds."""
    cats = sorted({a["category_id"] for ims in gts.values() for a in ims})
    by_img: Dict[int, List[dict]] = {}
    for d in dets:
        by_img.setdefault(int(d["image_id"]), []).append(d)
    for i in by_img:
        by_img[i] = sorted(by_img[i], key=lambda d: -d["score"])[:max_dets]
    rec_pts = np.linspace(0, 1, 101)
    ap = np.full((len(iou_thrs), len(cats)), np.nan)
    for ci, c in enumerate(cats):
        scores, tps, n_gt = [], [[] for _ in iou_thrs], 0
        for im in img_ids:
            g = [a for a in gts.get(im, []) if a["category_id"] == c]
            d = [x for x in by_img.get(im, []) if int(x["category_id"]) == c]
            crowd = np.array([bool(a.get("iscrowd", 0)) for a in g], dtype=bool)
            n_gt += int((~crowd).sum())
            if not d:
                continue
            gb = np.array([a["bbox"] for a in g], dtype=float).reshape(-1, 4)
            db = np.array([x["bbox"] for x in d], dtype=float).reshape(-1, 4)
            order_g = np.argsort(crowd, kind="stable")  # regular boxes first, crowd regions last
            iou = box_iou_xywh(db, gb, crowd)
            for ti, t in enumerate(iou_thrs):
                used = np.zeros(len(g), dtype=bool)
                for di in range(len(d)):
                    best, bj = min(t, 1 - 1e-10), -1
                    for gj in order_g:
                        if used[gj] and not crowd[gj]:
                            continue
                        if bj >= 0 and not crowd[bj] and crowd[gj]:
                            break  # a regular match beats any crowd region
                        if iou[di, gj] < best:
                            continue
                        best, bj = iou[di, gj], gj
                    if bj < 0:
                        tps[ti].append(0)
                    elif crowd[bj]:
                        tps[ti].append(-1)  # matched a crowd region: ignored
                    else:
                        used[bj] = True
                        tps[ti].append(1)
            scores += [x["score"] for x in d]
        if n_gt == 0:
            continue
        order = np.argsort(-np.asarray(scores), kind="mergesort")
        for ti in range(len(iou_thrs)):
            m = np.asarray(tps[ti])[order] if scores else np.zeros(0)
            keep = m >= 0
            tp = np.cumsum(m[keep] == 1)
            fp = np.cumsum(m[keep] == 0)
            rec = tp / n_gt
            prec = tp / np.maximum(tp + fp, np.finfo(float).eps)
            for k in range(len(prec) - 2, -1, -1):
                prec[k] = max(prec[k], prec[k + 1])
            q = np.zeros(len(rec_pts))
            idx = np.searchsorted(rec, rec_pts, side="left")
            for ri, pi in enumerate(idx):
                if pi < len(prec):
                    q[ri] = prec[pi]
            ap[ti, ci] = q.mean()
    def mean(a):
        v = a[~np.isnan(a)]
        return float(v.mean()) if v.size else 0.0
    t50 = int(np.argmin(np.abs(iou_thrs - 0.5)))
    t75 = int(np.argmin(np.abs(iou_thrs - 0.75)))
    return {"mAP": mean(ap), "mAP_50": mean(ap[t50]), "mAP_75": mean(ap[t75])}


class COCO2017Loader(_Base):
    """COCO val2017 instances. Labels per image: [image_id, width, height]. Predictions: the
    detector executor's {"scores", "labels", "boxes"} with boxes (cx, cy, w, h) normalised to the
    model input; they are scaled back to the original image (dataset.py:297-343)."""

    def __init__(self, root: str, batch_size: int, image_shape, ann_file: Optional[str] = None,
                 limit: Optional[int] = None, **kwargs):
        super().__init__(root, batch_size, image_shape, **kwargs)
        ann = ann_file or os.path.join(self.root, "annotations", "instances_val2017.json")
        data = json.load(open(ann))
        self.images = sorted(data["images"], key=lambda im: im["id"])
        if limit:
            self.images = self.images[: int(limit)]
        self.gts: Dict[int, List[dict]] = {}
        for a in data.get("annotations", []):
            self.gts.setdefault(int(a["image_id"]), []).append(a)
        self.img_dir = os.path.join(self.root, "val2017")
        self.results: List[dict] = []
        self.processed: List[int] = []

    def __len__(self) -> int:
        return -(-len(self.images) // self.batch_size)

    def __iter__(self):
        h, w = self.shape[:2]
        for i in range(0, len(self.images), self.batch_size):
            chunk = self.images[i:i + self.batch_size]
            imgs = [cv2.resize(_read_rgb(os.path.join(self.img_dir, im["file_name"])), (w, h),
                               interpolation=cv2.INTER_LINEAR) for im in chunk]
            yield np.stack(imgs), np.asarray([[im["id"], im["width"], im["height"]] for im in chunk])

    def evaluate_batch(self, preds: List[Any], labels, **_) -> Dict[str, Any]:
        n = 0
        for p, (img_id, W, H) in zip(preds, np.asarray(labels).tolist()):
            if img_id < 0:
                continue
            n += 1
            self.processed.append(int(img_id))
            if not isinstance(p, dict) or "boxes" not in p:
                continue
            for sc, cat, box in zip(p["scores"], p["labels"], p["boxes"]):
                cx, cy, bw, bh = (float(v) for v in box)
                self.results.append({"image_id": int(img_id), "category_id": int(cat), "score": float(sc),
                                     "bbox": [(cx - bw / 2) * W, (cy - bh / 2) * H, bw * W, bh * H]})
        return {"detected_images": n}

    def get_summary(self) -> Dict[str, Any]:
        if not self.results:
            return {"mAP": 0.0, "status": "no_results"}
        ids = sorted(set(self.processed))
        out = coco_box_map(self.gts, self.results, ids)
        out["total_images"] = len(ids)
        return out


# ---------------------------------------------------------------------------------- ADE20K
def intersect_and_union(pred: np.ndarray, gt: np.ndarray, num_classes: int, ignore_index: int = 255,
                        reduce_zero_label: bool = True) -> np.ndarray:
    """[4, C] areas (intersection, union, predicted, label) of one image (dataset.py:584-611):
    with reduce_zero_label, label 0 (other) becomes ignored and the rest shift down by one."""
    pred = np.asarray(pred).astype(np.int64)
    gt = np.asarray(gt).astype(np.int64)
    if pred.shape != gt.shape:
        pred = cv2.resize(pred.astype(np.int32), (gt.shape[1], gt.shape[0]), interpolation=cv2.INTER_NEAREST)
    if reduce_zero_label:
        gt = gt.copy()
        gt[gt == 0] = ignore_index + 1
        gt -= 1
        gt[gt == ignore_index] = ignore_index
    valid = gt != ignore_index
    p, g = pred[valid], gt[valid]
    inter = p[p == g]
    bc = lambda x: np.bincount(x[(x >= 0) & (x < num_classes)], minlength=num_classes)[:num_classes].astype(float)  # noqa: E731
    ai, ap_, al = bc(inter), bc(p), bc(g)
    return np.stack([ai, ap_ + al - ai, ap_, al])


def seg_metrics(areas: np.ndarray) -> Dict[str, float]:
    """mIoU, mean accuracy, aAcc, dice, fscore, precision, recall (percent; NaN classes skipped)."""
    ai, au, ap_, al = areas
    if al.sum() == 0:
        return {}
    with np.errstate(divide="ignore", invalid="ignore"):
        iou = np.where(au > 0, ai / au, np.nan)
        acc = np.where(al > 0, ai / al, np.nan)
        dice = np.where(ap_ + al > 0, 2 * ai / (ap_ + al), np.nan)
        prec = np.where(ap_ > 0, ai / ap_, np.nan)
        rec = np.where(al > 0, ai / al, np.nan)
        f = np.where(np.isfinite(prec) & np.isfinite(rec) & (prec + rec > 0), 2 * prec * rec / (prec + rec),
                     np.where(ap_ + al > 0, 0.0, np.nan))
    nm = lambda v: float(np.nanmean(v) * 100) if np.isfinite(v).any() else 0.0  # noqa: E731
    return {"mIoU": nm(iou), "acc": nm(acc), "aAcc": float(ai.sum() / al.sum() * 100), "dice": nm(dice),
            "fscore": nm(f), "precision": nm(prec), "recall": nm(rec)}


class ADE20KLoader(_Base):
    """ADEChallengeData2016 validation: images/validation/*.jpg with annotations/validation/*.png
    (150 classes, label 0 = other, reduce_zero_label). Images keep their native size, or their
    short side is resized to `resize_short_side` when given."""

    def __init__(self, root: str, batch_size: int, image_shape, num_classes: int = 150, reduce_zero_label: bool = True,
                 resize_short_side: Optional[int] = None, limit: Optional[int] = None, **kwargs):
        super().__init__(root, batch_size, image_shape, **kwargs)
        idir = os.path.join(self.root, "images", "validation")
        adir = os.path.join(self.root, "annotations", "validation")
        names = sorted(f for f in os.listdir(idir) if f.lower().endswith(IMG_EXT))
        if limit:
            names = names[: int(limit)]
        self.items = [(os.path.join(idir, f), os.path.join(adir, os.path.splitext(f)[0] + ".png")) for f in names]
        self.num_classes, self.reduce_zero_label = int(num_classes), bool(reduce_zero_label)
        self.short = resize_short_side
        self.areas = np.zeros((4, self.num_classes))

    def __len__(self) -> int:
        return -(-len(self.items) // self.batch_size)

    def _img(self, path):
        img = _read_rgb(path)
        if self.short:
            h, w = img.shape[:2]
            s = float(self.short) / min(h, w)
            img = cv2.resize(img, (round(w * s), round(h * s)), interpolation=cv2.INTER_LINEAR)
        return img

    def __iter__(self):
        for i in range(0, len(self.items), self.batch_size):
            chunk = self.items[i:i + self.batch_size]
            imgs = [self._img(p) for p, _ in chunk]
            masks = [cv2.imread(a, cv2.IMREAD_UNCHANGED) for _, a in chunk]
            if len({im.shape for im in imgs}) == 1:
                yield np.stack(imgs), masks
            else:
                yield [{"image": im, "metadata": {"target_shape": m.shape[:2]}} for im, m in zip(imgs, masks)], masks

    def evaluate_batch(self, preds: List[Any], labels, **_) -> Dict[str, Any]:
        for p, gt in zip(preds, labels):
            mask = p.get("mask") if isinstance(p, dict) else p
            if mask is None:
                continue
            self.areas += intersect_and_union(mask, gt, self.num_classes, 255, self.reduce_zero_label)
        return seg_metrics(self.areas)

    def get_summary(self) -> Dict[str, Any]:
        return seg_metrics(self.areas)


# ---------------------------------------------------------------------------------- NYU depth
def nyu_depth_metrics(pred: np.ndarray, gt: np.ndarray, min_depth: float = 1e-3, max_depth: float = 10.0):
    """Per-image NYU metrics (dataset.py:731-812): Eigen crop (rows 43:472, cols 45:608 of a
    480x640 map; else the top-left 93.75% x 81.25%), least-squares scale + shift of the prediction
    on the valid pixels, clipped to [min_depth, max_depth]. Returns (metrics, valid pixel count)."""
    pred = np.asarray(pred, dtype=np.float32)
    gt = np.asarray(gt, dtype=np.float32)
    if pred.shape != gt.shape:
        pred = cv2.resize(pred, (gt.shape[1], gt.shape[0]), interpolation=cv2.INTER_LINEAR)
    h, w = gt.shape
    if (h, w) == (480, 640):
        g, p = gt[43:472, 45:608], pred[43:472, 45:608]
    else:
        g, p = gt[: int(0.9375 * h), : int(0.8125 * w)], pred[: int(0.9375 * h), : int(0.8125 * w)]
    valid = (g > min_depth) & (g < max_depth)
    n = int(valid.sum())
    if n == 0:
        return None, 0
    A = np.stack([p[valid].astype(np.float64), np.ones(n)], axis=1)
    sol, *_ = np.linalg.lstsq(A, g[valid].astype(np.float64), rcond=None)
    pa = np.clip(p * sol[0] + sol[1], min_depth, max_depth)
    gv, pv = g[valid].astype(np.float64), pa[valid].astype(np.float64)
    r = np.maximum(gv / (pv + 1e-8), pv / (gv + 1e-8))
    return {"abs_rel": float(np.mean(np.abs(gv - pv) / gv)), "sq_rel": float(np.mean((gv - pv) ** 2 / gv)),
            "rmse": float(np.sqrt(np.mean((gv - pv) ** 2))),
            "rmse_log": float(np.sqrt(np.mean((np.log(gv) - np.log(np.maximum(pv, 1e-8))) ** 2))),
            "delta_1.25": float((r < 1.25).mean()), "delta_1.25^2": float((r < 1.25 ** 2).mean()),
            "delta_1.25^3": float((r < 1.25 ** 3).mean())}, n


class NYUDepthLoader(_Base):
    """<root>/nyu_test.txt lines "rgb_path depth_path [focal]"; depth PNGs in millimetres."""

    def __init__(self, root: str, batch_size: int, image_shape, limit: Optional[int] = None, **kwargs):
        super().__init__(root, batch_size, image_shape, **kwargs)
        lines = [ln.split() for ln in open(os.path.join(self.root, "nyu_test.txt")) if ln.strip()]
        if limit:
            lines = lines[: int(limit)]
        self.entries = lines
        self.sums: Dict[str, float] = {}
        self.pixels = 0
        self.samples = 0

    def __len__(self) -> int:
        return -(-len(self.entries) // self.batch_size)

    def __iter__(self):
        for i in range(0, len(self.entries), self.batch_size):
            chunk = self.entries[i:i + self.batch_size]
            imgs = [_read_rgb(os.path.join(self.root, e[0])) for e in chunk]
            labels = [{"idx": i + j, "depth": cv2.imread(os.path.join(self.root, e[1]), cv2.IMREAD_UNCHANGED)
                       .astype(np.float32) / 1000.0, "focal": float(e[2]) if len(e) > 2 else 518.8579}
                      for j, e in enumerate(chunk)]
            yield np.stack(imgs), labels

    def evaluate_batch(self, preds: List[Any], labels, **_) -> Dict[str, Any]:
        for p, lab in zip(preds, labels):
            d = p.get("depth") if isinstance(p, dict) else None
            if d is None or not isinstance(lab, dict):
                continue
            m, n = nyu_depth_metrics(d, lab["depth"])
            if m is None:
                continue
            self.samples += 1
            self.pixels += n
            for k, v in m.items():
                self.sums[k] = self.sums.get(k, 0.0) + v * n
        return {"depth_images": len(preds)}

    def get_summary(self) -> Dict[str, Any]:
        if not self.pixels:
            return {"total_samples": self.samples}
        return {"total_samples": self.samples, **{k: v / self.pixels for k, v in self.sums.items()}}


# ---------------------------------------------------------------------------------- Co3D
_P3D_TO_OPENCV = np.diag([-1.0, -1.0, 1.0])


def relative_rotation_errors(Rp: np.ndarray, Rg: np.ndarray) -> np.ndarray:
    """Angle (degrees) between predicted and true relative rotations over every frame pair."""
    errs = []
    for i in range(len(Rg)):
        for j in range(i + 1, len(Rg)):
            c = (np.trace((Rg[j] @ Rg[i].T).T @ (Rp[j] @ Rp[i].T)) - 1) / 2
            errs.append(np.degrees(np.arccos(np.clip(c, -1, 1))))
    return np.asarray(errs)


def median_aligned_depth_metrics(pred: np.ndarray, gts: List[np.ndarray]) -> Optional[Dict[str, float]]:
    ps, gs = [], []
    for p, g in zip(pred, gts):
        g = cv2.resize(np.asarray(g, np.float32), (p.shape[1], p.shape[0]), interpolation=cv2.INTER_NEAREST)
        m = g > 0
        if m.sum() > 50:
            ps.append(p[m])
            gs.append(g[m])
    if not ps:
        return None
    p, g = np.concatenate(ps), np.concatenate(gs)
    p = p * (np.median(g) / np.median(p))
    r = np.maximum(p / g, g / p)
    return {"absrel": float((np.abs(p - g) / g).mean()), "d125": float((r < 1.25).mean()),
            "d110": float((r < 1.10).mean())}


class CO3DSequenceLoader(_Base):
    """One Co3Dv2 sequence per batch: `frames_per_sequence` frames every `frame_stride` frames of
    each sequence of the chosen categories; labels carry depth maps (float16 bit-packed PNGs times
    the scale adjustment, masked) and OpenCV-convention camera rotations / translations
    (co3d_loader.py:27-110: R_cv = diag(-1,-1,1) R^T, T_cv = diag(-1,-1,1) T)."""

    def __init__(self, root: str, batch_size: int, image_shape, categories: Optional[List[str]] = None,
                 frames_per_sequence: int = 8, frame_stride: int = 5, **kwargs):
        super().__init__(root, batch_size, image_shape, **kwargs)
        self.categories = categories or ["hotdog", "tv", "parkingmeter", "baseballbat"]
        self.fps, self.stride = int(frames_per_sequence), int(frame_stride)
        self.seqs = self._sequences()
        self.n = 0
        self.sums = {"abs_rel": 0.0, "delta_1.25": 0.0, "delta_1.10": 0.0, "rot_deg": 0.0, "RRA@15": 0.0}

    def _sequences(self):
        out = []
        for cat in self.categories:
            path = os.path.join(self.root, cat, "frame_annotations.jgz")
            if not os.path.exists(path):
                continue
            by: Dict[str, list] = {}
            for a in json.loads(gzip.open(path).read()):
                by.setdefault(a["sequence_name"], []).append(a)
            for seq in sorted(by):
                anns = sorted(by[seq], key=lambda a: a["frame_number"])[:: self.stride][: self.fps]
                if len(anns) == self.fps:
                    out.append({"category": cat, "sequence": seq, "anns": anns})
        return out

    def __len__(self) -> int:
        return len(self.seqs)

    @staticmethod
    def _depth(path: str, mask_path: str, scale: float) -> np.ndarray:
        raw = cv2.imread(path, cv2.IMREAD_UNCHANGED)
        d = np.frombuffer(raw.astype(np.uint16).tobytes(), dtype=np.float16).astype(np.float32).reshape(raw.shape[:2])
        d = d * scale
        d[cv2.imread(mask_path, cv2.IMREAD_UNCHANGED) == 0] = 0
        return d

    def __iter__(self):
        for s in self.seqs:
            frames, depths, Rs, Ts = [], [], [], []
            for a in s["anns"]:
                frames.append(_read_rgb(os.path.join(self.root, a["image"]["path"])))
                depths.append(self._depth(os.path.join(self.root, a["depth"]["path"]),
                                          os.path.join(self.root, a["depth"]["mask_path"]),
                                          float(a["depth"]["scale_adjustment"])))
                Rs.append(_P3D_TO_OPENCV @ np.asarray(a["viewpoint"]["R"], dtype=np.float64).T)
                Ts.append(_P3D_TO_OPENCV @ np.asarray(a["viewpoint"]["T"], dtype=np.float64))
            yield np.stack(frames), [{"category": s["category"], "sequence": s["sequence"], "depths": depths,
                                      "R": np.stack(Rs), "T": np.stack(Ts)}]

    def evaluate_batch(self, preds: List[Any], labels, **_) -> Dict[str, Any]:
        for p, lab in zip(preds, labels):
            if not isinstance(p, dict) or "depth" not in p or "R" not in p:
                continue
            dm = median_aligned_depth_metrics(np.asarray(p["depth"]), lab["depths"])
            if dm is None:
                continue
            e = relative_rotation_errors(np.asarray(p["R"]), lab["R"])
            self.n += 1
            self.sums["abs_rel"] += dm["absrel"]
            self.sums["delta_1.25"] += dm["d125"]
            self.sums["delta_1.10"] += dm["d110"]
            self.sums["rot_deg"] += float(np.median(e)) if e.size else 0.0
            self.sums["RRA@15"] += float((e < 15).mean()) if e.size else 0.0
        return self.get_summary()

    def get_summary(self) -> Dict[str, Any]:
        if not self.n:
            return {}
        return {"sequences": self.n, **{k: v / self.n for k, v in self.sums.items()}}
