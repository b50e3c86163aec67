"""Dataset loaders and task metrics on tiny synthetic datasets in the standard on-disk layouts
(reference offload/mobile/dataset.py, co3d_loader.py)."""
import gzip
import json
import os

import cv2
import numpy as np
import pytest

from appcorr_b200.mobile import datasets as D
from appcorr_b200.mobile.dataset import get_dataset_loader


def _img(path, h=40, w=60, v=0):
    os.makedirs(os.path.dirname(path), exist_ok=True)
    cv2.imwrite(path, np.full((h, w, 3), v, np.uint8))


def test_imagenet_folder_and_topk(tmp_path):
    for c in ("a", "b", "c"):
        for i in range(3):
            _img(str(tmp_path / c / f"{i}.png"), v=10 * i)
    ld = get_dataset_loader("imagenet-1k", str(tmp_path), 4, (32, 32, 3))
    batches = list(ld)
    assert len(batches) == 3 and batches[0][0].shape == (4, 32, 32, 3)
    assert list(np.concatenate([b[1] for b in batches])) == [0, 0, 0, 1, 1, 1, 2, 2, 2]
    ld.evaluate_batch([{"topk": [0, 1]}, {"topk": [1, 0]}, {"topk": [2, 3, 4, 5, 1]}], [0, 0, 1])
    s = ld.get_summary()
    assert s["top1_acc"] == pytest.approx(100 / 3) and s["top5_acc"] == pytest.approx(100.0)


def test_coco_map_perfect_half_and_crowd():
    gts = {1: [{"category_id": 3, "bbox": [10, 10, 20, 20], "iscrowd": 0},
               {"category_id": 3, "bbox": [50, 50, 10, 10], "iscrowd": 0},
               {"category_id": 3, "bbox": [0, 0, 100, 100], "iscrowd": 1}]}
    perfect = [{"image_id": 1, "category_id": 3, "bbox": [10, 10, 20, 20], "score": 0.9},
               {"image_id": 1, "category_id": 3, "bbox": [50, 50, 10, 10], "score": 0.8}]
    assert D.coco_box_map(gts, perfect, [1])["mAP"] == pytest.approx(1.0)
    # one of two found, plus a false positive inside the crowd region (ignored, not an FP)
    half = [perfect[0], {"image_id": 1, "category_id": 3, "bbox": [70, 70, 20, 20], "score": 0.95}]
    r = D.coco_box_map(gts, half, [1])
    # recall reaches 0.5 at precision 1 (the crowd match is ignored): AP = 51 / 101
    assert r["mAP_50"] == pytest.approx(51 / 101, abs=1e-9)


def test_coco_loader_scales_boxes_back(tmp_path):
    os.makedirs(tmp_path / "annotations")
    _img(str(tmp_path / "val2017" / "000001.jpg"), h=100, w=200)
    json.dump({"images": [{"id": 1, "file_name": "000001.jpg", "width": 200, "height": 100}],
               "annotations": [{"image_id": 1, "category_id": 5, "bbox": [20, 10, 40, 30], "iscrowd": 0}],
               "categories": [{"id": 5}]}, open(tmp_path / "annotations" / "instances_val2017.json", "w"))
    ld = get_dataset_loader("coco2017", str(tmp_path), 2, (64, 64, 3))
    (imgs, labels), = list(ld)
    assert imgs.shape == (1, 64, 64, 3) and labels.tolist() == [[1, 200, 100]]
    # the detector's normalised (cx, cy, w, h) for the ground-truth box
    ld.evaluate_batch([{"scores": [0.9], "labels": [5], "boxes": [[0.2, 0.25, 0.2, 0.3]]}], labels)
    assert ld.get_summary()["mAP"] == pytest.approx(1.0)


def test_ade20k_miou_reduce_zero_label(tmp_path):
    _img(str(tmp_path / "images" / "validation" / "x.jpg"), h=4, w=4)
    gt = np.array([[0, 1, 1, 2], [1, 1, 2, 2], [3, 3, 3, 3], [0, 0, 2, 2]], np.uint8)
    os.makedirs(tmp_path / "annotations" / "validation")
    cv2.imwrite(str(tmp_path / "annotations" / "validation" / "x.png"), gt)
    ld = get_dataset_loader("ade20k", str(tmp_path), 1, (4, 4, 3), num_classes=3)
    (imgs, masks), = list(ld)
    pred = gt.astype(int) - 1          # labels 1..3 -> classes 0..2; the "other" pixels are ignored
    pred[0, 1] = 2                     # one wrong pixel (class 0 -> 2)
    m = ld.evaluate_batch([{"mask": pred}], masks)
    # class 0: inter 3, union 4; class 1: inter 5, union 5; class 2: inter 4, union 5
    assert m["mIoU"] == pytest.approx(100 * (3 / 4 + 1 + 4 / 5) / 3)
    assert m["aAcc"] == pytest.approx(100 * 12 / 13)


def test_nyu_depth_alignment_and_crop():
    gt = np.random.default_rng(0).uniform(1, 5, (480, 640)).astype(np.float32)
    pred = (gt - 0.3) / 2.0            # an affine distortion: least squares undoes it exactly
    m, n = D.nyu_depth_metrics(pred, gt)
    assert n == 429 * 563
    assert m["abs_rel"] < 1e-5 and m["delta_1.25"] == 1.0


def test_nyu_loader(tmp_path):
    _img(str(tmp_path / "rgb" / "0.png"), h=48, w=64)
    os.makedirs(tmp_path / "depth")
    cv2.imwrite(str(tmp_path / "depth" / "0.png"), np.full((48, 64), 2500, np.uint16))
    (tmp_path / "nyu_test.txt").write_text("rgb/0.png depth/0.png 518.8\n")
    ld = get_dataset_loader("nyu_depth", str(tmp_path), 2, (48, 64, 3))
    (imgs, labels), = list(ld)
    assert labels[0]["depth"].max() == pytest.approx(2.5)
    ld.evaluate_batch([{"depth": np.full((24, 32), 7.0, np.float32)}], labels)
    assert ld.get_summary()["total_samples"] == 1


def test_relative_rotation_error():
    def rz(a):
        c, s = np.cos(np.radians(a)), np.sin(np.radians(a))
        return np.array([[c, -s, 0], [s, c, 0], [0, 0, 1]])

    Rg = np.stack([rz(0), rz(30), rz(60)])
    assert np.allclose(D.relative_rotation_errors(Rg, Rg), 0, atol=1e-5)
    Rp = np.stack([rz(0), rz(40), rz(60)])
    assert np.allclose(sorted(D.relative_rotation_errors(Rp, Rg)), [0, 10, 10], atol=1e-4)


def test_co3d_loader(tmp_path):
    cat = tmp_path / "tv"
    os.makedirs(cat / "s1")
    anns = []
    for f in range(4):
        _img(str(cat / "s1" / f"im{f}.png"), h=32, w=32)
        d = np.full((32, 32), 1.5, np.float16).view(np.uint16)
        cv2.imwrite(str(cat / "s1" / f"d{f}.png"), d)
        cv2.imwrite(str(cat / "s1" / f"m{f}.png"), np.full((32, 32), 255, np.uint8))
        anns.append({"sequence_name": "s1", "frame_number": f, "image": {"path": f"tv/s1/im{f}.png", "size": [32, 32]},
                     "depth": {"path": f"tv/s1/d{f}.png", "mask_path": f"tv/s1/m{f}.png", "scale_adjustment": 2.0},
                     "viewpoint": {"R": np.eye(3).tolist(), "T": [0, 0, 1]}})
    with gzip.open(cat / "frame_annotations.jgz", "wt") as fh:
        json.dump(anns, fh)
    ld = get_dataset_loader("co3d", str(tmp_path), 1, (32, 32, 3), categories=["tv"], frames_per_sequence=4,
                            frame_stride=1)
    (frames, labels), = list(ld)
    assert frames.shape == (4, 32, 32, 3) and labels[0]["depths"][0].max() == pytest.approx(3.0)
    R = labels[0]["R"]
    s = ld.evaluate_batch([{"depth": np.full((4, 16, 16), 0.5, np.float32), "R": R}], labels)
    assert s["sequences"] == 1 and s["abs_rel"] < 1e-6 and s["rot_deg"] < 1e-6
