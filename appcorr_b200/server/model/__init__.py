"""Model executor registry (substring-matched, same names as the reference registry,
offload/server/model/__init__.py:4-40)."""
from __future__ import annotations

from .base import ModelExecutor, PyramidBatch  # noqa: F401


def get_model_executor(name: str, device) -> ModelExecutor:
    if "dinov3_segmentor_linhead" in name:
        from .dinov3_segmentor_linhead import DINOv3SegmentorLinheadExecutor

        return DINOv3SegmentorLinheadExecutor(device)
    if "dinov3_classifier" in name:
        from .dinov3_classifier import DINOv3ClassifierExecutor

        return DINOv3ClassifierExecutor(device)
    if "dinov3_detector" in name:
        from .dinov3_detector import DINOv3DetectorExecutor

        return DINOv3DetectorExecutor(device)
    if "dinov3_segmentor_m2f" in name or "dinov3_segmentor" in name:
        from .dinov3_segmentor_m2f import DINOv3SegmentorM2FExecutor

        return DINOv3SegmentorM2FExecutor(device)
    if "dinov3_depther" in name:
        from .dinov3_depther import DINOv3DeptherExecutor

        return DINOv3DeptherExecutor(device)
    if "qwen25vl" in name:
        from .qwen25vl_executor import Qwen25VLExecutor

        return Qwen25VLExecutor(device)
    if "vggt" in name:
        from .vggt_executor import VGGTExecutor

        return VGGTExecutor(device)
    if "sam3" in name:
        from .sam3_executor import Sam3Executor

        return Sam3Executor(device)
    if "openclip" in name or "clip" in name:
        from .openclip_executor import OpenCLIPExecutor

        return OpenCLIPExecutor(device)
    if "dinov3" in name:
        from .dinov3_classifier import DINOv3ClassifierExecutor

        return DINOv3ClassifierExecutor(device)
    raise ValueError(f"Unknown model executor for: {name}")
