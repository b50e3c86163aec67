"""Policy registries (same names as the reference registry, offload/policies/__init__.py:38-82)."""
from __future__ import annotations

from typing import Optional

from ..common.protocol import ExperimentConfig
from .interface import ISchedulingPolicy, ITransmissionPolicy  # noqa: F401
from . import scheduling as S
from . import transmission as T

SCHEDULER_REGISTRY = {
    "ADE20KApproxCorrect": S.ADE20KApproxCorrectPolicy,
    "ADE20KInterleavedDynamic": S.ADE20KInterleavedDynamicPolicy,
    "ADE20KSequential": S.ADE20KSequentialPolicy,
    "NYUApproxCorrect": S.NYUApproxCorrectPolicy,
    "VGGTInterleaved": S.VGGTInterleavedPolicy,
    "BatchCountBased": S.BatchCountBasedPolicy,
    "GroupTrigger": S.GroupTriggerPolicy,
    "DynamicGroupTrigger": S.DynamicGroupTriggerPolicy,
    "COCOWindowInterleaved": S.COCOWindowInterleavedPolicy,
    "COCOWindowDynamic": S.COCOWindowDynamicPolicy,
    "ADE20KWindowInterleaved": S.ADE20KWindowInterleavedPolicy,
}

TRANSMISSION_REGISTRY = {
    "Raw": T.RawTransmissionPolicy,
    "NYUAppCorrRaw": T.NYUAppCorrRawTransmissionPolicy,
    "Zlib": T.ZlibTransmissionPolicy,
    "Laplacian": T.LaplacianPyramidPolicy,
    "NYUAppCorrLaplacian": T.NYUAppCorrLaplacianPolicy,
    "ProgressiveLaplacian": T.ProgressiveLPyramidPolicy,
    "NYUAppCorrProgressiveLaplacian": T.NYUAppCorrProgressiveLaplacianPolicy,
    "COCOWindowProgressiveLaplacian": T.COCOWindowProgressiveLaplacianPolicy,
    "ADE20KWindowProgressiveLaplacian": T.ADE20KWindowProgressiveLaplacianPolicy,
    "FourierADE20KWindowHybrid": T.FourierADE20KWindowHybridPolicy,
    "FullImageCompression": T.FullImageCompressionPolicy,
    "FourierProgressive": T.FourierProgressiveTransmissionPolicy,
    "FourierLaplacianHybrid": T.FourierLaplacianHybridPolicy,
    "FourierLaplacianProgressive": T.FourierLaplacianProgressivePolicy,
    "NYUAppCorrFourierLaplacianHybrid": T.NYUAppCorrFourierLaplacianHybridPolicy,
    "VGGTLaplacian": T.VGGTLaplacianPolicy,
}


def get_scheduler(name: str, config: Optional[ExperimentConfig] = None) -> ISchedulingPolicy:
    cls = SCHEDULER_REGISTRY.get(name)
    if cls is None:
        raise ValueError(f"Unknown scheduler policy: {name}")
    return cls(config=config)


def get_transmission(name: str) -> ITransmissionPolicy:
    cls = TRANSMISSION_REGISTRY.get(name)
    if cls is None:
        raise ValueError(f"Unknown transmission policy: {name}")
    return cls()
