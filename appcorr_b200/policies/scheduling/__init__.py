from .policies import (  # noqa: F401
    ADE20KApproxCorrectPolicy,
    ADE20KInterleavedDynamicPolicy,
    ADE20KSequentialPolicy,
    ADE20KWindowInterleavedPolicy,
    BatchCountBasedPolicy,
    COCOWindowDynamicPolicy,
    COCOWindowInterleavedPolicy,
    DynamicGroupTriggerPolicy,
    GroupTriggerPolicy,
    NYUApproxCorrectPolicy,
    VGGTInterleavedPolicy,
)
