from .protocol import (  # noqa: F401
    ExperimentConfig,
    InferenceResult,
    Instruction,
    OpType,
    Patch,
    Task,
    default_appcorr_kwargs,
    normalize_appcorr_kwargs,
)
from .network import recv_msg, send_msg  # noqa: F401
from .config_overrides import apply_config_overrides, parse_override_value  # noqa: F401
