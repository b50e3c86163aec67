"""Wire-level data model shared by the mobile client and the server.

The field names, defaults and enum members follow the reference protocol so existing experiment
JSON files and client code keep working (reference offload/common/protocol.py:184-415). The
AppCorr option normaliser implements the same aliases and validation rules
(protocol.py:6-181) in a table-driven form.
"""
from __future__ import annotations

import os

from dataclasses import dataclass, field
from enum import Enum, auto
from typing import Any, Dict, List, Optional, Tuple

# ----------------------------------------------------------------------------- AppCorr options

_APPCORR_DEFAULTS: Dict[str, Any] = {
    "enabled": False,
    "generated_from_client": False,
    "global_source_mode": "global_first",
    "update_attn": False,
    "pyramid_levels": [0],
    "token_res": [1.0],
    "plan": [],
    "num_groups": 1,
    "group_strategy": "uniform",
    "token_keep_ratio": 0.2,
    "token_keep_thres": None,
    "token_keep_cap": 0,
    "attn_col_alive_ratio": 1.0,
    "mobile_pscore": "none",
    "mobile_pscore_weight": 0.0,
    "server_pscore": "cls_attn_prob",
    "server_pscore_weight": 1.0,
    "pscore_fusion": "add",
    "sdpa_query_bucket_size": 0,
    "sdpa_warmup": True,
    "sdpa_warmup_runs": 2,
    "correct_warmup_runs": 1,
    "token_prune_enabled": False,
    "token_prune_threshold": 0.0,
    "token_prune_min_keep": 1,
    "method": "partial_token",
    "debug": False,
}

# Server-side patch score names the correction pass understands. "random" is a control.
VALID_SERVER_PSCORES = frozenset({
    "cls_attn_prob",
    "patch_attn_prob",
    "patch_attn_prob_layermean",
    "patch_pseudo_attn_prob",
    "patch_pseudo_attn_prob_layermean",
    "cls_attn_prob_layermean",
    "random",
})
LAYERMEAN_SERVER_PSCORES = frozenset({
    "patch_attn_prob_layermean",
    "patch_pseudo_attn_prob_layermean",
    "cls_attn_prob_layermean",
})

_MOBILE_PSCORE_ALIAS = {
    "residual_rms": "residual_rms",
    "patch_residual_rms": "residual_rms",
    "residual_l2": "residual_energy",
    "residual_l2_energy": "residual_energy",
    "residual_energy": "residual_energy",
    "patch_residual_l2": "residual_energy",
    "patch_residual_energy": "residual_energy",
}
_SERVER_PSCORE_ALIAS = {
    "patch_attn_prune": "patch_attn_prob",
    "pseudo_patch_attn_prob": "patch_pseudo_attn_prob",
    "pseudo_patch_attn_prob_layermean": "patch_pseudo_attn_prob_layermean",
}
_LAYERMEAN_OF = {
    "patch_attn_prob": "patch_attn_prob_layermean",
    "patch_pseudo_attn_prob": "patch_pseudo_attn_prob_layermean",
    "cls_attn_prob": "cls_attn_prob_layermean",
}
_FUSION_ALIAS = {"mul": "multiply", "product": "multiply", "geomean": "geo_mean", "geometric_mean": "geo_mean"}
_NULLS = {"", "null", "None"}


def default_appcorr_kwargs() -> Dict[str, Any]:
    out = dict(_APPCORR_DEFAULTS)
    for key in ("pyramid_levels", "token_res", "plan"):
        out[key] = list(out[key])
    return out


def _inherit_from_transmission(raw: Dict[str, Any], tx: Optional[Dict[str, Any]]) -> None:
    """pyramid_levels / num_groups are owned by the transmission policy; a conflicting copy in
    appcorr_kwargs is a configuration error."""
    if not tx:
        return
    if "pyramid_levels" in tx:
        levels = list(tx["pyramid_levels"])
        if "pyramid_levels" in raw and list(raw["pyramid_levels"]) != levels:
            raise ValueError("appcorr_kwargs.pyramid_levels must match transmission_kwargs.pyramid_levels")
        raw["pyramid_levels"] = levels
    if "num_groups" in tx:
        groups = max(int(tx["num_groups"]), 1)
        if "num_groups" in raw and max(int(raw["num_groups"]), 1) != groups:
            raise ValueError("appcorr_kwargs.num_groups must match transmission_kwargs.num_groups")
        raw["num_groups"] = groups


def _resolve_server_pscore(raw: Dict[str, Any], current: str) -> str:
    name = current
    legacy = raw.get("token_prune_score")
    if legacy is not None and "server_pscore" not in raw:
        name = str(legacy)
    if raw.get("patch_attn_prune", False) and "server_pscore" not in raw and legacy is None:
        name = "patch_attn_prob"
    name = _SERVER_PSCORE_ALIAS.get(name, name)
    layer_fusion = str(raw.get("server_pscore_layer_fusion", "")).lower()
    if layer_fusion in {"mean", "avg", "all_layer_mean", "layer_mean", "mean_all_layers"}:
        name = _LAYERMEAN_OF.get(name, name)
    if name not in VALID_SERVER_PSCORES:
        raise ValueError(f"Unknown server_pscore '{name}'. Available values: {sorted(VALID_SERVER_PSCORES)}")
    return name


def normalize_appcorr_kwargs(appcorr_kwargs: Optional[Dict[str, Any]] = None,
                             transmission_kwargs: Optional[Dict[str, Any]] = None) -> Dict[str, Any]:
    """Fill defaults, resolve aliases and validate an `appcorr_kwargs` dict.

    AppCorr counts as enabled when the caller supplied any key (unless `enabled` says otherwise).
    """
    raw = dict(appcorr_kwargs or {})
    explicit_enabled = raw.pop("enabled", None)
    any_key = bool(raw)
    _inherit_from_transmission(raw, transmission_kwargs)
    if "persist_correction_residual" in raw:
        raise ValueError(
            "appcorr_kwargs.persist_correction_residual is not a setting: the corrected per-layer "
            "increment is always written back. Remove the key."
        )
    opt = default_appcorr_kwargs()
    opt.update(raw)
    d = _APPCORR_DEFAULTS
    opt["enabled"] = any_key if explicit_enabled is None else bool(explicit_enabled)
    opt["generated_from_client"] = bool(opt["generated_from_client"])
    gsm = str(opt["global_source_mode"])
    opt["global_source_mode"] = gsm if gsm in {"global_first", "final_correct", "approx"} else d["global_source_mode"]
    opt["update_attn"] = bool(opt["update_attn"])
    opt["pyramid_levels"] = list(opt["pyramid_levels"])
    opt["token_res"] = list(opt["token_res"])
    opt["plan"] = list(opt["plan"])
    opt["num_groups"] = max(int(opt["num_groups"]), 1)
    opt["group_strategy"] = str(opt["group_strategy"])
    keep = opt["token_keep_ratio"]
    if "token_keep_ratio" not in raw and "cls_alive_ratio" in raw:
        keep = raw["cls_alive_ratio"]
    opt["token_keep_ratio"] = float(keep)
    thr = opt["token_keep_thres"]
    opt["token_keep_thres"] = None if (thr is None or thr in _NULLS) else float(thr)
    opt["token_keep_cap"] = max(0, int(opt["token_keep_cap"] or 0))
    opt["attn_col_alive_ratio"] = float(opt["attn_col_alive_ratio"])
    mp = str(opt["mobile_pscore"])
    mp = d["mobile_pscore"] if mp in _NULLS else mp
    opt["mobile_pscore"] = _MOBILE_PSCORE_ALIAS.get(mp, mp)
    opt["mobile_pscore_weight"] = float(opt["mobile_pscore_weight"])
    opt["server_pscore"] = _resolve_server_pscore(raw, str(opt["server_pscore"]))
    opt["server_pscore_weight"] = float(opt["server_pscore_weight"])
    fusion = str(opt["pscore_fusion"]).lower()
    fusion = _FUSION_ALIAS.get(fusion, fusion)
    opt["pscore_fusion"] = fusion if fusion in {"add", "multiply", "geo_mean"} else d["pscore_fusion"]
    opt["sdpa_query_bucket_size"] = max(int(opt["sdpa_query_bucket_size"] or 0), 0)
    opt["sdpa_warmup"] = bool(opt["sdpa_warmup"])
    opt["sdpa_warmup_runs"] = max(int(opt["sdpa_warmup_runs"] or 0), 0)
    opt["correct_warmup_runs"] = max(int(opt["correct_warmup_runs"] or 0), 0)
    opt["token_prune_enabled"] = bool(opt["token_prune_enabled"])
    opt["token_prune_threshold"] = float(opt["token_prune_threshold"])
    opt["token_prune_min_keep"] = max(int(opt["token_prune_min_keep"]), 1)
    opt["method"] = str(opt["method"])
    opt["debug"] = bool(opt["debug"])
    return opt


# ----------------------------------------------------------------------------- input profiles

_INPUT_PROFILES: Dict[str, Dict[str, Any]] = {
    "fixed_image_shape": {},
    "dinov3_nyu_synthmix_dpt": {
        "depther_eval_size": 768,
        "depther_use_tta": True,
        "autocast_dtype": "bfloat16",
    },
    "dinov3_ade20k_m2f_official": {
        "mobile_resize_short_side": 896,
        "server_inference_mode": "slide",
        "server_crop_size": 896,
        "server_stride": 596,
        "server_eval_mode": "tta",
        "server_rescale_to": "input",
        "server_use_tta": True,
        "server_tta_ratios": [0.9, 0.95, 1.0, 1.05, 1.1],
        "decoder_head_type": "m2f",
        "num_classes": 150,
        "autocast_dtype": "bfloat16",
        "reduce_zero_label": True,
    },
    "dinov3_ade20k_linhead_official": {
        "mobile_resize_short_side": 512,
        "server_inference_mode": "slide",
        "server_crop_size": 512,
        "server_stride": 341,
        "server_eval_mode": "single",
        "server_rescale_to": "input",
        "decoder_head_type": "linear",
        "num_classes": 150,
        "autocast_dtype": "float32",
        "reduce_zero_label": True,
    },
    "vggt_omega_512": {
        "vggt_resolution": 512,
        "vggt_patch_size": 16,
        "vggt_resize_mode": "balanced",
        "vggt_weights_path": None,  # None: random init (no checkpoint shipped)
        "autocast_dtype": "bfloat16",
    },
}


@dataclass
class ExperimentConfig:
    """One experiment, as shipped by the client in the CONFIG handshake."""

    exp_id: str = "exp"
    model_name: str = "dinov3_classifier"
    device: Optional[str] = None
    precision: str = "bf16"
    fp8_auto_min_rows: int = 3072
    correct_precision: str = "bf16"
    correct_compile: bool = False
    correct_fp4_calib_events: int = 1
    correct_fp4_proj_precision: str = "fp8"
    correct_bucket_rows: int = 0
    dataset_name: str = "imagenet-1k"
    dataset_kwargs: Dict[str, Any] = field(default_factory=dict)
    batch_size: int = 32
    image_shape: Tuple[int, int, int] = (256, 256, 3)
    patch_size: Tuple[int, int] = (16, 16)
    input_profile_name: str = "fixed_image_shape"
    input_profile_kwargs: Dict[str, Any] = field(default_factory=dict)
    scheduler_policy_name: str = "BatchCountBased"
    transmission_policy_name: str = "Raw"
    scheduler_kwargs: Dict[str, Any] = field(default_factory=dict)
    transmission_kwargs: Dict[str, Any] = field(default_factory=dict)
    appcorr_kwargs: Dict[str, Any] = field(default_factory=dict)
    # B200 build additions (ignored by clients that do not send them).
    tp_size: int = 1
    dp_size: int = 1
    kernel_backend: str = "sm100a"
    collective_timeout_us: int = 1_000_000

    def __post_init__(self) -> None:
        self.precision = str(self.precision).lower()
        if self.precision not in {"bf16", "fp8", "fp4", "auto"}:
            raise ValueError(f"precision must be one of 'bf16', 'fp8', 'fp4', or 'auto', got {self.precision!r}")
        self.fp8_auto_min_rows = int(self.fp8_auto_min_rows)
        if self.fp8_auto_min_rows <= 0:
            raise ValueError(f"fp8_auto_min_rows must be positive, got {self.fp8_auto_min_rows}")
        self.correct_precision = str(self.correct_precision).lower()
        if self.correct_precision not in {"bf16", "fp8", "fp4"}:
            raise ValueError(f"correct_precision must be one of 'bf16', 'fp8', or 'fp4', got {self.correct_precision!r}")
        self.correct_compile = bool(self.correct_compile)
        self.correct_fp4_calib_events = max(0, int(self.correct_fp4_calib_events))
        self.correct_bucket_rows = max(0, int(self.correct_bucket_rows))
        if self.correct_fp4_proj_precision not in {"fp4", "fp8"}:
            raise ValueError(f"correct_fp4_proj_precision must be 'fp4' or 'fp8', got {self.correct_fp4_proj_precision!r}")
        self.image_shape = tuple(self.image_shape)
        self.patch_size = tuple(self.patch_size)
        self.tp_size = max(1, int(self.tp_size))
        self.dp_size = max(1, int(self.dp_size))
        if self.kernel_backend not in {"sm100a", "nccl_baseline", "cpu"}:
            raise ValueError(f"kernel_backend must be 'sm100a', 'nccl_baseline' or 'cpu', got {self.kernel_backend!r}")

    def get_input_profile_config(self) -> Dict[str, Any]:
        name = self.input_profile_name or "fixed_image_shape"
        if name not in _INPUT_PROFILES:
            raise ValueError(f"Unknown input_profile_name: {name}")
        opts = {"name": name, **_INPUT_PROFILES[name]}
        opts.update(self.input_profile_kwargs)
        return opts

    def use_official_ade20k_m2f_profile(self) -> bool:
        return (self.input_profile_name or "fixed_image_shape") == "dinov3_ade20k_m2f_official"

    def early_exit_enabled(self) -> bool:
        return bool(self.scheduler_kwargs.get("early_exit", False))

    def get_early_exit_config(self) -> Dict[str, Any]:
        return {k: v for k, v in self.scheduler_kwargs.items() if k in {"metric", "threshold"}}

    def lowres_sr_enabled(self) -> bool:
        return bool(self.scheduler_kwargs.get("lowres_sr", False))

    def get_lowres_sr_config(self) -> Dict[str, Any]:
        sk = self.scheduler_kwargs
        return {
            "model": sk.get("lowres_sr_model", "realesrgan_x4plus"),
            "dtype": sk.get("lowres_sr_dtype", "fp16"),
            "weights_dir": sk.get("lowres_sr_weights_dir", os.environ.get("APPCORR_SR_WEIGHTS_DIR")),
            "tile": sk.get("lowres_sr_tile", 0),
            "tile_pad": sk.get("lowres_sr_tile_pad", 10),
            "pre_pad": sk.get("lowres_sr_pre_pad", 0),
        }


@dataclass
class Patch:
    image_idx: int
    spatial_idx: int
    data: bytes
    res_level: int = 0
    group_id: int = 0
    batch_group_total: int = 0
    arrival_time: float = 0.0
    pscore_hint: float = 0.0
    target_shape: tuple = ()
    num_correction_groups: int = 0
    text_payload: str = ""


class OpType(Enum):
    # compute
    FULL_INFERENCE = auto()
    APPROX_FORWARD = auto()
    CORRECT_FORWARD = auto()
    HEAD_INFERENCE = auto()
    # control
    LOAD_INPUT = auto()
    PREPARE_TOKENS = auto()
    SEND_RESPONSE = auto()
    FREE_SESSION = auto()
    TIME_SYNC = auto()
    DECIDE_EXIT = auto()
    EXIT_ALL = auto()


@dataclass
class Instruction:
    op_type: OpType
    params: Dict[str, Any] = field(default_factory=dict)


@dataclass
class Task:
    task_id: int
    request_id: int
    payload: List[Patch]
    instructions: List[Instruction]


@dataclass
class InferenceResult:
    task_id: int
    timestamp: float
    output: Any
    server_events: List[Dict[str, Any]] = field(default_factory=list)
    cache_size_bytes: int = 0
    cache_breakdown_bytes: Dict[str, int] = field(default_factory=dict)
    attn_prob_mass_used: float = 0.0
    attn_prob_mass_full: float = 0.0
    token_prune_kept_patch: float = 0.0
    token_prune_full_patch: float = 0.0
    token_prune_kept_residual_mass: float = 0.0
    token_prune_full_residual_mass: float = 0.0
    token_pscore_kept_mass: float = 0.0
    token_pscore_full_mass: float = 0.0
    partial_token_kept_patch: float = 0.0
    partial_token_full_patch: float = 0.0
    partial_token_sample_count: float = 0.0
