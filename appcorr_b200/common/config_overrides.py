"""`--set a.b.c=value` overrides applied to a config dict before it becomes an ExperimentConfig.

Values parse as JSON when possible, with `none`/`true`/`false` accepted case-insensitively and
anything else kept as the raw string (reference offload/common/config_overrides.py:5-40).
"""
from __future__ import annotations

import json
from typing import Any, Iterable, Optional

_LITERALS = {"none": None, "true": True, "false": False}


def parse_override_value(raw: str) -> Any:
    text = raw.strip()
    low = text.lower()
    if low in _LITERALS:
        return _LITERALS[low]
    try:
        return json.loads(text)
    except json.JSONDecodeError:
        return raw


def apply_config_overrides(config_data: dict, overrides: Optional[Iterable[str]]) -> None:
    for item in overrides or []:
        key_path, sep, raw_value = item.partition("=")
        if not sep:
            raise ValueError(f"Config override must be KEY=VALUE, got: {item}")
        keys = [k for k in key_path.split(".") if k]
        if not keys:
            raise ValueError(f"Config override key is empty: {item}")
        node = config_data
        for k in keys[:-1]:
            nxt = node.get(k)
            if nxt is None:
                nxt = node[k] = {}
            if not isinstance(nxt, dict):
                raise ValueError(f"Cannot set {key_path}: {k} is {type(nxt).__name__}, not an object")
            node = nxt
        node[keys[-1]] = parse_override_value(raw_value)
