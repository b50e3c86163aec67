"""Loader for the in-tree sm_100a extension (`appcorr_b200/_C*.so`).

The extension is built by `python setup.py build_ext --inplace` (or `__graft_entry__.build()`).
Importing it is lazy so that CPU-only code paths (protocol, policies, the CPU oracle) work on a
machine without the build; any GPU op raises immediately and loudly when the library is absent,
so a GPU run can never silently fall back to eager PyTorch.
"""
from __future__ import annotations

import threading

import torch

_C = None
_IMPORT_ERROR: Exception | None = None
_LOCK = threading.Lock()
_ERR_WORDS: dict[int, torch.Tensor] = {}

ERROR_NAMES = {
    0: "ok",
    1: "producer wait timed out",
    2: "MMA wait timed out",
    3: "epilogue wait timed out",
    4: "peer wait timed out",
    5: "bad shape",
}


def lib():
    """Return the native module, importing it on first use; raise if it is not built."""
    global _C, _IMPORT_ERROR
    if _C is None:
        with _LOCK:
            if _C is None:
                try:
                    from appcorr_b200 import _C as mod  # noqa: WPS433
                except ImportError as exc:  # pragma: no cover - depends on the build
                    _IMPORT_ERROR = exc
                    raise RuntimeError(
                        "appcorr_b200 native extension is not built "
                        f"({exc}); run `python setup.py build_ext --inplace`"
                    ) from exc
                _C = mod
    return _C


def available() -> bool:
    try:
        lib()
        return True
    except RuntimeError:
        return False


def err_word(device: torch.device) -> torch.Tensor:
    """Per-device int32 word that kernels set when a bounded wait expires."""
    idx = device.index if device.index is not None else torch.cuda.current_device()
    t = _ERR_WORDS.get(idx)
    if t is None:
        t = torch.zeros(1, dtype=torch.int32, device=torch.device("cuda", idx))
        _ERR_WORDS[idx] = t
    return t


def check_errors(device: torch.device | None = None) -> None:
    """Raise if any kernel on `device` recorded a timeout. Synchronises with the host."""
    devs = [device] if device is not None else [torch.device("cuda", i) for i in _ERR_WORDS]
    for d in devs:
        w = err_word(d)
        code = int(w.item())
        if code != 0:
            w.zero_()
            raise RuntimeError(f"appcorr_b200 kernel error on {d}: {ERROR_NAMES.get(code, code)}")
