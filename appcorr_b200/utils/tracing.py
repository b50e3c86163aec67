"""Lightweight device-side phase timing and NVTX ranges.

`PhaseTimer` records a CUDA event pair on the current stream around each named phase and sums
the device time per name when `summary()` is called (it synchronises once, at the end). It is a
no-op unless enabled, so engines can wrap every phase unconditionally. The NVTX ranges use the
reference's naming (`APPCORR_SESSION|...`, `APPCORR_INSTR|...`; worker.py:509-525 in the
reference) so an nsys timeline lines up instruction by instruction.
"""
from __future__ import annotations

import contextlib
import os
from collections import defaultdict
from typing import Dict, List, Tuple

import torch


class PhaseTimer:
    def __init__(self, enabled: bool = False):
        self.enabled = enabled
        self._pairs: List[Tuple[str, torch.cuda.Event, torch.cuda.Event]] = []

    @classmethod
    def from_env(cls, var: str = "APPCORR_PHASE_TIMING") -> "PhaseTimer":
        return cls(os.environ.get(var, "0") not in ("", "0", "false", "False"))

    @contextlib.contextmanager
    def __call__(self, name: str):
        if not self.enabled:
            yield
            return
        s, e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        s.record()
        try:
            yield
        finally:
            e.record()
            self._pairs.append((name, s, e))

    def summary(self, reset: bool = True) -> Dict[str, float]:
        """Total milliseconds per phase name (device time)."""
        if not self._pairs:
            return {}
        torch.cuda.synchronize()
        out: Dict[str, float] = defaultdict(float)
        for name, s, e in self._pairs:
            out[name] += s.elapsed_time(e)
        if reset:
            self._pairs = []
        return dict(out)


@contextlib.contextmanager
def nvtx_range(name: str):
    """NVTX range (visible in nsys) around a host-side region; no-op without CUDA."""
    if torch.cuda.is_available():
        torch.cuda.nvtx.range_push(name)
        try:
            yield
        finally:
            torch.cuda.nvtx.range_pop()
    else:
        yield
