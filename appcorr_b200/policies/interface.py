"""Policy interfaces: when the server computes (scheduling) and how images travel (transmission).

Same call signatures as the reference (offload/policies/interface.py:7-39), so third-party
policies written against it plug into this runtime unchanged.
"""
from __future__ import annotations

from abc import ABC, abstractmethod
from typing import Any, Generator, List, Optional

import numpy as np

from ..common.protocol import ExperimentConfig, Patch, Task


class ISchedulingPolicy(ABC):
    def __init__(self, config: Optional[ExperimentConfig] = None):
        pass

    @abstractmethod
    def decide(self, buffer: List[Patch], config: ExperimentConfig, task_id_gen: Any, **kwargs) -> Optional[Task]:
        """Return a Task when the buffered patches allow progress, else None.

        The caller removes `len(task.payload)` patches from the front of `buffer` afterwards; a
        policy must not consume them itself. `feedback_events` (kwargs) lists approximate-pass
        layer indices completed since the last call.
        """


class ITransmissionPolicy(ABC):
    @abstractmethod
    def encode(self, image: np.ndarray, config: ExperimentConfig) -> Generator[List[Patch], None, None]:
        """Yield the image as successive groups of patches (group 0 first)."""

    @abstractmethod
    def decode(self, patches: List[Patch], config: ExperimentConfig) -> np.ndarray:
        """Reconstruct the image(s) from every patch received so far."""

    def decode_lowres(self, patches: List[Patch], config: ExperimentConfig) -> Optional[np.ndarray]:
        return None
