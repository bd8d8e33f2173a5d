"""Host phase clocks for the training and pipeline loops.

``PhaseClock`` sums wall-clock seconds per key (``with clock.time(key):``)
and counts calls.  With ``sync=True`` (``graspoflow.synchronize_cuda_timing``)
the current CUDA device is synchronised before each clock read, so a phase
covers its device work rather than only the launches.  ``NULL_CLOCK`` is the
do-nothing clock used when a caller asks for no timing.

Key names follow the reference's train metrics so its log analysis carries
over (reference: tensor_utils.py:246-288 pipeline stage keys,
qwen35_36/training.py:143-148 and 789-793 train-batch keys).
"""

from __future__ import annotations

import time
from collections import defaultdict
from contextlib import contextmanager
from typing import Iterator

import torch


class PhaseClock:
    def __init__(self, *, sync: bool = False) -> None:
        self.sync = bool(sync) and torch.cuda.is_available()
        self.sec: dict[str, float] = defaultdict(float)
        self.calls: dict[str, int] = defaultdict(int)
        self.peaks: dict[str, int] = {}

    def now(self) -> float:
        if self.sync:
            torch.cuda.synchronize()
        return time.monotonic()

    @contextmanager
    def time(self, key: str) -> Iterator[None]:
        t0 = self.now()
        try:
            yield
        finally:
            self.sec[key] += self.now() - t0
            self.calls[key] += 1

    def add(self, key: str, seconds: float) -> None:
        self.sec[key] += seconds

    def peak(self, key: str, value: int) -> None:
        """Keep the largest ``value`` seen under ``key``."""
        self.peaks[key] = max(int(value), self.peaks.get(key, int(value)))

    def summary(self, *, digits: int = 6) -> dict[str, float]:
        return {k: round(v, digits) for k, v in sorted(self.sec.items()) if v}


class _NullClock(PhaseClock):
    @contextmanager
    def time(self, key: str) -> Iterator[None]:
        yield

    def now(self) -> float:
        return 0.0

    def add(self, key: str, seconds: float) -> None:
        return None

    def peak(self, key: str, value: int) -> None:
        return None


NULL_CLOCK = _NullClock()


def schedule_phases(scheduler, chunk_count: int, max_inflight: int | None = None) -> list[tuple[str, object]]:
    """(phase, step) pairs of a pipeline plan: ``fill`` / ``steady`` / ``drain``
    for 1F1B; GPipe's all-forwards run as ``fill`` and its backwards as ``drain``.
    ``max_inflight`` (> 0) caps the 1F1B warm-up forwards, and with them the
    micro-batches whose activations a stage holds at once."""
    phases = scheduler.plan_phases(chunk_count, max_inflight=max_inflight or None)
    rename = {"forward": "fill", "backward": "drain", "all": "steady"}
    return [(rename.get(name, name), step) for name, steps in phases.items() for step in steps]


__all__ = ["PhaseClock", "NULL_CLOCK", "schedule_phases"]
