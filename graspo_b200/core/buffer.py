"""Completion-level replay buffer.

Reference counterpart: src/graspo/core/buffer.py:5-36.  ``Experience`` is the
record both runtimes exchange (``train_batch`` consumes a list of them), so
its fields and their order are kept as the reference defines them; the buffer
around it is a bounded FIFO of host-side records that the trainer fills with
finalized groups and drains after every optimize step.
"""

from __future__ import annotations

from collections import deque
from collections.abc import Iterable
from dataclasses import dataclass
from itertools import islice
from typing import Any


@dataclass(slots=True)
class Experience:
    sequences: Any
    old_log_probs: Any
    advantages: Any
    attention_mask: Any
    action_mask: Any
    rewards: Any
    metadata: dict[str, Any] | None = None


class ReplayBuffer:
    """FIFO of experiences waiting for an optimize step.

    ``limit`` > 0 bounds the buffer: appending past it drops the oldest
    records.  ``take(n)`` returns the oldest ``n`` without removing them;
    ``consume(n)`` removes them once they have been trained on."""

    def __init__(self, limit: int = 0) -> None:
        self.limit = max(0, int(limit))
        self._fifo: deque[Experience] = deque(maxlen=self.limit or None)

    @property
    def items(self) -> list[Experience]:
        """A snapshot of the buffered records, oldest first."""
        return list(self._fifo)

    def append_many(self, records: Iterable[Experience]) -> None:
        self._fifo.extend(records)

    def take(self, count: int) -> list[Experience]:
        return list(islice(self._fifo, max(0, int(count))))

    def consume(self, count: int) -> None:
        for _ in range(min(max(0, int(count)), len(self._fifo))):
            self._fifo.popleft()

    def clear(self) -> None:
        self._fifo.clear()

    def __len__(self) -> int:
        return len(self._fifo)

    def __getitem__(self, index: int) -> Experience:
        return self._fifo[index]
