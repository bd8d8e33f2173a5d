"""Completion-level replay buffer (reference: src/graspo/core/buffer.py:5-36).

Experiences hold host tensors so the device keeps only what the current step
needs; the buffer is drained after every optimize step.
"""

from __future__ import annotations

from dataclasses import dataclass
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
    def __init__(self, limit: int = 0) -> None:
        self.limit = int(limit)
        self.items: list[Experience] = []

    def append_many(self, items: list[Experience]) -> None:
        self.items.extend(items)
        if self.limit > 0 and len(self.items) > self.limit:
            del self.items[: len(self.items) - self.limit]

    def take(self, count: int) -> list[Experience]:
        """The ``count`` oldest experiences (not removed)."""
        return self.items[:count]

    def clear(self) -> None:
        self.items.clear()

    def __len__(self) -> int:
        return len(self.items)

    def __getitem__(self, index: int) -> Experience:
        return self.items[index]
