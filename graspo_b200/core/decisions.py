"""Group decisions and group-normalised advantages.

A "group" is the ``G`` completions sampled for one prompt.  The decision table
(reference: src/graspo/core/graspo_parity.py:80-151) is evaluated top to bottom
with the *lower* median:

1. median >= threshold                       -> PERFECT_SKIP (nothing to learn)
2. max >= threshold                          -> TRAINABLE_MAX_CORRECT
3. best completion unparseable (if rejecting) -> RETRY while retries remain, else INVALID
4. max > median                              -> TRAINABLE_NOT_CORRECT
5. retries remain                            -> RETRY
6. no reward variance / uniform partial content -> INVALID
7. max == median                             -> INVALID_NO_PREFERENCE_GAP

Advantages are ``(r - mean) / (std + eps)`` with the unbiased std; ``eps`` is
configurable (reference default 1e-8).
"""

from __future__ import annotations

from collections.abc import Sequence
from dataclasses import dataclass
from enum import StrEnum


class GroupDecision(StrEnum):
    PERFECT_SKIP = "perfect_skip"
    RETRY = "retry"
    INVALID = "invalid"
    INVALID_NO_PREFERENCE_GAP = "invalid_no_preference_gap"
    TRAINABLE_MAX_CORRECT = "trainable_max_correct"
    TRAINABLE_NOT_CORRECT = "trainable_not_correct"


TRAINABLE = frozenset({GroupDecision.TRAINABLE_MAX_CORRECT, GroupDecision.TRAINABLE_NOT_CORRECT})


@dataclass(frozen=True, slots=True)
class GroupSampleDecision:
    decision: GroupDecision
    reward_min: float
    reward_median: float
    reward_max: float
    reward_mean: float
    content_mean: float | None
    retry_count: int

    @property
    def should_retry(self) -> bool:
        return self.decision == GroupDecision.RETRY

    @property
    def should_train(self) -> bool:
        return self.decision in TRAINABLE

    @property
    def reward_max_median_gap(self) -> float:
        return self.reward_max - self.reward_median


def lower_median(values: Sequence[float]) -> float:
    if not values:
        return 0.0
    ordered = sorted(float(v) for v in values)
    return ordered[(len(ordered) - 1) // 2]


def group_advantages(rewards: Sequence[float], eps: float = 1e-8) -> list[float]:
    values = [float(r) for r in rewards]
    n = len(values)
    if n == 0:
        return []
    mean = sum(values) / n
    std = (sum((v - mean) ** 2 for v in values) / (n - 1)) ** 0.5 if n > 1 else 0.0
    return [(v - mean) / (std + eps) for v in values]


def has_reward_variance(rewards: Sequence[float], eps: float = 1e-12) -> bool:
    if len(rewards) < 2:
        return False
    values = [float(r) for r in rewards]
    return max(values) - min(values) > eps


def is_uniform_partial_content(content_scores: Sequence[float]) -> bool:
    """All completions earned the same content score strictly between 0 and 1."""
    if not content_scores:
        return False
    values = [float(s) for s in content_scores]
    return 0.0 < min(values) == max(values) < 1.0


def is_invalid_group(rewards: Sequence[float], content_scores: Sequence[float]) -> bool:
    return not has_reward_variance(rewards) or is_uniform_partial_content(content_scores)


def classify_group(
    rewards: Sequence[float],
    content_scores: Sequence[float],
    *,
    retry_count: int,
    rollout_max_retries: int,
    perfect_skip_reward_threshold: float = 1.0,
    best_completion_has_parse_error: bool = False,
    reject_unparseable_groups: bool = True,
) -> GroupSampleDecision:
    values = [float(r) for r in rewards]
    if not values:
        return GroupSampleDecision(GroupDecision.INVALID, 0.0, 0.0, 0.0, 0.0, None, retry_count)
    lo, hi, med = min(values), max(values), lower_median(values)
    mean = sum(values) / len(values)
    content_mean = (
        sum(float(s) for s in content_scores) / len(content_scores) if content_scores else None
    )
    can_retry = retry_count < rollout_max_retries
    thr = perfect_skip_reward_threshold
    if med >= thr:
        decision = GroupDecision.PERFECT_SKIP
    elif hi >= thr:
        decision = GroupDecision.TRAINABLE_MAX_CORRECT
    elif reject_unparseable_groups and best_completion_has_parse_error:
        decision = GroupDecision.RETRY if can_retry else GroupDecision.INVALID
    elif hi > med:
        decision = GroupDecision.TRAINABLE_NOT_CORRECT
    elif can_retry:
        decision = GroupDecision.RETRY
    elif is_invalid_group(values, content_scores):
        decision = GroupDecision.INVALID
    elif hi == med:
        decision = GroupDecision.INVALID_NO_PREFERENCE_GAP
    else:
        decision = GroupDecision.INVALID
    return GroupSampleDecision(decision, lo, med, hi, mean, content_mean, retry_count)


def replay_buffer_optimize_threshold(optimize_prompt_batch_size: int, rollout_group_size: int) -> int:
    return int(optimize_prompt_batch_size) * int(rollout_group_size)


def replay_ready(replay_size: int, optimize_prompt_batch_size: int, rollout_group_size: int) -> bool:
    return int(replay_size) >= replay_buffer_optimize_threshold(
        optimize_prompt_batch_size, rollout_group_size
    )
