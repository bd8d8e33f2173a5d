import pytest

from graspo_b200.core.buffer import Experience, ReplayBuffer
from graspo_b200.core.decisions import (
    GroupDecision,
    classify_group,
    group_advantages,
    has_reward_variance,
    lower_median,
    replay_ready,
)


def _c(rewards, contents=None, retry=0, max_retries=2, **kw):
    return classify_group(rewards, contents or [0.0] * len(rewards), retry_count=retry, rollout_max_retries=max_retries, **kw).decision


def test_lower_median_and_advantages():
    assert lower_median([3, 1, 2, 4]) == 2
    adv = group_advantages([1.0, 0.0, 0.0, 1.0])
    assert adv[0] == pytest.approx(-adv[1]) and sum(adv) == pytest.approx(0.0)
    assert group_advantages([0.5]) == [0.0]
    assert group_advantages([1.0, 0.0], eps=1e-4)[0] == pytest.approx(0.5 / (0.7071067811865476 + 1e-4))


def test_decision_table():
    assert _c([1.0, 1.0, 1.1]) == GroupDecision.PERFECT_SKIP
    assert _c([0.1, 0.2, 1.0]) == GroupDecision.TRAINABLE_MAX_CORRECT
    assert _c([0.1, 0.2, 0.5]) == GroupDecision.TRAINABLE_NOT_CORRECT
    assert _c([0.2, 0.2, 0.2]) == GroupDecision.RETRY
    assert _c([0.2, 0.2, 0.2], retry=2) == GroupDecision.INVALID
    assert _c([0.1, 0.2, 0.5], best_completion_has_parse_error=True) == GroupDecision.RETRY
    assert _c([0.1, 0.2, 0.5], retry=2, best_completion_has_parse_error=True) == GroupDecision.INVALID
    assert _c([0.1, 0.2, 0.5], best_completion_has_parse_error=True, reject_unparseable_groups=False) == GroupDecision.TRAINABLE_NOT_CORRECT
    # no variance at all but content differs: max == median after retries exhausted
    assert _c([0.3, 0.5, 0.5], contents=[0.0, 0.2, 0.3], retry=2) == GroupDecision.INVALID_NO_PREFERENCE_GAP
    assert classify_group([], [], retry_count=0, rollout_max_retries=1).decision == GroupDecision.INVALID


def test_should_train_flags():
    d = classify_group([0.1, 1.0], [0.0, 1.0], retry_count=0, rollout_max_retries=1)
    assert d.should_train and not d.should_retry and d.reward_max_median_gap == pytest.approx(0.9)
    assert has_reward_variance([0.0, 1e-9]) and not has_reward_variance([1.0])


def test_replay_buffer():
    buf = ReplayBuffer()
    buf.append_many([Experience(i, None, None, None, None, None) for i in range(5)])
    assert len(buf) == 5 and [e.sequences for e in buf.take(3)] == [0, 1, 2]
    assert replay_ready(len(buf), 2, 2) and not replay_ready(3, 2, 2)
    limited = ReplayBuffer(limit=2)
    limited.append_many([Experience(i, None, None, None, None, None) for i in range(5)])
    assert [e.sequences for e in limited.items] == [3, 4]
    buf.clear()
    assert len(buf) == 0


# (rewards, content scores, retry_count, rollout_max_retries, extra flags) -> decision.
# Priority order exercised: perfect skip (lower median at the threshold) > max correct >
# unparseable-best retry/discard > preference gap (max above the lower median) > retry while
# attempts remain > invalid filters (no variance, uniform partial content) > no preference gap.
_SCENARIOS = [
    ([1.0, 1.0, 1.0, 0.5], [1.0, 1.0, 1.0, 0.5], 0, 5, {}, GroupDecision.PERFECT_SKIP),
    ([1.0, 1.0, 1.0, 1.0], [1.0] * 4, 1, 5, {}, GroupDecision.PERFECT_SKIP),
    ([0.5, 0.5, 0.5, 1.0], [0.5, 0.5, 0.5, 1.0], 1, 5, {}, GroupDecision.TRAINABLE_MAX_CORRECT),
    ([0.1, 1.0], [0.1, 1.0], 1, 5, {}, GroupDecision.TRAINABLE_MAX_CORRECT),
    ([0.2, 0.2], [0.2, 0.2], 0, 1, {}, GroupDecision.RETRY),
    ([0.2, 0.2], [0.2, 0.2], 1, 1, {}, GroupDecision.INVALID),
    ([0.1, 0.2], [0.1, 0.2], 0, 5, {}, GroupDecision.TRAINABLE_NOT_CORRECT),
    ([0.1, 0.2, 0.2, 0.2], [0.0, 0.8, 0.8, 0.8], 5, 5, {}, GroupDecision.INVALID_NO_PREFERENCE_GAP),
    ([0.1, 0.2, 0.2, 0.3], [0.0, 0.8, 0.8, 0.9], 5, 5, {}, GroupDecision.TRAINABLE_NOT_CORRECT),
    # a preference gap trains even when every completion has the same partial content score
    ([0.1, 0.2, 0.2, 0.3], [0.8] * 4, 5, 5, {}, GroupDecision.TRAINABLE_NOT_CORRECT),
    # no reward variance is invalid, ahead of "no preference gap"
    ([0.2] * 4, [0.5] * 4, 5, 5, {}, GroupDecision.INVALID),
    ([0.1, 0.2], [0.1, 0.2], 0, 5, {"best_completion_has_parse_error": True}, GroupDecision.RETRY),
    ([0.1, 0.2], [0.1, 0.2], 5, 5, {"best_completion_has_parse_error": True}, GroupDecision.INVALID),
    ([0.1, 0.2], [0.1, 0.2], 5, 5, {"best_completion_has_parse_error": True, "reject_unparseable_groups": False},
     GroupDecision.TRAINABLE_NOT_CORRECT),
    # a lower perfect-skip threshold moves the boundary
    ([0.8, 0.9, 0.9], [0.8, 0.9, 0.9], 0, 5, {"perfect_skip_reward_threshold": 0.85}, GroupDecision.PERFECT_SKIP),
]


@pytest.mark.parametrize("rewards,content,retry,max_retries,flags,expected", _SCENARIOS)
def test_decision_priority(rewards, content, retry, max_retries, flags, expected):
    d = classify_group(rewards, content, retry_count=retry, rollout_max_retries=max_retries, **flags)
    assert d.decision == expected
    assert d.should_train == (expected in (GroupDecision.TRAINABLE_MAX_CORRECT, GroupDecision.TRAINABLE_NOT_CORRECT))
    assert d.should_retry == (expected == GroupDecision.RETRY)
    assert d.reward_max_median_gap == pytest.approx(max(rewards) - lower_median(rewards))


def test_invalid_filters():
    from graspo_b200.core.decisions import is_invalid_group, is_uniform_partial_content

    assert is_invalid_group([0.0, 0.0], [0.0, 0.0])
    assert is_invalid_group([0.2, 0.8], [0.5, 0.5])           # uniform partial content
    assert not is_invalid_group([0.1, 0.2, 0.2, 0.2], [0.0, 0.8, 0.8, 0.8])
    assert is_uniform_partial_content([0.5, 0.5, 0.5])
    assert not is_uniform_partial_content([0.0, 0.0]) and not is_uniform_partial_content([1.0, 1.0])
    assert not is_uniform_partial_content([])


def test_replay_threshold_is_prompts_times_group():
    from graspo_b200.core.decisions import replay_buffer_optimize_threshold

    assert replay_buffer_optimize_threshold(4, 8) == 32
    assert replay_ready(32, 4, 8) and not replay_ready(31, 4, 8)
