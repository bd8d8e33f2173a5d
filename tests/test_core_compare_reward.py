"""Reward and structured-compare behaviour (golden values from the reference's tests)."""

import pytest

from graspo_b200.core.compare import dict_compare_score
from graspo_b200.core.completion import ParsedCompletion
from graspo_b200.core.reward import GraspoReward, RewardConfig, normalize_targets


def _content(*contents):
    return [{"id": f"target-{i}", "output": {"content": c}} for i, c in enumerate(contents)]


def _tools(*calls):
    return [{"id": f"target-{i}", "output": {"tool_calls": list(c)}} for i, c in enumerate(calls)]


def test_compare_exact_and_partial():
    exact = dict_compare_score({"a": 1, "b": [1, 2]}, {"a": 1, "b": [1, 2]})
    assert exact.dcs == 1.0 and exact.total_score == exact.check_score
    part = dict_compare_score({"a": 1, "b": [1]}, {"a": 1, "b": [1, 2]})
    assert 0 < part.dcs < 1


def test_compare_list_order():
    un = dict_compare_score({"items": [2, 1]}, {"items": [1, 2]}, check_list_order=False)
    ordered = dict_compare_score({"items": [2, 1]}, {"items": [1, 2]}, check_list_order=True)
    assert un.dcs > ordered.dcs


def test_compare_numeric_leaf():
    r = dict_compare_score({"distance_cm": 8}, {"distance_cm": 6})
    assert r.total_score == 3
    assert r.check_score == pytest.approx(2 + 1 / 3)
    assert (r.base_total, r.base_check, r.base_dcs, r.all_right) == (1, 1.0, 1.0, True)


def test_compare_type_mismatches():
    s = dict_compare_score({"distance_cm": "6"}, {"distance_cm": 6})
    assert (s.total_score, s.check_score, s.base_total, s.base_check, s.all_right) == (3, 2, 1, 0.0, False)
    b = dict_compare_score({"enabled": True}, {"enabled": 1})
    assert (b.total_score, b.check_score, b.base_total, b.base_check) == (3, 2, 1, 0.0)
    assert dict_compare_score({"d": 6}, {"d": 6.0}).all_right


def test_compare_nested_list_dicts():
    r = dict_compare_score(
        {"tool_calls": [{"name": "move", "arguments": {"distance_cm": 8}}]},
        {"tool_calls": [{"name": "move", "arguments": {"distance_cm": 6}}]},
        check_list_order=True,
    )
    assert r.total_score == 11
    assert r.check_score == pytest.approx(25 / 3)
    assert (r.base_total, r.base_check, r.all_right) == (7, 7.0, True)


def test_reward_perfect_fence_exceeds_one():
    reward = GraspoReward(RewardConfig(check_json_markdown=True))
    r = reward.score('```json\n{"APN":"cmnet","fault_number":"138"}\n```', _content({"APN": "cmnet", "fault_number": "138"}))
    assert r.all_right and r.content_score == 1.0 and r.matched_target_index == 0
    assert r.max_score == 230.0 and r.raw_score == 231.0 and r.reward > 1.0


def test_reward_partial_and_numeric():
    reward = GraspoReward(RewardConfig(check_json_markdown=True))
    part = reward.score('```json\n{"APN":"wrong","fault_number":"138"}\n```', _content({"APN": "cmnet", "fault_number": "138"}))
    assert not part.all_right and 0 < part.content_score < 1 and 0 < part.reward < 1
    num = reward.score('```json\n{"action":"left","distance_cm":8}\n```', _content({"action": "left", "distance_cm": 6}))
    assert num.all_right and num.content_score == pytest.approx((4 + 1 / 3) / 5)


def test_reward_ordering_good_wrong_unfenced():
    reward = GraspoReward(RewardConfig())
    targets = _content({"name": "alice", "age": "30"})
    good = reward.score('```json\n{"name": "alice", "age": "30"}\n```', targets).reward
    wrong = reward.score('```json\n{"name": "bob", "age": "31"}\n```', targets).reward
    unfenced = reward.score('{"name": "alice", "age": "30"}', targets).reward
    verbose = reward.score("x" * 300 + '```json\n{"name": "alice", "age": "30"}\n```', targets).reward
    assert good > wrong > unfenced
    assert verbose < good


def test_reward_unclosed_fence_keeps_answer_text():
    reward = GraspoReward(RewardConfig())
    r = reward.score('```json\n{"a": "b"}', _content({"a": "b"}))
    assert r.extracted.get("answer") == '\n{"a": "b"}'
    # only the opening marker is found, yet the trailing JSON is still scored
    assert r.raw_score == pytest.approx(10 + 10 + 100 + 100 + 1.0)


def test_reward_selects_best_target():
    reward = GraspoReward(RewardConfig())
    r = reward.score('```json\n{"action":"down","distance_cm":5}\n```', _content({"action": "up", "distance_cm": 5}, {"action": "down", "distance_cm": 5}))
    assert r.matched_target_index == 1 and r.matched_target_id == "target-1" and r.all_right


def test_reward_tool_call_path():
    reward = GraspoReward(RewardConfig())
    parsed = ParsedCompletion(raw_text="<tool_call>...</tool_call>", tool_calls=[{"name": "move", "arguments": {"d": 3}}])
    r = reward.score_parsed(parsed, _tools([{"name": "move", "arguments": {"d": 3}}]), is_tool_call=True)
    assert r.all_right and r.content_score == 1.0
    assert r.max_score == 210.0 and r.raw_score == pytest.approx(10 + 100 + 100 + 1)
    bad = ParsedCompletion(raw_text="x", tool_calls=[{"name": "move", "arguments": {"d": 3}}], parse_errors=["e"])
    assert not reward.score_parsed(bad, _tools([{"name": "move", "arguments": {"d": 3}}]), is_tool_call=True).all_right


def test_normalize_targets_validation():
    with pytest.raises(ValueError):
        normalize_targets([])
    with pytest.raises(ValueError):
        normalize_targets([{"output": {}}])
    with pytest.raises(ValueError):
        normalize_targets([{"output": {"tool_calls": [{"name": "", "arguments": {}}]}}])
    assert normalize_targets([{"output": {"content": {"a": 1}}}])[0]["id"] is None
