"""Run statistics, batch / window summaries, health flags, JSONL logs and the
host-side fault injector (pure CPU).

Key names follow the reference's trainer (trainer/summary.py:17-459,
trainer/stats.py, backends/graspoflow/logger.py) so log tooling reads both.
"""

from __future__ import annotations

import dataclasses
import json

import pytest
import torch

from graspo_b200.train.logger import RolloutLogger, readable_payload, summarize_think, to_jsonable
from graspo_b200.train.summary import (
    compact_batch_summary,
    compact_decisions,
    compact_optimize_metrics,
    compact_timing_summary,
    is_pure_tool_call_task,
    likely_truncated_json,
    monitor_group,
    reward_batch_summary,
    reward_window_summary,
    scalar_generation_timing,
    tool_call_count_mismatch_count,
    training_health,
)
from graspo_b200.train.trainer import EpochStats, FaultInjector, InjectedFault, TrainStats, group_stats

CONTENT_TARGETS = [{"output": {"content": {"a": 1}}}]
TOOL_TARGETS = [{"output": {"tool_calls": [{"name": "f", "arguments": {}}]}}]


def _group(decision, rewards, content, completions=None, details=None, targets=CONTENT_TARGETS):
    n = len(rewards)
    return {"decision": decision, "rewards": rewards, "content_scores": content,
            "completions": completions or ['```json\n{"a": 1}\n```'] * n,
            "reward_details": details or [{"valid_extracted_json": True}] * n, "targets": targets}


def test_stats_defaults_and_round_trip():
    t = TrainStats()
    assert all(v == 0 for v in dataclasses.asdict(t).values())
    t.perfect_skipped += 2
    t.trainable_max_correct += 1
    assert TrainStats(**dataclasses.asdict(t)) == t
    e = EpochStats(epoch=3)
    e.reward_mean_sum += 0.5
    e.best_reward = max(e.best_reward, 0.9)
    e.samples_seen += 4
    assert EpochStats(**dataclasses.asdict(e)) == e and e.best_reward == 0.9


def test_group_stats():
    s = group_stats([0.2, 1.0, 0.4, 0.6])
    assert s == {"count": 4, "min": 0.2, "median": 0.4, "max": 1.0, "mean": pytest.approx(0.55), "range": 0.8}
    assert group_stats([])["count"] == 0


def test_monitor_group_perfect_and_empty():
    m = monitor_group(_group("perfect_skip", [1.0, 1.0], [1.0, 1.0]))
    assert m["decision"] == "perfect_skip" and m["reward_mean"] == 1.0 and m["reward_range"] == 0.0
    assert m["content_all_one"] and not m["content_all_zero"]
    assert m["missing_json_marker_count"] == 0 and m["likely_truncated_json_count"] == 0
    empty = monitor_group({"decision": "invalid", "rewards": [], "content_scores": []})
    assert empty["reward_mean"] == 0.0 and not empty["content_all_one"] and not empty["content_all_zero"]


def test_json_debug_counts():
    completions = ["no fence", '```json\n{"a": 1', '```json\n{"a": 1}\n```']
    details = [{}, {"valid_extracted_json": False, "extracted_answer": '{"a": 1'}, {"valid_extracted_json": True}]
    m = monitor_group(_group("trainable_not_correct", [0.0, 0.1, 1.0], [0.0, 0.0, 1.0], completions, details))
    assert m["missing_json_marker_count"] == 1
    assert m["unclosed_json_fence_count"] == 1
    assert m["invalid_extracted_json_count"] == 1
    assert m["likely_truncated_json_count"] == 1
    # pure tool-call tasks carry no JSON fence expectations
    tool = monitor_group(_group("invalid", [0.0], [0.0], ["x"], [{}], TOOL_TARGETS))
    assert tool["missing_json_marker_count"] == 0
    assert is_pure_tool_call_task(TOOL_TARGETS) and not is_pure_tool_call_task(CONTENT_TARGETS)
    assert likely_truncated_json("x", {"extracted_answer": '{"a": {"b": 1}'})
    assert not likely_truncated_json('```json\n{}\n```')


def test_tool_call_count_mismatch():
    targets = [{"output": {"tool_calls": [{"name": "f", "arguments": {}}] * 2}}]
    details = [{"tool_calls": [{}]}, {"tool_calls": [{}, {}]}, {"tool_calls": None}]
    assert tool_call_count_mismatch_count(details, targets) == 1
    assert tool_call_count_mismatch_count(details, CONTENT_TARGETS) == 0


def test_window_and_batch_summaries():
    groups = [monitor_group(_group("trainable_max_correct", [0.0, 1.0], [0.0, 1.0])),
              monitor_group(_group("invalid", [0.5, 0.5], [0.5, 0.5]))]
    w = reward_window_summary(groups)
    assert w["count"] == 2 and w["decision_counts"] == {"trainable_max_correct": 1, "invalid": 1}
    assert w["nonzero_range_rate"] == 0.5 and w["reward_mean_avg"] == 0.5
    attempts = [_group("trainable_max_correct", [0.0, 1.0], [0.0, 1.0]), _group("retry", [0.2, 0.2], [0.0, 0.0]),
                _group("perfect_skip", [1.0, 1.0], [1.0, 1.0])]
    b = reward_batch_summary(attempts, rollout_group_size=2, optimize_prompt_batch_size=4)
    assert b["attempt_group_count"] == 3 and b["completion_count"] == 6
    assert b["trainable_group_count"] == 1 and b["trainable_completion_count"] == 2
    assert b["retry_group_count"] == 1 and b["perfect_skip_completion_count"] == 2
    assert b["reward_nonzero_range_group_count"] == 1
    assert b["content_all_zero_group_count"] == 1 and b["content_all_one_group_count"] == 1
    assert b["reward_max_median_gap_mean"] == pytest.approx(1.0 / 3)
    c = compact_batch_summary(b)
    assert c["decisions"]["rollout_attempts"] == {"total": 3, "retry": 1, "terminal": 2}
    assert c["decisions"]["trainable"] == {"max_correct": 1, "not_correct": 0, "total": 1}
    assert c["reward"]["max"] == 1.0


def test_compact_decisions_totals():
    d = compact_decisions(perfect_skip=1, trainable_max_correct=2, trainable_not_correct=3, invalid=4,
                          invalid_no_preference_gap=5, retry_attempts=6)
    assert d["terminal"]["total"] == 15 and d["rollout_attempts"]["total"] == 21 and d["trainable"]["total"] == 5


def test_timing_and_optimize_roll_ups():
    timings = [{"rollout_sec": 1.0, "decode_sec": 0.8, "decode_tokens": 100, "old_logprob_sec": 0.25},
               {"rollout_sec": 2.0, "decode_sec": 1.5, "decode_tokens": 50}]
    t = compact_timing_summary(timings, optimize_sec=4.0, checkpoint_sec=0.5, metrics={"micro_batch_count": 3})
    assert t["rollout_sec"] == 3.0 and t["decode_tokens"] == 150 and t["micro_batch_count"] == 3
    assert t["total_observed_sec"] == pytest.approx(7.75)
    assert t["decode_tokens_per_sec"] == pytest.approx(50.0)
    assert t["step_decode_tokens_per_sec"] == pytest.approx(150 / 7.75, rel=1e-3)
    o = compact_optimize_metrics({"optimized": True, "optimizer_steps": 2, "global_loss_mean": 0.3,
                                  "loss_mean": 9.0, "grad_norm_mean": 1.5, "skipped_nonfinite": 1})
    assert o["loss_mean"] == 0.3 and o["grad_norm_mean"] == 1.5 and o["global_optimizer_steps_sum"] == 2
    assert scalar_generation_timing({"decode_sec": 1.0, "other": 2}) == {"decode_sec": 1.0}


def test_training_health_flags():
    ok = training_health({"optimized": True, "lora_norm_delta": 0.1}, {"attempt_group_count": 1, "reward_mean": 0.5},
                         {"count": 3})
    assert ok == {"ok": True, "early_stop_recommended": False, "reasons": []}
    bad = training_health({"optimized": True, "lora_norm_delta": 0.0, "skipped_nonfinite": 2},
                          {"attempt_group_count": 2, "reward_mean": 0.0, "likely_truncated_json_count": 1},
                          {"count": 10, "reward_mean_avg": 0.0, "nonzero_range_rate": 0.0, "content_all_zero_rate": 0.9})
    assert bad["early_stop_recommended"] and set(bad["reasons"]) == {
        "nonfinite_loss_or_grad", "zero_lora_delta", "batch_reward_all_zero", "batch_json_truncation_detected",
        "reward_all_zero_window", "no_group_reward_variance_window", "content_score_all_zero_window"}


def test_rollout_logger_files(tmp_path):
    log = RolloutLogger(tmp_path)
    payload = {"event": None, "decision": "invalid", "completions": ["<think>a</think>```json\n{}\n```"],
               "rewards": [0.5], "reward_details": [{"raw_score": 1.0, "max_score": 2.0}], "tokens": torch.tensor([1, 2])}
    log.write_readable(payload)
    log.write_raw(payload)
    log.write_timing_event({"phase": "rollout", "sec": 1.5})
    log.write_error({"error": "boom"})
    log.write_train_batch_readable({"attempts": [{"decision": "retry", "extra": 1}]})
    files = {p.name for p in (tmp_path / "logs").iterdir()}
    assert files == {"rollouts.readable.jsonl", "rollouts.raw.jsonl", "timing_events.jsonl", "error.log",
                     "train_batches.readable.jsonl"}
    readable = json.loads((tmp_path / "logs" / "rollouts.readable.jsonl").read_text())
    assert readable["event"] == "graspo_group" and readable["completions"][0]["think"]["closed"]
    assert readable["completions"][0]["json"]["has_closing_json_fence"]
    raw = json.loads((tmp_path / "logs" / "rollouts.raw.jsonl").read_text())
    assert raw["tokens"] == [1, 2]
    batch = json.loads((tmp_path / "logs" / "train_batches.readable.jsonl").read_text())
    assert "extra" not in batch["attempts"][0]
    quiet = RolloutLogger(tmp_path / "q", readable_enabled=False, raw_enabled=False)
    quiet.write_readable(payload)
    quiet.write_raw(payload)
    assert not (tmp_path / "q" / "logs" / "rollouts.readable.jsonl").exists()


def test_jsonable_and_think_summary():
    assert to_jsonable({1: (torch.tensor(2.0), object)})["1"][0] == 2.0
    assert summarize_think("<think>abc</think>") == {"has_think": True, "closed": True, "chars": 3}
    assert summarize_think("<think>abc")["closed"] is False
    assert readable_payload({"completions": []})["completions"] == []


def test_fault_injector(monkeypatch):
    monkeypatch.setenv("GRASPO_FAULT", "optimize:2")
    inj = FaultInjector(rank=0)
    inj.hit("optimize")
    inj.hit("rollout")
    with pytest.raises(InjectedFault, match="optimize"):
        inj.hit("optimize")
    monkeypatch.setenv("GRASPO_FAULT_RANK", "1")
    other = FaultInjector(rank=0)
    for _ in range(3):
        other.hit("optimize")  # armed for rank 1 only
    monkeypatch.delenv("GRASPO_FAULT")
    FaultInjector(rank=1).hit("optimize")
