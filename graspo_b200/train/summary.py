"""Batch / window reward summaries, timing roll-ups and training health flags.

The dictionaries produced here are the payloads of the ``train_step`` and
``epoch_summary`` events and of ``logs/train_batches.readable.jsonl``; their
keys follow the reference (trainer/summary.py:17-459) so existing
log-analysis tooling reads both frameworks' runs.
"""

from __future__ import annotations

import json
from collections import deque
from typing import Any

from graspo_b200.core.decisions import lower_median

TRAINABLE = ("trainable_max_correct", "trainable_not_correct")


def is_pure_tool_call_task(targets: Any) -> bool:
    if not isinstance(targets, list) or not targets:
        return False
    outs = [t.get("output") for t in targets if isinstance(t, dict)]
    return all(isinstance(o, dict) and "tool_calls" in o and "content" not in o for o in outs) and bool(outs)


def _target_tool_call_counts(targets: Any) -> set[int]:
    counts: set[int] = set()
    for t in targets or []:
        calls = (t.get("output") or {}).get("tool_calls") if isinstance(t, dict) else None
        if isinstance(calls, list):
            counts.add(len(calls))
    return counts


def tool_call_count_mismatch_count(details: list[dict[str, Any]], targets: Any) -> int:
    expected = _target_tool_call_counts(targets)
    if not expected:
        return 0
    n = 0
    for d in details:
        calls = d.get("tool_calls")
        if isinstance(calls, list) and len(calls) not in expected:
            n += 1
    return n


def likely_truncated_json(text: str, detail: dict[str, Any] | None = None) -> bool:
    """An opened ```json fence that never closes, or JSON that stops mid-object."""
    if "```json" in text and text.count("```") < 2:
        return True
    extracted = (detail or {}).get("extracted_answer")
    if isinstance(extracted, str) and extracted.strip().startswith("{"):
        try:
            json.loads(extracted)
        except ValueError:
            return extracted.count("{") > extracted.count("}")
    return False


def _json_counts(completions, details, pure_tool_call: bool) -> dict[str, int]:
    if pure_tool_call:
        return {"missing": 0, "unclosed": 0, "invalid": 0, "truncated": 0}
    return {
        "missing": sum(1 for t in completions if "```json" not in t),
        "unclosed": sum(1 for t in completions if "```json" in t and t.count("```") < 2),
        "invalid": sum(1 for d in details if d.get("valid_extracted_json") is False),
        "truncated": sum(1 for t, d in zip(completions, details, strict=False) if likely_truncated_json(t, d)),
    }


def monitor_group(payload: dict[str, Any]) -> dict[str, Any]:
    rewards = [float(v) for v in payload.get("rewards", [])]
    content = [float(v) for v in payload.get("content_scores", [])]
    details = payload.get("reward_details", [])
    counts = _json_counts(payload.get("completions", []), details, is_pure_tool_call_task(payload.get("targets")))
    return {
        "decision": payload.get("decision"),
        "reward_mean": sum(rewards) / len(rewards) if rewards else 0.0,
        "reward_max": max(rewards) if rewards else 0.0,
        "reward_range": max(rewards) - min(rewards) if rewards else 0.0,
        "content_mean": sum(content) / len(content) if content else 0.0,
        "content_all_zero": bool(content) and all(v == 0.0 for v in content),
        "content_all_one": bool(content) and all(v == 1.0 for v in content),
        "missing_json_marker_count": counts["missing"],
        "unclosed_json_fence_count": counts["unclosed"],
        "invalid_extracted_json_count": counts["invalid"],
        "likely_truncated_json_count": counts["truncated"],
        "tool_call_parse_error_count": sum(1 for d in details if d.get("parse_errors")),
        "tool_call_count_mismatch_count": tool_call_count_mismatch_count(details, payload.get("targets")),
    }


_WINDOW_COUNTS = ("missing_json_marker_count", "unclosed_json_fence_count", "invalid_extracted_json_count",
                  "likely_truncated_json_count", "tool_call_parse_error_count", "tool_call_count_mismatch_count")


def reward_window_summary(groups: deque[dict[str, Any]] | list) -> dict[str, Any]:
    items = list(groups)
    n = len(items)
    out: dict[str, Any] = {"count": n, "decision_counts": {}}
    for item in items:
        key = str(item.get("decision"))
        out["decision_counts"][key] = out["decision_counts"].get(key, 0) + 1

    def avg(fn) -> float:
        return sum(fn(i) for i in items) / n if n else 0.0

    out.update({
        "reward_mean_avg": avg(lambda i: float(i["reward_mean"])),
        "reward_max_avg": avg(lambda i: float(i["reward_max"])),
        "nonzero_range_rate": avg(lambda i: float(i["reward_range"]) > 0.0),
        "content_mean_avg": avg(lambda i: float(i["content_mean"])),
        "content_all_zero_rate": avg(lambda i: bool(i["content_all_zero"])),
        "content_all_one_rate": avg(lambda i: bool(i["content_all_one"])),
    })
    for key in _WINDOW_COUNTS:
        out[key] = sum(int(i.get(key) or 0) for i in items)
    return out


def reward_batch_summary(attempts: list[dict[str, Any]], *, rollout_group_size: int,
                         optimize_prompt_batch_size: int) -> dict[str, Any]:
    G = int(rollout_group_size)
    decisions: dict[str, int] = {}
    rewards: list[float] = []
    content: list[float] = []
    ranges: list[float] = []
    gaps: list[float] = []
    totals = dict.fromkeys(("missing", "unclosed", "invalid", "truncated", "parse", "mismatch"), 0)
    for att in attempts:
        d = str(att.get("decision"))
        decisions[d] = decisions.get(d, 0) + 1
        r = [float(v) for v in att.get("rewards", [])]
        rewards += r
        content += [float(v) for v in att.get("content_scores", [])]
        if r:
            ranges.append(max(r) - min(r))
            gaps.append(max(r) - lower_median(r))
        details = att.get("reward_details", [])
        c = _json_counts(att.get("completions", []), details, is_pure_tool_call_task(att.get("targets")))
        for k in ("missing", "unclosed", "invalid", "truncated"):
            totals[k] += c[k]
        totals["parse"] += sum(1 for dd in details if dd.get("parse_errors"))
        totals["mismatch"] += tool_call_count_mismatch_count(details, att.get("targets"))
    trainable = sum(decisions.get(k, 0) for k in TRAINABLE)

    def groups(key: str) -> int:
        return decisions.get(key, 0)

    return {
        "unit": "batch_attempt",
        "rollout_group_size": G,
        "optimize_prompt_batch_size": int(optimize_prompt_batch_size),
        "attempt_group_count": len(attempts),
        "completion_count": len(attempts) * G,
        "observed_completion_count": len(rewards),
        "trainable_group_count": trainable,
        "trainable_completion_count": trainable * G,
        "retry_group_count": groups("retry"),
        "retry_completion_count": groups("retry") * G,
        "perfect_skip_group_count": groups("perfect_skip"),
        "perfect_skip_completion_count": groups("perfect_skip") * G,
        "invalid_group_count": groups("invalid"),
        "invalid_completion_count": groups("invalid") * G,
        "invalid_no_preference_gap_group_count": groups("invalid_no_preference_gap"),
        "invalid_no_preference_gap_completion_count": groups("invalid_no_preference_gap") * G,
        "decision_counts": decisions,
        "reward_min": min(rewards) if rewards else 0.0,
        "reward_median": lower_median(rewards),
        "reward_mean": sum(rewards) / len(rewards) if rewards else 0.0,
        "reward_max": max(rewards) if rewards else 0.0,
        "reward_nonzero_range_group_count": sum(v > 0.0 for v in ranges),
        "reward_nonzero_range_rate": sum(v > 0.0 for v in ranges) / len(ranges) if ranges else 0.0,
        "reward_max_median_gap_mean": sum(gaps) / len(gaps) if gaps else 0.0,
        "content_mean": sum(content) / len(content) if content else 0.0,
        "content_all_zero_group_count": sum(
            bool(a.get("content_scores")) and all(float(v) == 0.0 for v in a.get("content_scores", []))
            for a in attempts
        ),
        "content_all_one_group_count": sum(
            bool(a.get("content_scores")) and all(float(v) == 1.0 for v in a.get("content_scores", []))
            for a in attempts
        ),
        "missing_json_marker_count": totals["missing"],
        "unclosed_json_fence_count": totals["unclosed"],
        "invalid_extracted_json_count": totals["invalid"],
        "likely_truncated_json_count": totals["truncated"],
        "tool_call_parse_error_count": totals["parse"],
        "tool_call_count_mismatch_count": totals["mismatch"],
    }


def compact_decisions(*, perfect_skip: int, trainable_max_correct: int, trainable_not_correct: int, invalid: int,
                      invalid_no_preference_gap: int, retry_attempts: int) -> dict[str, Any]:
    trainable = int(trainable_max_correct) + int(trainable_not_correct)
    terminal = int(perfect_skip) + trainable + int(invalid) + int(invalid_no_preference_gap)
    return {
        "rollout_attempts": {"total": terminal + int(retry_attempts), "retry": int(retry_attempts),
                             "terminal": terminal},
        "terminal": {"perfect_skip": int(perfect_skip), "trainable": trainable, "invalid": int(invalid),
                     "invalid_no_preference_gap": int(invalid_no_preference_gap), "total": terminal},
        "trainable": {"max_correct": int(trainable_max_correct), "not_correct": int(trainable_not_correct),
                      "total": trainable},
    }


def compact_batch_summary(summary: dict[str, Any]) -> dict[str, Any]:
    d = dict(summary.get("decision_counts") or {})

    def f(key):
        return float(summary.get(key) or 0.0)

    def i(key):
        return int(summary.get(key) or 0)

    return {
        "attempt_groups": i("attempt_group_count"),
        "completions": i("completion_count"),
        "decisions": compact_decisions(
            perfect_skip=int(d.get("perfect_skip") or 0), trainable_max_correct=int(d.get("trainable_max_correct") or 0),
            trainable_not_correct=int(d.get("trainable_not_correct") or 0), invalid=int(d.get("invalid") or 0),
            invalid_no_preference_gap=int(d.get("invalid_no_preference_gap") or 0),
            retry_attempts=int(d.get("retry") or 0),
        ),
        "reward": {"min": f("reward_min"), "median": f("reward_median"), "mean": f("reward_mean"),
                   "max": f("reward_max"), "nonzero_range_rate": f("reward_nonzero_range_rate"),
                   "max_median_gap_mean": f("reward_max_median_gap_mean")},
        "content": {"mean": f("content_mean"), "all_zero_groups": i("content_all_zero_group_count"),
                    "all_one_groups": i("content_all_one_group_count")},
        "debug": {"missing_json_marker": i("missing_json_marker_count"),
                  "unclosed_json_fence": i("unclosed_json_fence_count"),
                  "invalid_json": i("invalid_extracted_json_count"), "truncated_json": i("likely_truncated_json_count"),
                  "tool_call_parse_error": i("tool_call_parse_error_count"),
                  "tool_call_count_mismatch": i("tool_call_count_mismatch_count")},
    }


def _sum(items: list[dict[str, Any]], key: str) -> float:
    return sum(float(x.get(key) or 0.0) for x in items)


def compact_timing_summary(timings: list[dict[str, Any]], *, optimize_sec: float, checkpoint_sec: float,
                           metrics: dict[str, Any]) -> dict[str, Any]:
    phases = ("rollout_sec", "reward_cpu_sec", "decision_sec", "old_logprob_sec", "replay_append_sec")
    total = sum(_sum(timings, p) for p in phases) + float(optimize_sec) + float(checkpoint_sec)
    out: dict[str, Any] = {"attempt_count": len(timings)}
    out["rollout_prompt_queue_batch_size"] = max(
        [int(t.get("rollout_prompt_queue_batch_size") or 1) for t in timings], default=1)
    out["rollout_prompt_queue_effective_size"] = max(
        [int(t.get("rollout_prompt_queue_effective_size") or 1) for t in timings], default=1)
    out["rollout_prompt_queue_fallback_count"] = sum(bool(t.get("rollout_prompt_queue_fallback")) for t in timings)
    for p in phases:
        out[p] = round(_sum(timings, p), 6)
    out["optimize_sec"] = round(float(optimize_sec), 6)
    out["checkpoint_sec"] = round(float(checkpoint_sec), 6)
    for p in ("prefill_sec", "decode_sec", "sampling_sec", "stop_check_sec"):
        out[p] = round(_sum(timings, p), 6)
    out["train_batch_total_sec"] = round(float(metrics.get("train_batch_total_sec") or optimize_sec), 6)
    for p in ("optimize_round_sec_sum", "micro_batch_forward_sec", "backward_sec", "optimizer_step_sec"):
        out[p] = round(float(metrics.get(p) or 0.0), 6)
    out["micro_batch_count"] = int(metrics.get("micro_batch_count") or metrics.get("optimizer_steps") or 0)
    out["decode_tokens"] = int(_sum(timings, "decode_tokens"))
    out["rollout_generation_split_count"] = int(_sum(timings, "rollout_generation_split_count"))
    out["total_observed_sec"] = round(total, 6)
    # throughput: generated tokens per rollout second and per observed step second
    out["decode_tokens_per_sec"] = round(out["decode_tokens"] / out["rollout_sec"], 3) if out["rollout_sec"] > 0 else None
    out["step_decode_tokens_per_sec"] = round(out["decode_tokens"] / total, 3) if total > 0 else None
    return out


def round_timing_details(details: dict[str, Any]) -> dict[str, Any]:
    out: dict[str, Any] = {}
    for key, value in details.items():
        if isinstance(value, float):
            out[key] = round(value, 6)
        elif isinstance(value, (str, int, bool)) or value is None:
            out[key] = value
    return out


_GEN_TIMING_KEYS = {
    "tokenize_sec", "prefill_sec", "decode_sec", "sampling_sec", "stop_check_sec", "decode_tokens",
    "rollout_elapsed_sec", "rollout_use_kv_cache", "rollout_generation_micro_batch_size",
    "rollout_generation_split_count", "rollout_empty_cache_after_split", "prefill_len", "generated_tokens_max",
    "rollout_prompt_queue_batch_size", "rollout_prompt_queue_effective_size", "rollout_prompt_queue_fallback",
}


def scalar_generation_timing(metadata: dict[str, Any]) -> dict[str, Any]:
    return {k: v for k, v in metadata.items() if k in _GEN_TIMING_KEYS}


def _metric(metrics: dict[str, Any], preferred: str, fallback: str) -> float:
    value = metrics.get(preferred)
    if value is None:
        value = metrics.get(fallback)
    return float(value or 0.0)


def compact_optimize_metrics(metrics: dict[str, Any]) -> dict[str, Any]:
    per_rank = int(metrics.get("optimizer_steps") or 0)
    return {
        "optimized": bool(metrics.get("optimized")),
        "replay_buffer_trainable_completion_count": int(metrics.get("replay_buffer_trainable_completion_count") or 0),
        "replay_buffer_trainable_group_count": float(metrics.get("replay_buffer_trainable_group_count") or 0.0),
        "replay_buffer_optimize_threshold": int(metrics.get("replay_buffer_optimize_threshold") or 0),
        "optimize_prompt_batch_size": int(metrics.get("optimize_prompt_batch_size") or 0),
        "optimize_iterations_per_step": int(metrics.get("optimize_iterations_per_step") or 0),
        "optimizer_steps_per_rank": per_rank,
        "global_optimizer_steps_sum": int(metrics.get("global_optimizer_steps_sum") or per_rank),
        "loss_mean": _metric(metrics, "global_loss_mean", "loss_mean"),
        "grad_norm_mean": _metric(metrics, "global_grad_norm_mean", "grad_norm_mean"),
        "lora_delta_mean": _metric(metrics, "global_lora_norm_delta_mean", "lora_norm_delta"),
        "skipped_nonfinite": int(metrics.get("skipped_nonfinite") or 0),
        "force_flush": bool(metrics.get("force_flush")),
    }


def training_health(metrics: dict[str, Any], batch: dict[str, Any], window: dict[str, Any]) -> dict[str, Any]:
    reasons: list[str] = []
    if int(metrics.get("skipped_nonfinite") or 0) > 0:
        reasons.append("nonfinite_loss_or_grad")
    if metrics.get("optimized") and _metric(metrics, "global_lora_norm_delta_mean", "lora_norm_delta") == 0.0:
        reasons.append("zero_lora_delta")
    if int(batch.get("attempt_group_count") or 0) > 0:
        if float(batch.get("reward_mean") or 0.0) == 0.0:
            reasons.append("batch_reward_all_zero")
        if int(batch.get("likely_truncated_json_count") or 0) > 0:
            reasons.append("batch_json_truncation_detected")
    if int(window.get("count") or 0) >= 10:
        if float(window.get("reward_mean_avg") or 0.0) == 0.0:
            reasons.append("reward_all_zero_window")
        if float(window.get("nonzero_range_rate") or 0.0) == 0.0:
            reasons.append("no_group_reward_variance_window")
        if float(window.get("content_all_zero_rate") or 0.0) >= 0.8:
            reasons.append("content_score_all_zero_window")
    return {"ok": not reasons, "early_stop_recommended": bool(reasons), "reasons": reasons}
