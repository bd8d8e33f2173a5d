"""Reward scoring shared by the evaluation tools (native checkpoint, an
OpenAI-compatible serving endpoint, a transformers baseline).

Every tool produces one row per completion with the same keys and the same
summary, so their ``summary.json`` files compare directly.
"""

from __future__ import annotations

import json
from pathlib import Path
from statistics import mean
from typing import Any

from graspo_b200.core.completion import ParsedCompletion


def scrubbed_metadata(sample) -> dict[str, Any]:
    """Record metadata with media paths reduced to their type (private file
    names stay out of reports)."""
    meta = {k: v for k, v in (sample.metadata or {}).items() if k not in ("image", "images", "video", "videos")}
    meta["media"] = [{"type": m.get("type")} for m in (sample.media or [])]
    return meta


def score_row(reward, parsed: ParsedCompletion, sample, *, sample_index: int, completion_index: int,
              **extra: Any) -> dict[str, Any]:
    res = reward.score_parsed(parsed, sample.targets, is_tool_call=sample.expects_tool_calls)
    row = {"sample_index": sample_index, "completion_index": completion_index, "completion": parsed.raw_text,
           "reward": float(res.reward), "content_score": float(res.content_score), "all_right": bool(res.all_right),
           "matched_target_index": res.matched_target_index, "matched_target_id": res.matched_target_id,
           "parser_name": parsed.parser_name, "parse_errors": list(parsed.parse_errors),
           "tool_calls": list(parsed.tool_calls or []), "targets": sample.targets,
           "metadata": scrubbed_metadata(sample)}
    row.update(extra)
    return row


def summarize(rows: list[dict[str, Any]], sample_count: int, **extra: Any) -> dict[str, Any]:
    groups: dict[int, list[float]] = {}
    for r in rows:
        groups.setdefault(r["sample_index"], []).append(r["reward"])
    flat = [r["reward"] for r in rows]
    out = {
        "count": int(sample_count),
        "completion_count": len(rows),
        "reward_mean": mean(flat) if flat else 0.0,
        "reward_max_mean": mean(max(g) for g in groups.values()) if groups else 0.0,
        "reward_range_mean": mean(max(g) - min(g) for g in groups.values()) if groups else 0.0,
        "content_mean": mean(r["content_score"] for r in rows) if rows else 0.0,
        "all_right_rate": (sum(r["all_right"] for r in rows) / len(rows)) if rows else 0.0,
        "parse_error_rate": (sum(bool(r["parse_errors"]) for r in rows) / len(rows)) if rows else 0.0,
    }
    out.update(extra)
    return out


def write_report(output_dir: str | Path, rows: list[dict[str, Any]], summary: dict[str, Any]) -> None:
    out = Path(output_dir)
    out.mkdir(parents=True, exist_ok=True)
    with (out / "completions.jsonl").open("w", encoding="utf-8") as fh:
        for row in rows:
            fh.write(json.dumps(row, ensure_ascii=False) + "\n")
    (out / "summary.json").write_text(json.dumps(summary, ensure_ascii=False, indent=2) + "\n", encoding="utf-8")
