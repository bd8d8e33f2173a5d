"""Structured JSONL logs under ``<output_dir>/logs``.

File names follow the reference layout (backends/graspoflow/logger.py):
``rollouts.readable.jsonl`` (compact per-group view), ``rollouts.raw.jsonl``
(everything, tensors as lists), ``train_batches.readable.jsonl``,
``timing_events.jsonl``, ``error.log`` (invalid groups, failures), ``events.jsonl``
(every stdout event of the primary rank, for post-run analysis) and
``rank_metrics.rank_NNNNN.jsonl`` (per-rank memory/metrics events).
"""

from __future__ import annotations

import json
from pathlib import Path
from typing import Any


def to_jsonable(value: Any) -> Any:
    if isinstance(value, dict):
        return {str(k): to_jsonable(v) for k, v in value.items()}
    if isinstance(value, (list, tuple)):
        return [to_jsonable(v) for v in value]
    if hasattr(value, "tolist"):
        return value.tolist()
    if isinstance(value, (str, int, float, bool)) or value is None:
        return value
    return str(value)


def summarize_json_markers(text: str) -> dict[str, Any]:
    opened = "```json" in text
    return {
        "has_json_fence": opened,
        "has_closing_json_fence": opened and text.count("```") >= 2,
        "fence_count": text.count("```"),
    }


def summarize_think(text: str) -> dict[str, Any]:
    start = text.find("<think>")
    end = text.find("</think>", start + 7) if start >= 0 else -1
    return {"has_think": start >= 0, "closed": end >= 0, "chars": (end - start - 7) if end >= 0 else 0}


def readable_payload(payload: dict[str, Any]) -> dict[str, Any]:
    """One group, compacted: prompt, decision, and per-completion scoring detail."""
    from graspo_b200.train.summary import likely_truncated_json

    def at(seq, i):
        return seq[i] if isinstance(seq, list) and i < len(seq) else None

    out = {k: payload.get(k) for k in (
        "event", "step", "epoch", "sample_index", "attempt_index", "max_attempts", "messages", "tools",
        "prompt_preview", "targets", "decision", "retry_count", "reward_max_median_gap", "group_stats")}
    out["event"] = out["event"] or "graspo_group"
    if payload.get("invalid_reason") is not None:
        out["invalid_reason"] = payload["invalid_reason"]
    rows = []
    for i, text in enumerate(payload.get("completions", [])):
        detail = at(payload.get("reward_details", []), i) or {}
        rows.append({
            "idx": i,
            "completion": text,
            "reward": at(payload.get("rewards", []), i),
            "content_score": at(payload.get("content_scores", []), i),
            "all_right": at(payload.get("all_right", []), i),
            "raw_score": detail.get("raw_score"),
            "max_score": detail.get("max_score"),
            "extracted": detail.get("extracted"),
            "parsed": at(payload.get("parsed_completions", []), i) or {},
            "parse_errors": detail.get("parse_errors"),
            "matched_target_index": detail.get("matched_target_index"),
            "matched_target_id": detail.get("matched_target_id"),
            "target_scores": detail.get("target_scores"),
            "useless_text_length": detail.get("useless_text_length"),
            "valid_extracted_json": detail.get("valid_extracted_json"),
            "completion_chars": len(text),
            "generated_tokens": at(payload.get("generated_tokens", []), i),
            "likely_truncated_json": likely_truncated_json(text, detail),
            "think": summarize_think(text),
            "json": summarize_json_markers(text),
        })
    out["completions"] = rows
    return to_jsonable(out)


class RolloutLogger:
    def __init__(self, output_dir: str | Path, *, readable_enabled: bool = True, raw_enabled: bool = True) -> None:
        self.logs_dir = Path(output_dir) / "logs"
        self.logs_dir.mkdir(parents=True, exist_ok=True)
        self.readable_enabled = readable_enabled
        self.raw_enabled = raw_enabled
        self.readable_path = self.logs_dir / "rollouts.readable.jsonl"
        self.raw_path = self.logs_dir / "rollouts.raw.jsonl"
        self.train_batches_readable_path = self.logs_dir / "train_batches.readable.jsonl"
        self.timing_path = self.logs_dir / "timing_events.jsonl"
        self.error_path = self.logs_dir / "error.log"

    @staticmethod
    def _append(path: Path, payload: dict[str, Any]) -> None:
        with path.open("a", encoding="utf-8") as handle:
            handle.write(json.dumps(payload, ensure_ascii=False) + "\n")

    def write_readable(self, payload: dict[str, Any]) -> None:
        if self.readable_enabled:
            self._append(self.readable_path, readable_payload(payload))

    def write_raw(self, payload: dict[str, Any]) -> None:
        if self.raw_enabled:
            self._append(self.raw_path, to_jsonable(payload))

    def write_train_batch_readable(self, payload: dict[str, Any]) -> None:
        if self.readable_enabled:
            slim = dict(payload)
            slim["attempts"] = [
                {k: a.get(k) for k in ("sample_index", "attempt_index", "decision", "group_stats", "prompt_preview")}
                for a in payload.get("attempts", [])
            ]
            self._append(self.train_batches_readable_path, to_jsonable(slim))

    def write_timing_event(self, payload: dict[str, Any]) -> None:
        if self.readable_enabled:
            self._append(self.timing_path, to_jsonable(payload))

    def write_error(self, payload: dict[str, Any]) -> None:
        self._append(self.error_path, to_jsonable(payload))


def append_event(output_dir: str | Path, payload: dict[str, Any]) -> None:
    """Append one stdout event to ``<output_dir>/logs/events.jsonl``."""
    path = Path(output_dir) / "logs" / "events.jsonl"
    path.parent.mkdir(parents=True, exist_ok=True)
    with path.open("a", encoding="utf-8") as handle:
        handle.write(json.dumps(payload, ensure_ascii=False, default=str) + "\n")


def memory_snapshot(device: Any) -> dict[str, Any]:
    """Allocator and device memory of ``device`` in MiB (empty on CPU)."""
    import torch

    if getattr(device, "type", "cpu") != "cuda" or not torch.cuda.is_available():
        return {}
    mib = 1 << 20
    free, total = torch.cuda.mem_get_info(device)
    return {
        "allocated_mib": torch.cuda.memory_allocated(device) / mib,
        "reserved_mib": torch.cuda.memory_reserved(device) / mib,
        "max_allocated_mib": torch.cuda.max_memory_allocated(device) / mib,
        "device_free_mib": free / mib,
        "device_total_mib": total / mib,
    }


def append_rank_metrics(output_dir: str | Path, rank: int, payload: dict[str, Any]) -> None:
    """One line of ``<output_dir>/logs/rank_metrics.rank_NNNNN.jsonl`` (every rank writes its own)."""
    path = Path(output_dir) / "logs" / f"rank_metrics.rank_{int(rank):05d}.jsonl"
    path.parent.mkdir(parents=True, exist_ok=True)
    with path.open("a", encoding="utf-8") as handle:
        handle.write(json.dumps(to_jsonable(payload), ensure_ascii=False) + "\n")
