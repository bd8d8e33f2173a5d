"""Summarise GRASPO runs from their ``train_step`` events.

    python -m graspo_b200.analysis.profile OUTPUT_DIR [OUTPUT_DIR ...] [--json] [--skip-warmup-steps N]

Reads the JSON events a run printed (``logs/events.jsonl``, written by the
trainer next to stdout, or a captured ``nohup.out`` / ``train.log``), the GPU
memory recorder's output (``gpu_memory/``) and per-rank metric files, and
reports mean phase timings over the measured steps plus two throughput
figures with the reference's definitions (scripts/analyze_native_profile.py:97-100):

* ``decode_tokens_per_sec`` = sum(decode_tokens) / sum(rollout_sec)
* ``trainable_groups_per_hour`` = trainable groups x 3600 / (mean step seconds x steps)
"""

from __future__ import annotations

import argparse
import json
from pathlib import Path
from statistics import mean
from typing import Any

TIMING_KEYS = (
    "total_observed_sec", "rollout_sec", "prefill_sec", "decode_sec", "sampling_sec", "stop_check_sec",
    "old_logprob_sec", "optimize_sec", "train_batch_total_sec", "micro_batch_forward_sec", "backward_sec",
    "optimizer_step_sec", "checkpoint_sec", "decode_tokens", "rollout_generation_split_count",
)
EVENT_FILES = ("logs/events.jsonl", "nohup.out", "logs/train.log", "train.log")


def json_lines(path: Path) -> list[dict[str, Any]]:
    """Every line of ``path`` that parses as a JSON object (others are skipped)."""
    out = []
    for line in path.read_text(encoding="utf-8", errors="replace").splitlines():
        line = line.strip()
        if line.startswith("{"):
            try:
                value = json.loads(line)
            except json.JSONDecodeError:
                continue
            if isinstance(value, dict):
                out.append(value)
    return out


def train_steps(run_dir: Path) -> list[dict[str, Any]]:
    """``train_step`` events, one per step (a step logged twice keeps its last copy)."""
    by_step: dict[Any, dict[str, Any]] = {}
    for name in EVENT_FILES:
        path = run_dir / name
        if path.exists():
            for event in json_lines(path):
                if event.get("event") == "train_step":
                    key = event.get("step", event.get("run", {}).get("step"))
                    by_step[key if key is not None else len(by_step)] = event
    return list(by_step.values())


def _get(d: Any, *path: str) -> Any:
    for key in path:
        if not isinstance(d, dict):
            return None
        d = d.get(key)
    return d


def _mean(rows: list[dict[str, Any]], key: str) -> float | None:
    vals = [float(r[key]) for r in rows if r.get(key) is not None]
    return mean(vals) if vals else None


def gpu_summary(run_dir: Path) -> dict[str, Any]:
    summary = run_dir / "gpu_memory" / "gpu_memory_summary.json"
    if summary.exists():
        data = json.loads(summary.read_text(encoding="utf-8"))
        return {"sample_count": data.get("sample_count"), "per_gpu": {
            str(g): {k: v.get(k) for k in ("samples", "memory_used_mib_peak", "memory_used_mib_p95",
                                           "memory_used_mib_mean", "utilization_gpu_pct_mean")}
            for g, v in (data.get("per_gpu") or {}).items()}}
    rows_path = run_dir / "gpu_memory" / "gpu_memory.jsonl"
    if not rows_path.exists():
        return {}
    from graspo_b200.analysis.gpu_memory import summarize_samples

    return summarize_samples(json_lines(rows_path))


def rank_summary(run_dir: Path) -> dict[str, Any]:
    latest: dict[int, dict[str, Any]] = {}
    for path in sorted(run_dir.glob("logs/rank_metrics.rank_*.jsonl")) + sorted(run_dir.glob("rank_metrics.rank_*.jsonl")):
        for row in json_lines(path):
            if "rank" in row:   # the last event of each rank: phase, memory snapshot, metrics
                latest[int(row["rank"])] = row
    return {"per_rank": {str(r): m for r, m in sorted(latest.items())}}


def summarize_run(run_dir: str | Path, *, skip_warmup_steps: int = 1) -> dict[str, Any]:
    run_dir = Path(run_dir)
    steps = train_steps(run_dir)
    measured = steps[skip_warmup_steps:] if len(steps) > skip_warmup_steps else steps
    latest = steps[-1] if steps else {}
    timing = [dict(s.get("timing") or {}) for s in measured]
    total_sec = _mean(timing, "total_observed_sec")
    decode_tokens = sum(float(t.get("decode_tokens") or 0) for t in timing)
    rollout_sec = sum(float(t.get("rollout_sec") or 0) for t in timing)
    trainable = sum(float(_get(s, "batch", "decisions", "trainable", "total") or 0) for s in measured)
    decisions = _get(latest, "batch", "decisions") or {}
    return {
        "run_dir": str(run_dir),
        "name": run_dir.name,
        "step_count": len(steps),
        "measured_step_count": len(measured),
        "latest_step": latest.get("step", _get(latest, "run", "optimized_steps")),
        "latest_epoch": _get(latest, "epoch", "epoch"),
        "latest_reward_mean": _get(latest, "batch", "reward", "mean"),
        "latest_content_mean": _get(latest, "batch", "content", "mean"),
        "latest_trainable_groups": _get(decisions, "trainable", "total"),
        "latest_invalid": _get(decisions, "terminal", "invalid"),
        "latest_invalid_no_preference_gap": _get(decisions, "terminal", "invalid_no_preference_gap"),
        "timing_mean": {k: _mean(timing, k) for k in TIMING_KEYS},
        "latest_timing": {k: v for k, v in (latest.get("timing") or {}).items() if k in TIMING_KEYS},
        "decode_tokens_per_sec": decode_tokens / rollout_sec if rollout_sec > 0 else None,
        "trainable_groups_per_hour": (trainable * 3600.0 / (total_sec * len(measured))
                                      if total_sec and measured else None),
        "gpu": gpu_summary(run_dir),
        "rank": rank_summary(run_dir),
    }


def format_table(summaries: list[dict[str, Any]]) -> str:
    cols = ("name", "step_count", "latest_reward_mean", "decode_tokens_per_sec", "trainable_groups_per_hour")
    lines = ["\t".join(cols)]
    for s in summaries:
        row = []
        for c in cols:
            v = s.get(c)
            row.append(f"{v:.3f}" if isinstance(v, float) else str(v))
        tm = s["timing_mean"]
        lines.append("\t".join(row))
        lines.append("  mean sec: " + ", ".join(f"{k}={tm[k]:.3f}" for k in ("total_observed_sec", "rollout_sec",
                     "old_logprob_sec", "optimize_sec") if tm.get(k) is not None))
    return "\n".join(lines)


def main(argv: list[str] | None = None) -> int:
    p = argparse.ArgumentParser(description="Summarise GRASPO run outputs (train_step events).")
    p.add_argument("run_dirs", nargs="+")
    p.add_argument("--skip-warmup-steps", type=int, default=1)
    p.add_argument("--json", action="store_true")
    args = p.parse_args(argv)
    summaries = [summarize_run(d, skip_warmup_steps=args.skip_warmup_steps) for d in args.run_dirs]
    print(json.dumps(summaries, indent=2, ensure_ascii=False) if args.json else format_table(summaries))
    return 0


if __name__ == "__main__":
    raise SystemExit(main())
