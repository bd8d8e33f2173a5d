"""Evaluate a checkpoint: generate groups for held-out records and score them.

    python -m graspo_b200.analysis.evaluate --config run.yaml --data eval.jsonl \
        [--checkpoint OUTPUT/final] --output-dir OUT [--limit N] [--rollout-group-size G] \
        [--temperature T] [--top-p P]

Builds the runtime from the training config (same model, LoRA and parallel
layout; launch it with ``torchrun`` when the layout spans several ranks),
loads the recoverable checkpoint, generates ``rollout_group_size``
completions per record, scores them with the run's reward and writes
``completions.jsonl`` (one row per completion; media paths are reduced to
their type so private file names do not leak into reports) and
``summary.json``.  Reference behaviour: scripts/evaluate_native_checkpoint.py.
"""

from __future__ import annotations

import argparse
import json
import time
from pathlib import Path
from statistics import mean
from typing import Any

from graspo_b200.core.completion import raw_parsed_completion
from graspo_b200.core.reward import GraspoReward


def _scrubbed_metadata(sample) -> dict[str, Any]:
    meta = {k: v for k, v in (sample.metadata or {}).items() if k not in ("image", "images", "video", "videos")}
    meta["media"] = [{"type": m.get("type")} for m in (sample.media or [])]
    return meta


def evaluate_samples(runtime, config, samples: list, output_dir: str | Path, *,
                     checkpoint: str | None = None) -> dict[str, Any]:
    """Score ``rollout_group_size`` completions per sample; returns the summary."""
    out = Path(output_dir)
    out.mkdir(parents=True, exist_ok=True)
    tr = config.training
    reward = GraspoReward(config.reward)
    primary = bool(getattr(runtime, "is_primary", lambda: True)())
    t0 = time.monotonic()
    rows, group_rewards, group_ranges = [], [], []
    for idx, sample in enumerate(samples):
        (gen,) = runtime.generate_sample_groups(
            samples=[sample], rollout_group_size=tr.rollout_group_size, max_new_tokens=tr.max_new_tokens,
            max_prompt_length=config.data.max_prompt_length, temperature=tr.temperature, top_p=tr.top_p,
            chat_template_kwargs=config.model.chat_template_kwargs)
        parse = getattr(runtime, "parse_completion", None)
        rewards = []
        for text in gen.completions:
            parsed = parse(text, sample) if callable(parse) else raw_parsed_completion(text)
            res = reward.score_parsed(parsed, sample.targets, is_tool_call=sample.expects_tool_calls)
            rewards.append(float(res.reward))
            rows.append({"sample_index": idx, "completion": text, "reward": float(res.reward),
                         "content_score": float(res.content_score), "all_right": bool(res.all_right),
                         "matched_target_index": res.matched_target_index, "matched_target_id": res.matched_target_id,
                         "parse_errors": list(parsed.parse_errors), "targets": sample.targets,
                         "metadata": _scrubbed_metadata(sample)})
        group_rewards.append(rewards)
        group_ranges.append(max(rewards) - min(rewards) if rewards else 0.0)
    flat = [r["reward"] for r in rows]
    summary = {
        "checkpoint": checkpoint,
        "count": len(samples),
        "completion_count": len(rows),
        "rollout_group_size": int(tr.rollout_group_size),
        "reward_mean": mean(flat) if flat else 0.0,
        "reward_max_mean": mean(max(g) for g in group_rewards if g) if group_rewards else 0.0,
        "reward_range_mean": mean(group_ranges) if group_ranges else 0.0,
        "content_mean": mean(r["content_score"] for r in rows) if rows else 0.0,
        "all_right_rate": (sum(r["all_right"] for r in rows) / len(rows)) if rows else 0.0,
        "elapsed_sec": round(time.monotonic() - t0, 3),
    }
    if primary:
        with (out / "completions.jsonl").open("w", encoding="utf-8") as fh:
            for row in rows:
                fh.write(json.dumps(row, ensure_ascii=False) + "\n")
        (out / "summary.json").write_text(json.dumps(summary, indent=2) + "\n", encoding="utf-8")
    return summary


def main(argv: list[str] | None = None) -> int:
    p = argparse.ArgumentParser(description="Generate and score completions for an evaluation JSONL.")
    p.add_argument("--config", required=True)
    p.add_argument("--data", required=True)
    p.add_argument("--checkpoint")
    p.add_argument("--output-dir", required=True)
    p.add_argument("--limit", type=int, default=0)
    p.add_argument("--rollout-group-size", type=int)
    p.add_argument("--temperature", type=float)
    p.add_argument("--top-p", type=float)
    args = p.parse_args(argv)

    from graspo_b200.core.data import load_jsonl
    from graspo_b200.core.schema import GraspoConfig
    from graspo_b200.engine.runtime import GraspoFlowRuntime

    config = GraspoConfig.from_yaml(args.config)
    config.data.train_path = args.data
    config.training.output_dir = args.output_dir
    for key, value in (("rollout_group_size", args.rollout_group_size), ("temperature", args.temperature),
                       ("top_p", args.top_p)):
        if value is not None:
            setattr(config.training, key, value)
    samples = load_jsonl(args.data)
    if args.limit > 0:
        samples = samples[: args.limit]
    runtime = GraspoFlowRuntime.from_config(config)
    runtime.setup()
    if args.checkpoint:
        runtime.load_checkpoint(args.checkpoint)
    summary = evaluate_samples(runtime, config, samples, args.output_dir, checkpoint=args.checkpoint)
    if getattr(runtime, "is_primary", lambda: True)():
        print(json.dumps(summary))
    return 0


if __name__ == "__main__":
    raise SystemExit(main())
