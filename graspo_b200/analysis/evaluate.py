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
from typing import Any

from graspo_b200.analysis.scoring import score_row, summarize, write_report
from graspo_b200.core.completion import raw_parsed_completion
from graspo_b200.core.reward import GraspoReward


def evaluate_samples(runtime, config, samples: list, output_dir: str | Path, *,
                     checkpoint: str | None = None) -> dict[str, Any]:
    """Score ``rollout_group_size`` completions per sample; returns the summary."""
    tr = config.training
    reward = GraspoReward(config.reward)
    primary = bool(getattr(runtime, "is_primary", lambda: True)())
    parse = getattr(runtime, "parse_completion", None)
    t0 = time.monotonic()
    rows = []
    for idx, sample in enumerate(samples):
        (gen,) = runtime.generate_sample_groups(
            samples=[sample], rollout_group_size=tr.rollout_group_size, max_new_tokens=tr.max_new_tokens,
            max_prompt_length=config.data.max_prompt_length, temperature=tr.temperature, top_p=tr.top_p,
            chat_template_kwargs=config.model.chat_template_kwargs)
        for j, text in enumerate(gen.completions):
            parsed = parse(text, sample) if callable(parse) else raw_parsed_completion(text)
            rows.append(score_row(reward, parsed, sample, sample_index=idx, completion_index=j))
    summary = summarize(rows, len(samples), checkpoint=checkpoint, rollout_group_size=int(tr.rollout_group_size),
                        elapsed_sec=round(time.monotonic() - t0, 3))
    if primary:
        write_report(output_dir, rows, summary)
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
