"""``graspo`` command line: ``launch``, ``export``, ``validate-reward``.

``graspo launch --config X.yaml`` validates the config and paths, resolves the
world size (``tp * pp * dp``; ``launch.nproc_per_node`` / ``launch.gpus`` may
pin it), and runs the training worker -- directly for one process, under
``torchrun`` (rendezvous on ``launch.master_addr``) otherwise (reference:
cli/app.py:51-233).  ``graspo export`` turns a native checkpoint into a PEFT
adapter or a merged Hugging Face model.  ``graspo validate-reward`` loads a
JSONL file through the strict validator and scores completions (given in the
records as ``completion``/``completions``, or rendered from the targets) with
the configured reward, printing a JSON summary.
"""

from __future__ import annotations

import argparse
import json
import os
import shutil
import subprocess
import sys
from dataclasses import dataclass
from pathlib import Path
from typing import Any

from graspo_b200.core.schema import GraspoConfig

SUPPORTED_BACKENDS = {"graspoflow"}


@dataclass(slots=True)
class BackendSelection:
    name: str
    reason: str
    requested: str


def select_backend(config: GraspoConfig, requested: str | None = None) -> BackendSelection:
    name = (requested or config.backend or "graspoflow").strip()
    if name not in SUPPORTED_BACKENDS:
        raise ValueError(f"Unsupported backend '{name}'. GRASPO only supports 'graspoflow'.")
    return BackendSelection("graspoflow", "TP x PP x DP LoRA training on sm_100a kernels", name)


@dataclass(slots=True)
class LaunchPlan:
    command: list[str]
    env: dict[str, str]
    backend: str
    uses_torchrun: bool
    nproc_per_node: int
    nnodes: int


def _require(value: Any, name: str) -> None:
    text = str(value or "").strip()
    if not text or "${" in text or text.startswith("<"):
        raise SystemExit(f"{name} must be set in the YAML config")


def _format_gpus(value) -> str | None:
    if value is None:
        return None
    parts = [p.strip() for p in value.split(",")] if isinstance(value, str) else [str(int(v)) for v in value]
    parts = [p for p in parts if p]
    return ",".join(parts) or None


def world_size(config: GraspoConfig, nproc_total: int | None = None) -> int:
    flow = config.graspoflow
    base = int(flow.tp_size) * int(flow.pp_size)
    if int(flow.dp_size) > 0:
        return base * int(flow.dp_size)
    return nproc_total or base


def build_launch_plan(config_path: str | Path, config: GraspoConfig | None = None) -> LaunchPlan:
    config_path = Path(config_path)
    if not config_path.is_file():
        raise SystemExit(f"Config file does not exist: {config_path}")
    config = config or GraspoConfig.from_yaml(config_path)
    selection = select_backend(config)
    launch = config.launch
    nnodes = int(launch.nnodes)
    if nnodes < 1:
        raise SystemExit("launch.nnodes must be >= 1")
    if launch.nproc_per_node is not None:
        nproc = int(launch.nproc_per_node)
    else:
        world = world_size(config)
        if world % nnodes:
            raise SystemExit(f"graspoflow world size must divide evenly across launch.nnodes ({world} % {nnodes} != 0)")
        nproc = world // nnodes
    if nproc < 1:
        raise SystemExit("launch.nproc_per_node must be >= 1")
    _require(config.model.model_path, "model.model_path")
    _require(config.data.train_path, "data.train_path")
    if not Path(config.data.train_path).is_file():
        raise SystemExit(f"data.train_path does not exist: {config.data.train_path}")
    Path(config.training.output_dir).mkdir(parents=True, exist_ok=True)
    actual = nnodes * nproc
    flow = config.graspoflow
    cell = int(flow.tp_size) * int(flow.pp_size)
    if actual % cell or (int(flow.dp_size) > 0 and actual != cell * int(flow.dp_size)):
        raise SystemExit(
            f"graspoflow launch world size must equal tp_size x pp_size x dp_size ({actual} vs "
            f"{cell} x {flow.dp_size or actual // max(cell, 1)})"
        )
    gpus = _format_gpus(launch.gpus)
    if gpus is not None and len(gpus.split(",")) != nproc:
        raise SystemExit(f"launch.gpus count must match launch.nproc_per_node ({len(gpus.split(','))} != {nproc})")
    env = dict(os.environ)
    env.update({str(k): str(v) for k, v in launch.env.items()})
    env.setdefault("TOKENIZERS_PARALLELISM", "false")
    # one run name for every worker (auto-named runs would otherwise race on the clock)
    env.setdefault("GRASPO_RUN_NAME", config.training.run_name)
    if gpus is not None:
        env["CUDA_VISIBLE_DEVICES"] = gpus
    root = str(Path(__file__).resolve().parents[2])
    env["PYTHONPATH"] = root if not env.get("PYTHONPATH") else f"{root}{os.pathsep}{env['PYTHONPATH']}"
    python = str(launch.python or sys.executable)
    worker = ["-m", "graspo_b200.cli.train_worker", "--config", str(config_path)]
    uses_torchrun = actual > 1
    if uses_torchrun:
        if launch.torchrun:
            prefix = [str(launch.torchrun)]
        elif shutil.which("torchrun"):
            prefix = [shutil.which("torchrun")]
        else:
            prefix = [python, "-m", "torch.distributed.run"]
        command = prefix + [f"--nnodes={nnodes}", f"--node_rank={int(launch.node_rank)}",
                            f"--nproc_per_node={nproc}", f"--master_addr={launch.master_addr}",
                            f"--master_port={int(launch.master_port)}"] + worker
    else:
        command = [python] + worker
    return LaunchPlan(command, env, selection.name, uses_torchrun, nproc, nnodes)


def cmd_launch(args: argparse.Namespace) -> int:
    plan = build_launch_plan(args.config)
    print(json.dumps({"backend": plan.backend, "uses_torchrun": plan.uses_torchrun, "nnodes": plan.nnodes,
                      "nproc_per_node": plan.nproc_per_node, "command": plan.command}, ensure_ascii=False))
    if getattr(args, "dry_run", False):
        return 0
    return int(subprocess.run(plan.command, env=plan.env, check=False).returncode)


def cmd_export(args: argparse.Namespace) -> int:
    config = GraspoConfig.from_yaml(args.config)
    _require(config.export.checkpoint_path, "export.checkpoint_path")
    _require(config.export.export_output, "export.export_output")
    _require(config.model.model_path, "model.model_path")
    from graspo_b200.models.lora_io import export_from_checkpoint

    export_from_checkpoint(config.export.checkpoint_path, config.export.export_output,
                           export_format=config.export.export_format, base_model_path=config.model.model_path)
    print(json.dumps({"checkpoint": config.export.checkpoint_path, "format": config.export.export_format,
                      "output": config.export.export_output, "base_model": config.model.model_path},
                     ensure_ascii=False))
    return 0


def validate_reward(records_path: str | Path, config: GraspoConfig, limit: int | None = None) -> dict[str, Any]:
    """Validate a JSONL file and score its completions; returns the summary."""
    from graspo_b200.core.data import build_sft_target_text, sample_from_record
    from graspo_b200.core.decisions import lower_median
    from graspo_b200.core.reward import GraspoReward
    from graspo_b200.core.tool_parser import parse_qwen_tool_completion

    reward = GraspoReward(config.reward)
    rows, errors, scores = 0, [], []
    with Path(records_path).open("r", encoding="utf-8") as handle:
        for line_no, line in enumerate(handle, start=1):
            if not line.strip():
                continue
            if limit is not None and rows >= limit:
                break
            rows += 1
            try:
                record = json.loads(line)
                extra = {k: record.pop(k) for k in ("completion", "completions") if k in record}
                sample = sample_from_record(record)
            except Exception as exc:  # noqa: BLE001 - reported per line
                errors.append({"line": line_no, "error": str(exc)})
                continue
            texts = extra.get("completions") or ([extra["completion"]] if "completion" in extra else
                                                 [build_sft_target_text(sample.targets[0]["output"])])
            for text in texts:
                parsed = parse_qwen_tool_completion(text, expect_tool_calls=sample.expects_tool_calls,
                                                    tools=sample.tools)
                res = reward.score_parsed(parsed, sample.targets, is_tool_call=sample.expects_tool_calls)
                scores.append({"line": line_no, "reward": res.reward, "content_score": res.content_score,
                               "all_right": res.all_right})
    rewards = [s["reward"] for s in scores]
    return {
        "path": str(records_path), "records": rows, "valid_records": rows - len(errors), "invalid_records": len(errors),
        "errors": errors[:20], "scored_completions": len(scores),
        "reward": {"min": min(rewards) if rewards else 0.0, "median": lower_median(rewards),
                   "mean": sum(rewards) / len(rewards) if rewards else 0.0, "max": max(rewards) if rewards else 0.0},
        "all_right_rate": sum(s["all_right"] for s in scores) / len(scores) if scores else 0.0,
    }


def cmd_validate_reward(args: argparse.Namespace) -> int:
    config = GraspoConfig.from_yaml(args.config) if args.config else GraspoConfig.from_dict({})
    path = args.data or config.data.train_path
    _require(path, "--data or data.train_path")
    summary = validate_reward(path, config, args.limit)
    print(json.dumps(summary, ensure_ascii=False))
    return 0 if summary["invalid_records"] == 0 else 1


def build_parser() -> argparse.ArgumentParser:
    parser = argparse.ArgumentParser(prog="graspo", description="GRASPO training utilities (B200 build).")
    sub = parser.add_subparsers(dest="command", required=True)
    launch = sub.add_parser("launch", help="Launch training from a single YAML config.")
    launch.add_argument("--config", "-c", required=True)
    launch.add_argument("--dry-run", action="store_true", help="print the launch plan without running it")
    launch.set_defaults(func=cmd_launch)
    export = sub.add_parser("export", help="Export a native GRASPO checkpoint to a PEFT adapter or merged model.")
    export.add_argument("--config", "-c", required=True)
    export.set_defaults(func=cmd_export)
    val = sub.add_parser("validate-reward", help="Validate JSONL records and score completions with the reward.")
    val.add_argument("--config", "-c", default=None)
    val.add_argument("--data", "-d", default=None)
    val.add_argument("--limit", type=int, default=None)
    val.set_defaults(func=cmd_validate_reward)
    return parser


def main(argv: list[str] | None = None) -> None:
    args = build_parser().parse_args(argv)
    raise SystemExit(args.func(args))


if __name__ == "__main__":
    main()
