"""BASELINE config 0 end to end on CPU: `graspo launch` (2 gloo ranks, TP=2),
2 GRASPO steps, per-rank checkpoint + manifest, PEFT export, resume."""

import json
import os
import subprocess
import sys
from pathlib import Path

import pytest
import yaml

ROOT = Path(__file__).resolve().parents[1]


def _config(tmp: Path, **training) -> Path:
    from graspo_b200.utils.make_smoke_assets import make

    assets = make(tmp / "assets")
    cfg = yaml.safe_load((ROOT / "configs" / "config0_cpu_tp2.yaml").read_text())
    cfg["model"]["model_path"] = str(assets / "tiny-qwen3")
    cfg["data"]["train_path"] = str(assets / "train.jsonl")
    cfg["training"]["output_dir"] = str(tmp / "run")
    cfg["training"].update(training)
    cfg["launch"]["master_port"] = 29000 + os.getpid() % 2000
    # decode the 2 prompts of a step in two engine calls (one group of 4 rows each)
    cfg["graspoflow"].update(rollout_engine_batch=4, synchronize_cuda_timing=True)
    path = tmp / "config.yaml"
    path.write_text(yaml.safe_dump(cfg))
    return path


def _launch(config: Path) -> list[dict]:
    env = dict(os.environ, PYTHONPATH=str(ROOT), CUDA_VISIBLE_DEVICES="")
    proc = subprocess.run([sys.executable, "-m", "graspo_b200", "launch", "--config", str(config)], env=env,
                          capture_output=True, text=True, timeout=900, cwd=ROOT)
    assert proc.returncode == 0, proc.stdout[-3000:] + proc.stderr[-3000:]
    events = []
    for line in proc.stdout.splitlines():
        if line.startswith("{"):
            try:
                events.append(json.loads(line))
            except json.JSONDecodeError:
                pass
    return events


@pytest.mark.slow
def test_config0_tp2_gloo_end_to_end(tmp_path):
    config = _config(tmp_path)
    events = _launch(config)
    steps = [e for e in events if e.get("event") == "train_step"]
    assert len(steps) == 2, [e.get("event") for e in events]
    assert steps[-1]["optimize"]["optimizer_steps_per_rank"] >= 1
    final = tmp_path / "run" / "final"
    manifest = json.loads((final / "manifest.json").read_text())
    assert manifest["tp_size"] == 2 and manifest["format"] == "graspoflow-lora"
    assert sorted(p.name for p in final.glob("rank_*.pt")) == ["rank_00000_tp_00_pp_00.pt", "rank_00001_tp_01_pp_00.pt"]
    logs = tmp_path / "run" / "logs"
    assert (logs / "rollouts.readable.jsonl").exists() and (logs / "timing_events.jsonl").exists()
    # per-rank memory / metrics lines from both ranks, and the primary rank's event log
    for rank in (0, 1):
        lines = [json.loads(x) for x in (logs / f"rank_metrics.rank_{rank:05d}.jsonl").read_text().splitlines()]
        phases = {x["phase"] for x in lines}
        assert {"setup_after", "rollout_before", "rollout_after", "train_batch_after"} <= phases, phases
        assert all(x["rank"] == rank for x in lines)
    assert any(json.loads(x).get("event") == "train_step" for x in (logs / "events.jsonl").read_text().splitlines())
    groups = [json.loads(x) for x in (logs / "rollouts.readable.jsonl").read_text().splitlines()]
    assert groups and all(g["completions"] for g in groups)
    assert steps[0]["timing"]["rollout_generation_split_count"] >= 2

    # PEFT export through the CLI
    cfg = yaml.safe_load(config.read_text())
    cfg["export"] = {"checkpoint_path": str(final), "export_output": str(tmp_path / "peft"),
                     "export_format": "peft-adapter"}
    config.write_text(yaml.safe_dump(cfg))
    out = subprocess.run([sys.executable, "-m", "graspo_b200", "export", "--config", str(config)], cwd=ROOT,
                         env=dict(os.environ, PYTHONPATH=str(ROOT)), capture_output=True, text=True, timeout=300)
    assert out.returncode == 0, out.stderr[-2000:]
    adapter_cfg = json.loads((tmp_path / "peft" / "adapter_config.json").read_text())
    assert adapter_cfg["r"] == 8 and adapter_cfg["lora_alpha"] == 16 and "q_proj" in adapter_cfg["target_modules"]
    from safetensors.torch import load_file

    tensors = load_file(str(tmp_path / "peft" / "adapter_model.safetensors"))
    assert tensors["base_model.model.model.layers.0.self_attn.q_proj.lora_A.weight"].shape == (8, 128)
    assert tensors["base_model.model.model.layers.0.self_attn.q_proj.lora_B.weight"].shape == (128, 8)
    assert tensors["base_model.model.model.layers.0.self_attn.o_proj.lora_A.weight"].shape == (8, 128)

    # resume from the final checkpoint with one more step allowed
    cfg["training"]["resume_from_checkpoint"] = str(final)
    cfg["training"]["max_steps"] = 3
    cfg["training"]["output_dir"] = str(tmp_path / "run2")
    config.write_text(yaml.safe_dump(cfg))
    events = _launch(config)
    resumed = [e for e in events if e.get("event") == "checkpoint_resumed"]
    assert resumed and resumed[0]["global_step"] == 2
