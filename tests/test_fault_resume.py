"""Failure detection and resume on CPU ranks (gloo, TP=2).

* A rank that raises (host-side fault injection, ``GRASPO_FAULT``) ends the
  whole job with a non-zero exit well inside the process-group timeout: the
  launcher tears the surviving rank down instead of leaving it blocked in a
  collective.
* Resuming from the step-1 checkpoint and running to step 2 reproduces the
  uninterrupted run's LoRA weights and optimizer state exactly (same sample
  order, same rollout seeds, restored AdamW moments and RNG state).

Reference behaviour being extended: trainer/trainer.py:169-185 (resume from
``epoch_stats.samples_seen``), transformer_adapter.py:305-425 (checkpoint
payload); the reference has no fault injection or collective timeouts.
"""

import os
import subprocess
import sys
import time
from pathlib import Path

import pytest
import torch
import yaml

ROOT = Path(__file__).resolve().parents[1]


def _config(tmp: Path, name: str, flow: dict | None = None, **training) -> Path:
    from graspo_b200.utils.make_smoke_assets import make

    assets = make(tmp / "assets")
    cfg = yaml.safe_load((ROOT / "configs" / "config0_cpu_tp2.yaml").read_text())
    cfg["model"]["model_path"] = str(assets / "tiny-qwen3")
    cfg["data"]["train_path"] = str(assets / "train.jsonl")
    cfg["training"]["output_dir"] = str(tmp / name)
    cfg["training"].update(training)
    cfg["graspoflow"]["pg_timeout_sec"] = 60.0
    cfg["graspoflow"].update(flow or {})
    cfg["launch"]["master_port"] = 29000 + (os.getpid() * 7 + len(name)) % 2000
    path = tmp / f"{name}.yaml"
    path.write_text(yaml.safe_dump(cfg))
    return path


def _launch(config: Path, **env_extra) -> subprocess.CompletedProcess:
    env = {k: v for k, v in os.environ.items() if not k.startswith("GRASPO_FAULT")}
    env.update(PYTHONPATH=str(ROOT), CUDA_VISIBLE_DEVICES="", **env_extra)
    return subprocess.run([sys.executable, "-m", "graspo_b200", "launch", "--config", str(config)], env=env,
                          capture_output=True, text=True, timeout=600, cwd=ROOT)


@pytest.mark.slow
def test_failed_rank_ends_the_job(tmp_path):
    config = _config(tmp_path, "faulty", max_steps=2)
    t0 = time.monotonic()
    proc = _launch(config, GRASPO_FAULT="optimize:1", GRASPO_FAULT_RANK="1")
    elapsed = time.monotonic() - t0
    assert proc.returncode != 0
    assert "injected fault in optimize" in proc.stdout + proc.stderr
    assert elapsed < 300, elapsed
    # nothing claims to be a finished run
    assert not (tmp_path / "faulty" / "final" / "manifest.json").exists()


def _rank_state(ckpt: Path, rank: int) -> dict:
    name = f"rank_{rank:05d}_tp_{rank:02d}_pp_00.pt"
    return torch.load(ckpt / name, map_location="cpu", weights_only=False)


@pytest.mark.slow
def test_resume_reproduces_the_uninterrupted_run(tmp_path):
    full = _config(tmp_path, "full", max_steps=2, save_steps=1)
    proc = _launch(full)
    assert proc.returncode == 0, proc.stdout[-3000:] + proc.stderr[-3000:]
    step1 = tmp_path / "full" / "step_1"
    assert (step1 / "manifest.json").exists()
    resumed = _config(tmp_path, "resumed", max_steps=2, resume_from_checkpoint=str(step1))
    proc = _launch(resumed)
    assert proc.returncode == 0, proc.stdout[-3000:] + proc.stderr[-3000:]
    for rank in (0, 1):
        a = _rank_state(tmp_path / "full" / "final", rank)
        b = _rank_state(tmp_path / "resumed" / "final", rank)
        assert a["trainer_state"]["global_step"] == b["trainer_state"]["global_step"] == 2
        assert a["lora_state_dict"].keys() == b["lora_state_dict"].keys()
        for key, ta in a["lora_state_dict"].items():
            assert torch.equal(ta, b["lora_state_dict"][key]), key
        sa, sb = a["optimizer_state_dict"], b["optimizer_state_dict"]
        for key in sa:
            va, vb = sa[key], sb[key]
            if isinstance(va, torch.Tensor):
                assert torch.equal(va, vb), key


@pytest.mark.slow
def test_background_checkpoint_is_a_snapshot(tmp_path):
    """With graspoflow.async_checkpoint the step-1 shards are written by a
    background thread while step 2 trains; they must still hold the step-1
    state: resuming from them reproduces the uninterrupted run."""
    full = _config(tmp_path, "full", {"async_checkpoint": True}, max_steps=2, save_steps=1)
    proc = _launch(full)
    assert proc.returncode == 0, proc.stdout[-3000:] + proc.stderr[-3000:]
    step1 = tmp_path / "full" / "step_1"
    assert (step1 / "manifest.json").exists()
    resumed = _config(tmp_path, "resumed", max_steps=2, resume_from_checkpoint=str(step1))
    proc = _launch(resumed)
    assert proc.returncode == 0, proc.stdout[-3000:] + proc.stderr[-3000:]
    for rank in (0, 1):
        a = _rank_state(tmp_path / "full" / "final", rank)
        b = _rank_state(tmp_path / "resumed" / "final", rank)
        for key, ta in a["lora_state_dict"].items():
            assert torch.equal(ta, b["lora_state_dict"][key]), key
