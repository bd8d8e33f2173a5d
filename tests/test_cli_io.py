"""CLI launch plans, validate-reward, LoRA I/O round trips, fault injection."""

import json
import os
from pathlib import Path

import pytest
import torch
import yaml

from graspo_b200.cli.app import build_launch_plan, build_parser, validate_reward
from graspo_b200.core.schema import GraspoConfig


def _write_cfg(tmp: Path, **flow) -> Path:
    data = tmp / "train.jsonl"
    data.write_text(json.dumps({"messages": [{"role": "user", "content": "x"}],
                                "targets": [{"output": {"content": {"a": "b"}}}]}) + "\n")
    cfg = {"model": {"model_path": str(tmp)}, "data": {"train_path": str(data)},
           "training": {"output_dir": str(tmp / "out")}, "graspoflow": {"tp_size": 2, "pp_size": 1, **flow},
           "launch": {"master_addr": "127.0.0.1"}}
    path = tmp / "c.yaml"
    path.write_text(yaml.safe_dump(cfg))
    return path


def test_parser_commands():
    parser = build_parser()
    for cmd in ("launch", "export"):
        assert parser.parse_args([cmd, "--config", "x.yaml"]).command == cmd
    assert parser.parse_args(["validate-reward", "--data", "d.jsonl"]).command == "validate-reward"


def test_launch_plans(tmp_path):
    plan = build_launch_plan(_write_cfg(tmp_path))
    assert plan.uses_torchrun and plan.nproc_per_node == 2
    assert "--master_addr=127.0.0.1" in plan.command and "graspo_b200.cli.train_worker" in plan.command
    plan = build_launch_plan(_write_cfg(tmp_path, tp_size=1))
    assert not plan.uses_torchrun and plan.nproc_per_node == 1
    plan = build_launch_plan(_write_cfg(tmp_path, dp_size=4))
    assert plan.nproc_per_node == 8
    cfg = yaml.safe_load(_write_cfg(tmp_path).read_text())
    cfg["launch"]["gpus"] = [0, 1, 2]
    path = tmp_path / "bad.yaml"
    path.write_text(yaml.safe_dump(cfg))
    with pytest.raises(SystemExit):
        build_launch_plan(path)
    cfg["launch"]["gpus"] = "4,5"
    path.write_text(yaml.safe_dump(cfg))
    assert build_launch_plan(path).env["CUDA_VISIBLE_DEVICES"] == "4,5"


def test_validate_reward(tmp_path):
    rows = [
        {"messages": [{"role": "user", "content": "q"}], "targets": [{"output": {"content": {"k": "v"}}}],
         "completion": '```json\n{"k": "v"}\n```'},
        {"messages": [{"role": "user", "content": "q"}], "targets": [{"output": {"content": {"k": "v"}}}]},
        {"prompt": "removed field", "targets": []},
    ]
    path = tmp_path / "d.jsonl"
    path.write_text("\n".join(json.dumps(r) for r in rows) + "\n")
    summary = validate_reward(path, GraspoConfig.from_dict({}))
    assert summary["records"] == 3 and summary["invalid_records"] == 1
    assert summary["scored_completions"] == 2 and summary["all_right_rate"] == 1.0


def _tiny_model(tmp, tp_size=1):
    from graspo_b200.models.config import load_decoder_config
    from graspo_b200.models.loader import SafetensorIndex
    from graspo_b200.models.qwen3 import Qwen3Model
    from graspo_b200.parallel.state import ParallelState
    from graspo_b200.utils.synth import TINY, write_qwen3_checkpoint

    path = write_qwen3_checkpoint(tmp / "base", TINY, seed=1, device="cpu", with_tokenizer=False)
    targets = {"language.self_attn.q_proj", "language.self_attn.o_proj", "language.mlp.down_proj"}
    m = Qwen3Model(load_decoder_config(path), SafetensorIndex(path), ps=ParallelState(), lora_targets=targets,
                   lora_r=4, lora_alpha=8, dtype=torch.float32, device=torch.device("cpu"))
    with torch.no_grad():
        m.lora.params.normal_(0, 0.05)
    return m, path


class _Adapter:
    """Just enough of an adapter for save_rank_checkpoint."""

    def __init__(self, model, cfg):
        from graspo_b200.engine.optim import FlatAdamW
        from graspo_b200.parallel.state import ParallelState

        self.ps = ParallelState()
        self.model = model
        self.placement = None
        self.optimizer = FlatAdamW(model.lora, lr=1e-3, weight_decay=0.0)
        self.config = cfg
        self._train_batch_call_index = 3


def test_checkpoint_peft_and_merged_round_trip(tmp_path):
    from safetensors.torch import load_file

    from graspo_b200.models.lora_io import export_merged_hf, export_peft_adapter, load_peft_adapter
    from graspo_b200.train.checkpoint import load_rank_checkpoint, read_manifest, save_rank_checkpoint

    model, base = _tiny_model(tmp_path)
    cfg = GraspoConfig.from_dict({"model": {"model_path": str(base)}, "lora": {"r": 4, "alpha": 8}})
    adapter = _Adapter(model, cfg)
    save_rank_checkpoint(adapter, tmp_path / "ckpt", trainer_state={"global_step": 5})
    manifest = read_manifest(tmp_path / "ckpt")
    assert manifest["checkpoint_type"] == "recoverable_lora_training_state" and manifest["has_trainer_state"]
    saved = model.lora.params.clone()
    with torch.no_grad():
        model.lora.params.zero_()
    state = load_rank_checkpoint(adapter, tmp_path / "ckpt")
    assert state == {"global_step": 5} and torch.equal(model.lora.params, saved)
    assert adapter._train_batch_call_index == 3

    export_peft_adapter(tmp_path / "ckpt", tmp_path / "peft", base_model_path=str(base))
    with torch.no_grad():
        model.lora.params.zero_()
    load_peft_adapter(model, tmp_path / "peft", base_model_path=str(base))
    assert torch.allclose(model.lora.params, saved)

    export_merged_hf(tmp_path / "ckpt", tmp_path / "merged", base_model_path=base)
    merged = {}
    for f in (tmp_path / "merged").glob("*.safetensors"):
        merged.update(load_file(str(f)))
    orig = {}
    for f in Path(base).glob("*.safetensors"):
        orig.update(load_file(str(f)))
    mod = model.lora.module(0, "q")
    delta = (mod.b @ mod.a) * 2.0
    name = "model.layers.0.self_attn.q_proj.weight"
    assert torch.allclose(merged[name].float(), (orig[name].float() + delta).bfloat16().float(), atol=1e-2)
    assert torch.equal(merged["model.layers.0.mlp.up_proj.weight"], orig["model.layers.0.mlp.up_proj.weight"])
    with pytest.raises(FileExistsError):
        export_peft_adapter(tmp_path / "ckpt", tmp_path / "peft")


def test_fault_injector(monkeypatch):
    from graspo_b200.train.trainer import FaultInjector, InjectedFault

    monkeypatch.setenv("GRASPO_FAULT", "optimize:2")
    inj = FaultInjector(rank=0)
    inj.hit("optimize")
    with pytest.raises(InjectedFault):
        inj.hit("optimize")
    monkeypatch.setenv("GRASPO_FAULT_RANK", "1")
    inj = FaultInjector(rank=0)
    inj.hit("optimize")
    inj.hit("optimize")  # other rank: never fires


def test_every_shipped_config_loads_and_plans(tmp_path, monkeypatch):
    """Each YAML under configs/ validates against the strict schema and gives a
    launch plan whose world matches tp x pp x dp (paths made to exist here)."""

    root = Path(__file__).resolve().parents[1] / "configs"
    files = sorted(root.glob("*.yaml"))
    assert len(files) >= 6
    monkeypatch.chdir(tmp_path)
    data = tmp_path / "train.jsonl"
    data.write_text(json.dumps({"messages": [{"role": "user", "content": "x"}],
                                "targets": [{"output": {"content": {"a": 1}}}]}) + "\n")
    for f in files:
        raw = yaml.safe_load(f.read_text())
        raw["data"]["train_path"] = str(data)
        raw["training"]["output_dir"] = str(tmp_path / "out" / f.stem)
        raw.setdefault("launch", {}).pop("gpus", None)
        path = tmp_path / f.name
        path.write_text(yaml.safe_dump(raw))
        cfg = GraspoConfig.from_yaml(path)
        plan = build_launch_plan(path, cfg)
        flow = cfg.graspoflow
        cell = flow.tp_size * flow.pp_size
        assert plan.nproc_per_node % cell == 0, f.name
        if flow.dp_size:
            assert plan.nproc_per_node == cell * flow.dp_size, f.name
        assert plan.uses_torchrun == (plan.nproc_per_node > 1), f.name


@pytest.mark.parametrize("command", ["train", "prepare-data", "analyze"])
def test_removed_commands_are_not_public(command):
    """Only launch / export / validate-reward are public (validate-reward is kept:
    the reference README documents it and the baseline asks for it)."""
    with pytest.raises(SystemExit):
        build_parser().parse_args([command])


def test_world_size_one_runs_in_process(tmp_path):
    plan = build_launch_plan(_write_cfg(tmp_path, tp_size=1))
    assert not plan.uses_torchrun and plan.nproc_per_node == 1
    assert "torchrun" not in " ".join(plan.command)
