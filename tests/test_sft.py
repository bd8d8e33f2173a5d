"""Supervised fine-tuning end to end (CPU, one process) on both model families.

``SFTTrainer`` tokenizes prompt + target (labels masked on the prompt), runs
``train_batch_sft`` batches and writes the final checkpoint; repeated passes
over a tiny dataset must lower the token cross-entropy, and the metrics carry
the phase timers.  Reference behaviour: trainer/sft_trainer.py:26-172,
qwen35_36/training.py:25-154.
"""

import json

import pytest
import torch


@pytest.mark.parametrize("family", ["qwen3", "qwen3_5"])
def test_sft_lowers_the_loss_and_checkpoints(tmp_path, family, capsys):
    from graspo_b200.core.schema import GraspoConfig
    from graspo_b200.engine.runtime import GraspoFlowRuntime
    from graspo_b200.train.sft_trainer import SFTTrainer
    from graspo_b200.utils.synth import (QWEN35_TINY, TINY, synthetic_json_records, write_jsonl_records,
                                         write_qwen3_checkpoint, write_qwen35_checkpoint)

    if family == "qwen3":
        path = write_qwen3_checkpoint(tmp_path / "m", TINY, seed=1, device="cpu", dtype=torch.float32)
        targets = ["language.self_attn.q_proj", "language.self_attn.v_proj", "language.mlp.down_proj"]
    else:
        path = write_qwen35_checkpoint(tmp_path / "m", QWEN35_TINY, seed=1, std=0.05, dtype=torch.float32)
        targets = ["language.full_attn.q_proj", "language.linear_attn.v_proj", "language.mlp.down_proj"]
    data = write_jsonl_records(synthetic_json_records(2, seed=0), tmp_path / "sft.jsonl")
    cfg = GraspoConfig.from_dict({
        "train_method": "sft",
        "model": {"model_path": str(path), "torch_dtype": "float32", "gradient_checkpointing": False},
        "data": {"train_path": str(data), "max_prompt_length": 256},
        "lora": {"r": 8, "alpha": 16, "dropout": 0.0, "target_modules": targets},
        "training": {"output_dir": str(tmp_path / "run"), "run_name": "sft", "optimize_prompt_batch_size": 2,
                     "learning_rate": 5e-3, "max_new_tokens": 128, "max_epochs": 12, "max_steps": 12,
                     "save_checkpoint_every_epoch": False},
        "graspoflow": {"tp_size": 1, "pp_size": 1, "forward_batch_size": 2, "raw_log_enabled": False,
                       "readable_log_enabled": False},
    })
    runtime = GraspoFlowRuntime.from_config(cfg)
    metrics = []

    def recording(*args, **kwargs):      # the runtime forwards to its adapter once set up
        out = runtime.adapter.train_batch_sft(*args, **kwargs)
        metrics.append(out)
        return out

    runtime.train_batch_sft = recording
    SFTTrainer(cfg, runtime=runtime).train()
    assert len(metrics) == 12
    losses = [m["loss_mean"] for m in metrics]
    assert losses[-1] < 0.9 * losses[0] and losses[-1] == min(losses), losses
    for key in ("micro_batch_forward_sec", "backward_sec", "optimizer_step_sec"):
        assert metrics[-1][key] > 0, key
    final = tmp_path / "run" / "final"
    manifest = json.loads((final / "manifest.json").read_text())
    assert manifest["has_trainer_state"]
    steps = [json.loads(line) for line in capsys.readouterr().out.splitlines() if line.startswith("{")]
    assert sum(1 for e in steps if e.get("event") == "sft_step") == 12


@pytest.mark.parametrize("family", ["qwen3", "qwen3_5"])
def test_sft_with_images(tmp_path, family):
    """Multimodal SFT records (reference: models/qwen35_36/training.py:75-90):
    each image placeholder becomes one token per merged vision patch (labels
    -100 there), the image features condition the loss, and LoRA on the vision
    tower trains through them."""
    from graspo_b200.core.data import sample_from_record, sft_tokenize
    from graspo_b200.core.schema import GraspoConfig
    from graspo_b200.engine.runtime import GraspoFlowRuntime
    from graspo_b200.utils.synth import (QWEN35_TINY, TINY, VIT_TINY, add_vision_tower, synthetic_image_records,
                                         write_qwen3_checkpoint, write_qwen35_checkpoint)

    if family == "qwen3":
        base = write_qwen3_checkpoint(tmp_path / "vl", dict(TINY, vocab_size=2048), seed=1, device="cpu")
        targets = ["language.self_attn.q_proj", "language.mlp.down_proj", "vision_merger"]
    else:
        base = write_qwen35_checkpoint(tmp_path / "vl35", dict(QWEN35_TINY, vocab_size=2048, head_dim=64), seed=1,
                                       std=0.05)
        targets = ["language.full_attn.q_proj", "language.mlp.down_proj", "vision_merger"]
    path = add_vision_tower(base, VIT_TINY, seed=2)
    cfg = GraspoConfig.from_dict({
        "train_method": "sft",
        "model": {"model_path": str(path), "torch_dtype": "float32", "gradient_checkpointing": False},
        "data": {"train_path": "", "max_prompt_length": 600},
        "lora": {"r": 4, "alpha": 8, "dropout": 0.0, "target_modules": targets},
        "training": {"output_dir": str(tmp_path / "run"), "run_name": "sft", "optimize_prompt_batch_size": 2,
                     "learning_rate": 1e-2},
        "graspoflow": {"tp_size": 1, "pp_size": 1, "forward_batch_size": 2, "raw_log_enabled": False,
                       "readable_log_enabled": False},
    })
    (tmp_path / "run" / "logs").mkdir(parents=True)
    api = GraspoFlowRuntime.from_config(cfg)
    api.setup()
    ad = api.adapter
    samples = [sample_from_record(r) for r in synthetic_image_records(2, tmp_path / "img", seed=3, size=64,
                                                                      text_words=4)]
    items = [sft_tokenize(s, ad.tokenizer, max_seq_length=600) for s in samples]
    assert all("_multimodal_row" in it for it in items)
    pad = ad._vision_pad_id
    ids, labels, media = ad._sft_images(items[0])
    assert int((ids == pad).sum()) == 4 and len(media) == 1          # 64 x 64 image -> 2 x 2 merged tokens
    assert bool((labels[ids == pad] == -100).all())
    assert int((labels != -100).sum()) == int((items[0]["labels"] != -100).sum())
    lora = ad.model.lora
    start = lora.params.clone()
    vis = [m.module_name for m in lora.vision_modules()]
    assert vis
    with_images = ad.train_batch_sft(items, optimize_iterations_per_step=1, max_grad_norm=1.0)["loss_mean"]
    moved = [n for n in vis if lora.by_name[n].b.abs().max() > 0]
    assert moved, "the step trained the tower's LoRA factors"
    with torch.no_grad():
        lora.params.copy_(start)
    lora.invalidate()
    text_only = [{k: v for k, v in it.items() if k != "_multimodal_row"} for it in items]
    without = ad.train_batch_sft(text_only, optimize_iterations_per_step=1, max_grad_norm=1.0)["loss_mean"]
    assert abs(with_images - without) > 1e-6, (with_images, without)
