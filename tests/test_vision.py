"""Vision tower + multimodal GRASPO on CPU: patch layout, placeholder expansion,
and an image-conditioned rollout / old log-probs / training round trip
through the public runtime API (Qwen3 and Qwen3.5 decoders with a ViT, eager
backend)."""

import pytest
import torch

from graspo_b200.models.vision import VisionConfig, expand_image_placeholders, merged_tokens, preprocess


def test_patch_layout_and_token_counts():
    cfg = VisionConfig(hidden_size=64, num_heads=4)
    img = torch.zeros(448, 448, 3, dtype=torch.uint8)
    img[:16, 16:32] = 255                                   # patch (row 0, col 1) bright
    patches, grid = preprocess(img, cfg)
    assert grid == (1, 28, 28) and patches.shape == (784, 1536)
    assert merged_tokens(grid, cfg) == 196
    # merge-block order: block (0, 0) holds patches (0,0), (0,1), (1,0), (1,1)
    bright = patches.mean(-1) > 0
    assert bright[1] and not bright[0] and not bright[2] and bright.sum() == 1
    assert expand_image_placeholders([1, 9, 2, 9, 3], 9, [2, 3]) == [1, 9, 9, 2, 9, 9, 9, 3]


@pytest.mark.parametrize("family", ["qwen3", "qwen3_5"])
def test_multimodal_grpo_round_trip(tmp_path, family):
    """Image prompts through the public runtime API on both families (the
    Qwen3.5 hybrid with multimodal RoPE positions): rollout, old log-probs
    that the image changes, one GRPO step."""
    from graspo_b200.core.buffer import Experience
    from graspo_b200.core.data import sample_from_record
    from graspo_b200.core.schema import GraspoConfig
    from graspo_b200.engine.runtime import GraspoFlowRuntime
    from graspo_b200.utils.synth import (QWEN35_TINY, TINY, VIT_TINY, add_vision_tower, synthetic_image_records,
                                         write_qwen3_checkpoint, write_qwen35_checkpoint)

    if family == "qwen3":
        dims = dict(TINY, vocab_size=2048)
        base = write_qwen3_checkpoint(tmp_path / "vl", dims, seed=1, device="cpu")
        targets = ["language.self_attn.q_proj", "language.mlp.down_proj"]
    else:
        dims = dict(QWEN35_TINY, vocab_size=2048, head_dim=64)
        base = write_qwen35_checkpoint(tmp_path / "vl35", dims, seed=1, std=0.05)
        targets = ["language.full_attn.q_proj", "language.linear_attn.out_proj", "language.mlp.down_proj"]
    path = add_vision_tower(base, VIT_TINY, seed=2)
    cfg = GraspoConfig.from_dict({
        "train_method": "graspo",
        "model": {"model_path": str(path), "torch_dtype": "float32"},
        "data": {"train_path": "", "max_prompt_length": 600},
        "lora": {"r": 4, "alpha": 8, "dropout": 0.0, "target_modules": targets},
        "training": {"output_dir": str(tmp_path / "run"), "run_name": "t", "rollout_group_size": 2,
                     "optimize_prompt_batch_size": 2, "learning_rate": 1e-3, "max_new_tokens": 4},
        "graspoflow": {"tp_size": 1, "pp_size": 1, "raw_log_enabled": False, "readable_log_enabled": False},
    })
    (tmp_path / "run" / "logs").mkdir(parents=True)
    api = GraspoFlowRuntime.from_config(cfg)
    api.setup()
    samples = [sample_from_record(r) for r in synthetic_image_records(2, tmp_path / "img", seed=3, size=64,
                                                                      text_words=4)]
    assert samples[0].media
    gens = api.generate_sample_groups(samples=samples, rollout_group_size=2, max_new_tokens=4, temperature=1.0,
                                      top_p=1.0)
    pad = api.adapter._vision_pad_id
    assert int((gens[0].sequences[0] == pad).sum()) == 4          # 64 x 64 image -> 2 x 2 merged tokens
    exps = []
    for gen in gens:
        old = api.sequence_log_probs(gen.sequences, gen.attention_mask, metadata=gen.metadata)
        # the image changes the log-probs of the text after it
        plain = api.sequence_log_probs(gen.sequences, gen.attention_mask)
        assert (old - plain).abs().max() > 1e-6
        for i in range(2):
            exps.append(Experience(sequences=gen.sequences[i], old_log_probs=old[i].cpu(),
                                   advantages=torch.full_like(old[i].cpu(), 1.0 - 2 * i),
                                   attention_mask=gen.attention_mask[i], action_mask=gen.action_mask[i],
                                   rewards=torch.zeros(()), metadata={"_media": gen.metadata["_media_rows"][i]}))
    before = api.adapter.model.lora.params.clone()
    metrics = api.train_batch(exps, policy_ratio_clip_eps=0.2, optimize_iterations_per_step=1, max_grad_norm=1.0)
    assert metrics["optimizer_steps"] == 2
    assert not torch.equal(before, api.adapter.model.lora.params)


def test_vision_lora_targets_train_and_export(tmp_path):
    """The reference's vision presets (``vision_common``: merger and every block's
    attention / MLP linears) become LoRA modules of the tower; one GRPO step moves
    their B factors (gradients reach them through the image-feature rows), and
    the PEFT export names them under ``model.visual``."""
    from graspo_b200.core.buffer import Experience
    from graspo_b200.core.data import sample_from_record
    from graspo_b200.core.schema import GraspoConfig
    from graspo_b200.engine.runtime import GraspoFlowRuntime
    from graspo_b200.utils.synth import TINY, VIT_TINY, add_vision_tower, synthetic_image_records, write_qwen3_checkpoint

    base = write_qwen3_checkpoint(tmp_path / "vl", dict(TINY, vocab_size=2048), seed=1, device="cpu")
    path = add_vision_tower(base, VIT_TINY, seed=2)
    cfg = GraspoConfig.from_dict({
        "train_method": "graspo",
        "model": {"model_path": str(path), "torch_dtype": "float32"},
        "data": {"train_path": "", "max_prompt_length": 600},
        "lora": {"r": 4, "alpha": 8, "dropout": 0.0,
                 "target_modules": ["language.self_attn.q_proj", "vision_common"]},
        "training": {"output_dir": str(tmp_path / "run"), "run_name": "t", "rollout_group_size": 2,
                     "optimize_prompt_batch_size": 2, "learning_rate": 1e-2, "max_new_tokens": 4},
        "graspoflow": {"tp_size": 1, "pp_size": 1, "raw_log_enabled": False, "readable_log_enabled": False},
    })
    (tmp_path / "run" / "logs").mkdir(parents=True)
    api = GraspoFlowRuntime.from_config(cfg)
    api.setup()
    lora = api.adapter.model.lora
    vis = lora.vision_modules()
    depth = VIT_TINY["depth"]
    assert len(vis) == 2 + 4 * depth
    assert {m.target_name for m in vis} >= {"visual.merger.linear_fc1", "visual.blocks.0.attn.qkv"}
    samples = [sample_from_record(r) for r in synthetic_image_records(2, tmp_path / "img", seed=3, size=64,
                                                                      text_words=4)]
    gens = api.generate_sample_groups(samples=samples, rollout_group_size=2, max_new_tokens=4, temperature=1.0,
                                      top_p=1.0)
    exps = []
    for gen in gens:
        old = api.sequence_log_probs(gen.sequences, gen.attention_mask, metadata=gen.metadata)
        for i in range(2):
            exps.append(Experience(sequences=gen.sequences[i], old_log_probs=old[i].cpu(),
                                   advantages=torch.full_like(old[i].cpu(), 1.0 - 2 * i),
                                   attention_mask=gen.attention_mask[i], action_mask=gen.action_mask[i],
                                   rewards=torch.zeros(()), metadata={"_media": gen.metadata["_media_rows"][i]}))
    before = {m.module_name: m.b.detach().clone() for m in vis}
    api.train_batch(exps, policy_ratio_clip_eps=0.2, optimize_iterations_per_step=1, max_grad_norm=1.0)
    moved = [name for name, b in before.items() if not torch.equal(b, lora.by_name[name].b)]
    assert "visual.merger.linear_fc2" in moved and len(moved) >= len(vis) // 2
    # the features now follow the trained factors (no stale cache)
    feats_after, _ = api.adapter._image_features([gens[0].metadata["_media_rows"][0]])
    api.adapter.model.lora.params.zero_()
    feats_zero, _ = api.adapter._image_features([gens[0].metadata["_media_rows"][0]])
    assert (feats_after - feats_zero).abs().max() > 0
    from safetensors.torch import load_file

    from graspo_b200.models.lora_io import export_peft_adapter

    api.adapter.save_checkpoint(tmp_path / "ckpt" / "final")
    out = export_peft_adapter(tmp_path / "ckpt" / "final", tmp_path / "peft")
    keys = load_file(str(out / "adapter_model.safetensors")).keys()
    assert any("model.visual.merger.linear_fc2.lora_B" in k for k in keys)
    assert any("model.visual.blocks.1.attn.qkv.lora_A" in k for k in keys)
