"""Synthetic, seeded inputs: random-init HF checkpoints and JSON-extraction data.

* ``write_qwen3_checkpoint`` writes a Hugging Face style directory
  (``config.json`` with ``model_type: qwen3``, sharded ``*.safetensors`` with an
  index, an offline tokenizer) whose weights are N(0, 0.02) from a seed and
  whose norm weights are ones.  Both this framework and the reference load
  it, so the two run identical models.
* ``synthetic_json_records`` produces the seeded JSON-extraction prompts of
  the benchmark configs: a system message and a user message holding 2-4
  random snake_case keys, each with a random lowercase 3-8 character value or
  an 11-digit number; the target is the dict of those pairs.
"""

from __future__ import annotations

import json
import random
import string
from pathlib import Path

import torch

QWEN3_8B = dict(
    vocab_size=151936, hidden_size=4096, intermediate_size=12288, num_hidden_layers=36,
    num_attention_heads=32, num_key_value_heads=8, head_dim=128,
)
DENSE_32B = dict(
    vocab_size=151936, hidden_size=5120, intermediate_size=25600, num_hidden_layers=64,
    num_attention_heads=64, num_key_value_heads=8, head_dim=128,
)
TINY = dict(
    vocab_size=2048, hidden_size=128, intermediate_size=384, num_hidden_layers=2,
    num_attention_heads=4, num_key_value_heads=2, head_dim=32,
)


def qwen3_config_dict(dims: dict, *, rms_norm_eps: float = 1e-6, rope_theta: float = 1e6) -> dict:
    return {
        "architectures": ["Qwen3ForCausalLM"],
        "model_type": "qwen3",
        "hidden_act": "silu",
        "rms_norm_eps": rms_norm_eps,
        "rope_theta": rope_theta,
        "max_position_embeddings": 40960,
        "tie_word_embeddings": False,
        "attention_bias": False,
        "torch_dtype": "bfloat16",
        "bos_token_id": None,
        "eos_token_id": 151643 if dims["vocab_size"] >= 151654 else dims["vocab_size"] - 4,
        **dims,
    }


def _qwen3_tensor_specs(dims: dict) -> list[tuple[str, tuple[int, ...], str]]:
    H, I, V = dims["hidden_size"], dims["intermediate_size"], dims["vocab_size"]
    q = dims["num_attention_heads"] * dims["head_dim"]
    kv = dims["num_key_value_heads"] * dims["head_dim"]
    D = dims["head_dim"]
    specs = [("model.embed_tokens.weight", (V, H), "normal")]
    for i in range(dims["num_hidden_layers"]):
        p = f"model.layers.{i}"
        specs += [
            (f"{p}.input_layernorm.weight", (H,), "ones"),
            (f"{p}.post_attention_layernorm.weight", (H,), "ones"),
            (f"{p}.self_attn.q_proj.weight", (q, H), "normal"),
            (f"{p}.self_attn.k_proj.weight", (kv, H), "normal"),
            (f"{p}.self_attn.v_proj.weight", (kv, H), "normal"),
            (f"{p}.self_attn.o_proj.weight", (H, q), "normal"),
            (f"{p}.self_attn.q_norm.weight", (D,), "ones"),
            (f"{p}.self_attn.k_norm.weight", (D,), "ones"),
            (f"{p}.mlp.gate_proj.weight", (I, H), "normal"),
            (f"{p}.mlp.up_proj.weight", (I, H), "normal"),
            (f"{p}.mlp.down_proj.weight", (H, I), "normal"),
        ]
    specs += [("model.norm.weight", (H,), "ones"), ("lm_head.weight", (V, H), "normal")]
    return specs


QWEN35_TINY = dict(
    vocab_size=512, hidden_size=128, intermediate_size=256, num_hidden_layers=4,
    num_attention_heads=4, num_key_value_heads=2, head_dim=32,
    linear_num_key_heads=2, linear_num_value_heads=4, linear_key_head_dim=32, linear_value_head_dim=32,
    linear_conv_kernel_dim=4, full_attention_interval=4, partial_rotary_factor=0.25,
)

# Qwen3.5-9B-shaped hybrid decoder (the dimensions transformers' Qwen3_5TextConfig
# defaults to): three gated-DeltaNet layers per gated-attention layer
QWEN35_9B = dict(
    vocab_size=248320, hidden_size=4096, intermediate_size=12288, num_hidden_layers=32,
    num_attention_heads=16, num_key_value_heads=4, head_dim=256,
    linear_num_key_heads=16, linear_num_value_heads=32, linear_key_head_dim=128, linear_value_head_dim=128,
    linear_conv_kernel_dim=4, full_attention_interval=4, partial_rotary_factor=0.25,
)


def _qwen35_tensor_specs(dims: dict) -> list[tuple[str, tuple[int, ...], str]]:
    H, I, V = dims["hidden_size"], dims["intermediate_size"], dims["vocab_size"]
    D = dims["head_dim"]
    nq, nkv = dims["num_attention_heads"], dims["num_key_value_heads"]
    kd = dims["linear_num_key_heads"] * dims["linear_key_head_dim"]
    vd = dims["linear_num_value_heads"] * dims["linear_value_head_dim"]
    hv = dims["linear_num_value_heads"]
    pre = "model.language_model"
    specs = [(f"{pre}.embed_tokens.weight", (V, H), "normal")]
    for i, kind in enumerate(qwen35_layer_types(dims)):
        p = f"{pre}.layers.{i}"
        specs += [(f"{p}.input_layernorm.weight", (H,), "zeros"), (f"{p}.post_attention_layernorm.weight", (H,), "zeros")]
        if kind == "full_attention":
            specs += [(f"{p}.self_attn.q_proj.weight", (2 * nq * D, H), "normal"),
                      (f"{p}.self_attn.k_proj.weight", (nkv * D, H), "normal"),
                      (f"{p}.self_attn.v_proj.weight", (nkv * D, H), "normal"),
                      (f"{p}.self_attn.o_proj.weight", (H, nq * D), "normal"),
                      (f"{p}.self_attn.q_norm.weight", (D,), "zeros"), (f"{p}.self_attn.k_norm.weight", (D,), "zeros")]
        else:
            specs += [(f"{p}.linear_attn.in_proj_qkv.weight", (2 * kd + vd, H), "normal"),
                      (f"{p}.linear_attn.in_proj_z.weight", (vd, H), "normal"),
                      (f"{p}.linear_attn.in_proj_b.weight", (hv, H), "normal"),
                      (f"{p}.linear_attn.in_proj_a.weight", (hv, H), "normal"),
                      (f"{p}.linear_attn.conv1d.weight", (2 * kd + vd, 1, dims["linear_conv_kernel_dim"]), "conv"),
                      (f"{p}.linear_attn.dt_bias", (hv,), "ones"),
                      (f"{p}.linear_attn.A_log", (hv,), "alog"),
                      (f"{p}.linear_attn.norm.weight", (dims["linear_value_head_dim"],), "ones"),
                      (f"{p}.linear_attn.out_proj.weight", (H, vd), "normal")]
        specs += [(f"{p}.mlp.gate_proj.weight", (I, H), "normal"), (f"{p}.mlp.up_proj.weight", (I, H), "normal"),
                  (f"{p}.mlp.down_proj.weight", (H, I), "normal")]
    specs += [(f"{pre}.norm.weight", (H,), "zeros"), ("lm_head.weight", (V, H), "normal")]
    return specs


def qwen35_layer_types(dims: dict) -> list[str]:
    every = int(dims.get("full_attention_interval", 4))
    return ["full_attention" if (i + 1) % every == 0 else "linear_attention" for i in range(dims["num_hidden_layers"])]


def write_qwen35_checkpoint(output_dir: str | Path, dims: dict, *, seed: int = 0, std: float = 0.02,
                            dtype: torch.dtype = torch.bfloat16, with_tokenizer: bool = True) -> Path:
    """Random-init Qwen3.5 hybrid (``model_type: qwen3_5`` with a ``qwen3_5_text`` text config)."""
    from safetensors.torch import save_file

    out = Path(output_dir)
    if (out / ".complete").exists():
        return out
    out.mkdir(parents=True, exist_ok=True)
    gen = torch.Generator().manual_seed(seed)
    tensors = {}
    for name, shape, kind in _qwen35_tensor_specs(dims):
        if kind == "normal":
            t = torch.randn(shape, generator=gen) * std
        elif kind == "zeros":
            t = torch.zeros(shape)
        elif kind == "ones":
            t = torch.ones(shape)
        elif kind == "conv":
            t = torch.randn(shape, generator=gen) * 0.3
        else:  # A_log: decays between exp(-1) and exp(-16) per step scale
            t = torch.log(torch.rand(shape, generator=gen) * 15 + 1)
        tensors[name] = t.to(dtype).contiguous()
    save_file(tensors, str(out / "model.safetensors"), metadata={"format": "pt"})
    (out / "model.safetensors.index.json").write_text(json.dumps(
        {"metadata": {}, "weight_map": {k: "model.safetensors" for k in tensors}}, indent=2))
    text = {
        "model_type": "qwen3_5_text", "hidden_act": "silu", "rms_norm_eps": 1e-6,
        "layer_types": qwen35_layer_types(dims), "tie_word_embeddings": False,
        "rope_parameters": {"rope_theta": 1e7, "partial_rotary_factor": dims.get("partial_rotary_factor", 0.25)},
        **{k: v for k, v in dims.items() if k not in ("full_attention_interval", "partial_rotary_factor")},
    }
    eos = dims["vocab_size"] - 4
    config = {"model_type": "qwen3_5", "architectures": ["Qwen3_5ForConditionalGeneration"], "text_config": text,
              "tie_word_embeddings": False, "eos_token_id": eos}
    (out / "config.json").write_text(json.dumps(config, indent=2))
    (out / "generation_config.json").write_text(json.dumps({"eos_token_id": eos}))
    if with_tokenizer:
        from graspo_b200.utils.tokenizer import build_tokenizer

        build_tokenizer(out, dims["vocab_size"])
    (out / ".complete").write_text("ok")
    return out


def write_qwen3_checkpoint(
    output_dir: str | Path,
    dims: dict,
    *,
    seed: int = 0,
    dtype: torch.dtype = torch.bfloat16,
    std: float = 0.02,
    shard_bytes: int = 4 << 30,
    device: str | None = None,
    with_tokenizer: bool = True,
) -> Path:
    """Write a random-init Qwen3 checkpoint (skipped if a complete one exists)."""
    from safetensors.torch import save_file

    out = Path(output_dir)
    marker = out / ".complete"
    config = qwen3_config_dict(dims)
    if marker.exists() and json.loads((out / "config.json").read_text())["hidden_size"] == dims["hidden_size"]:
        return out
    out.mkdir(parents=True, exist_ok=True)
    dev = device or ("cuda" if torch.cuda.is_available() else "cpu")
    gen = torch.Generator(device=dev).manual_seed(seed)
    weight_map: dict[str, str] = {}
    shard: dict[str, torch.Tensor] = {}
    size = 0
    index = 0

    def flush() -> None:
        nonlocal shard, size, index
        if not shard:
            return
        index += 1
        name = f"model-{index:05d}.safetensors"
        save_file(shard, str(out / name), metadata={"format": "pt"})
        for key in shard:
            weight_map[key] = name
        shard, size = {}, 0

    for name, shape, kind in _qwen3_tensor_specs(dims):
        if kind == "ones":
            t = torch.ones(shape, dtype=dtype)
        else:
            t = (torch.randn(shape, generator=gen, device=dev, dtype=torch.float32) * std).to(dtype).cpu()
        nbytes = t.numel() * t.element_size()
        if size and size + nbytes > shard_bytes:
            flush()
        shard[name] = t.contiguous()
        size += nbytes
    flush()
    total = sum((out / f).stat().st_size for f in set(weight_map.values()))
    (out / "model.safetensors.index.json").write_text(
        json.dumps({"metadata": {"total_size": total}, "weight_map": weight_map}, indent=2)
    )
    (out / "config.json").write_text(json.dumps(config, indent=2))
    (out / "generation_config.json").write_text(json.dumps({"eos_token_id": config["eos_token_id"]}))
    if with_tokenizer:
        from graspo_b200.utils.tokenizer import build_tokenizer

        build_tokenizer(out, dims["vocab_size"])
    marker.write_text("ok")
    return out


def _snake_key(rng: random.Random) -> str:
    words = ["".join(rng.choice(string.ascii_lowercase) for _ in range(rng.randint(3, 7))) for _ in range(rng.randint(1, 3))]
    return "_".join(words)


def synthetic_json_records(
    count: int, *, seed: int = 0, pad_words_to: int | None = None
) -> list[dict]:
    """Seeded JSON-extraction records in the JSONL schema.

    ``pad_words_to`` appends filler words to the user message so prompts reach
    a target length (used by the 1024-token benchmark prompts).
    """
    rng = random.Random(seed)
    records = []
    for idx in range(count):
        fields: dict[str, object] = {}
        for _ in range(rng.randint(2, 4)):
            key = _snake_key(rng)
            if rng.random() < 0.5:
                fields[key] = "".join(rng.choice(string.ascii_lowercase) for _ in range(rng.randint(3, 8)))
            else:
                fields[key] = rng.randint(10**10, 10**11 - 1)
        facts = "; ".join(f"{k.replace('_', ' ')} is {v}" for k, v in fields.items())
        text = f"Extract the following fields as JSON with keys {list(fields)}: {facts}."
        if pad_words_to:
            filler = []
            while len(filler) < pad_words_to:
                filler.append("".join(rng.choice(string.ascii_lowercase) for _ in range(rng.randint(2, 9))))
            text += " Context: " + " ".join(filler)
        records.append(
            {
                "id": f"synthetic-{idx}",
                "messages": [
                    {"role": "system", "content": "You extract structured data. Answer with a ```json fenced object."},
                    {"role": "user", "content": text},
                ],
                "targets": [{"id": f"t{idx}", "output": {"content": fields}}],
            }
        )
    return records


VIT_27L = dict(depth=27, hidden_size=1152, intermediate_size=4304, num_heads=16, in_channels=3, patch_size=16,
               spatial_merge_size=2, temporal_patch_size=2, num_position_embeddings=2304)
VIT_TINY = dict(depth=2, hidden_size=64, intermediate_size=128, num_heads=4, in_channels=3, patch_size=16,
                spatial_merge_size=2, temporal_patch_size=2, num_position_embeddings=64)


def add_vision_tower(model_dir: str | Path, vdims: dict, *, seed: int = 0, std: float = 0.02,
                     dtype: torch.dtype = torch.bfloat16) -> Path:
    """Add a random-init vision tower (``model.visual.*``) to a synthetic Qwen3 or Qwen3.5 checkpoint."""
    from safetensors.torch import save_file

    out = Path(model_dir)
    config = json.loads((out / "config.json").read_text())
    if config.get("vision_config"):
        return out
    Hd, I = vdims["hidden_size"], vdims["intermediate_size"]
    pdim = vdims["in_channels"] * vdims["temporal_patch_size"] * vdims["patch_size"] ** 2
    merged = Hd * vdims["spatial_merge_size"] ** 2
    text = config.get("text_config") or config
    out_h = text["hidden_size"]
    gen = torch.Generator().manual_seed(seed)
    specs = [("patch_embed.proj.weight", (Hd, vdims["in_channels"], vdims["temporal_patch_size"], vdims["patch_size"],
                                          vdims["patch_size"]), "n"),
             ("patch_embed.proj.bias", (Hd,), "z"), ("pos_embed.weight", (vdims["num_position_embeddings"], Hd), "n")]
    for i in range(vdims["depth"]):
        b = f"blocks.{i}"
        specs += [(f"{b}.norm1.weight", (Hd,), "o"), (f"{b}.norm1.bias", (Hd,), "z"), (f"{b}.norm2.weight", (Hd,), "o"),
                  (f"{b}.norm2.bias", (Hd,), "z"), (f"{b}.attn.qkv.weight", (3 * Hd, Hd), "n"),
                  (f"{b}.attn.qkv.bias", (3 * Hd,), "z"), (f"{b}.attn.proj.weight", (Hd, Hd), "n"),
                  (f"{b}.attn.proj.bias", (Hd,), "z"), (f"{b}.mlp.linear_fc1.weight", (I, Hd), "n"),
                  (f"{b}.mlp.linear_fc1.bias", (I,), "z"), (f"{b}.mlp.linear_fc2.weight", (Hd, I), "n"),
                  (f"{b}.mlp.linear_fc2.bias", (Hd,), "z")]
    specs += [("merger.norm.weight", (Hd,), "o"), ("merger.norm.bias", (Hd,), "z"),
              ("merger.linear_fc1.weight", (merged, merged), "n"), ("merger.linear_fc1.bias", (merged,), "z"),
              ("merger.linear_fc2.weight", (out_h, merged), "n"), ("merger.linear_fc2.bias", (out_h,), "z")]
    tensors = {}
    for name, shape, kind in specs:
        t = torch.randn(shape, generator=gen) * std if kind == "n" else (torch.ones(shape) if kind == "o"
                                                                         else torch.zeros(shape))
        tensors[f"model.visual.{name}"] = t.to(dtype).contiguous()
    save_file(tensors, str(out / "model-vision.safetensors"), metadata={"format": "pt"})
    index = json.loads((out / "model.safetensors.index.json").read_text())
    index["weight_map"].update({k: "model-vision.safetensors" for k in tensors})
    (out / "model.safetensors.index.json").write_text(json.dumps(index, indent=2))
    config["vision_config"] = {**vdims, "out_hidden_size": out_h}
    if config.get("image_token_id") is None:
        from graspo_b200.utils.tokenizer import special_token_ids

        config["image_token_id"] = special_token_ids(text["vocab_size"])["<|vision_pad|>"]
    (out / "config.json").write_text(json.dumps(config, indent=2))
    return out


def synthetic_image_records(count: int, image_dir: str | Path, *, seed: int = 0, size: int = 448,
                            text_words: int = 40) -> list[dict]:
    """Seeded multimodal JSON-extraction records: one uniform-random uint8 RGB
    image (PNG) plus a text instruction per record."""
    import numpy as np
    from PIL import Image

    image_dir = Path(image_dir)
    image_dir.mkdir(parents=True, exist_ok=True)
    base = synthetic_json_records(count, seed=seed, pad_words_to=text_words)
    rs = np.random.RandomState(seed)
    for i, rec in enumerate(base):
        path = image_dir / f"img_{seed}_{i}.png"
        if not path.exists():
            Image.fromarray(rs.randint(0, 256, (size, size, 3), dtype=np.uint8)).save(path)
        text = rec["messages"][1]["content"]
        rec["messages"][1]["content"] = [{"type": "image", "image": str(path)}, {"type": "text", "text": text}]
    return base


def write_jsonl_records(records: list[dict], path: str | Path) -> Path:
    out = Path(path)
    out.parent.mkdir(parents=True, exist_ok=True)
    with out.open("w", encoding="utf-8") as handle:
        for rec in records:
            handle.write(json.dumps(rec, ensure_ascii=False) + "\n")
    return out
