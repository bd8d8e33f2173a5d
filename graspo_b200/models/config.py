"""Decoder configuration read from a Hugging Face ``config.json``.

Supported families (reference: models/qwen3/model.py:99-117):

* ``qwen3`` -- dense Qwen3 (``model_type: qwen3``), weights under ``model.``;
* ``qwen3_5_text`` -- the Qwen3.5/3.6 hybrid (``model_type: qwen3_5`` with a
  ``text_config``), weights under ``model.language_model.``; an optional
  ``vision_config`` describes a vision tower.
"""

from __future__ import annotations

import json
from dataclasses import dataclass, field
from pathlib import Path
from typing import Any


@dataclass
class DecoderConfig:
    family: str
    key_prefix: str
    vocab_size: int
    hidden_size: int
    intermediate_size: int
    num_hidden_layers: int
    num_attention_heads: int
    num_key_value_heads: int
    head_dim: int
    rms_norm_eps: float = 1e-6
    rope_theta: float = 1_000_000.0
    tie_word_embeddings: bool = False
    max_position_embeddings: int = 40960
    layer_types: list[str] = field(default_factory=list)
    extra: dict[str, Any] = field(default_factory=dict)

    @property
    def q_size(self) -> int:
        return self.num_attention_heads * self.head_dim

    @property
    def kv_size(self) -> int:
        return self.num_key_value_heads * self.head_dim

    @property
    def has_vision(self) -> bool:
        return bool(self.extra.get("vision_config"))

    def layer_kind(self, idx: int) -> str:
        if self.layer_types:
            return self.layer_types[idx]
        return "full_attention"


def _from_values(values: dict[str, Any], family: str, key_prefix: str, extra: dict[str, Any]) -> DecoderConfig:
    heads = int(values["num_attention_heads"])
    hidden = int(values["hidden_size"])
    return DecoderConfig(
        family=family,
        key_prefix=key_prefix,
        vocab_size=int(values["vocab_size"]),
        hidden_size=hidden,
        intermediate_size=int(values["intermediate_size"]),
        num_hidden_layers=int(values["num_hidden_layers"]),
        num_attention_heads=heads,
        num_key_value_heads=int(values.get("num_key_value_heads", heads)),
        head_dim=int(values.get("head_dim") or hidden // heads),
        rms_norm_eps=float(values.get("rms_norm_eps", 1e-6)),
        rope_theta=float(values.get("rope_theta", (values.get("rope_parameters") or {}).get("rope_theta", 1e6))),
        tie_word_embeddings=bool(values.get("tie_word_embeddings", False)),
        max_position_embeddings=int(values.get("max_position_embeddings", 40960)),
        layer_types=list(values.get("layer_types") or []),
        extra=extra,
    )


def load_decoder_config(model_path: str | Path) -> DecoderConfig:
    raw = json.loads((Path(model_path) / "config.json").read_text(encoding="utf-8"))
    model_type = str(raw.get("model_type") or "")
    if model_type == "qwen3":
        extra = {}
        if raw.get("vision_config"):
            # a dense Qwen3 decoder with a vision tower (weights under model.visual.)
            extra = {"vision_config": dict(raw["vision_config"]), "image_token_id": raw.get("image_token_id")}
        return _from_values(raw, "qwen3", "model", extra)
    text = dict(raw.get("text_config") or {})
    if model_type == "qwen3_5" and text.get("model_type") == "qwen3_5_text":
        extra = {
            "vision_config": dict(raw.get("vision_config") or {}),
            "image_token_id": raw.get("image_token_id"),
            "video_token_id": raw.get("video_token_id"),
            "text_config": text,
        }
        return _from_values(text, "qwen3_5_text", "model.language_model", extra)
    raise ValueError(
        f"supported model families are qwen3 and qwen3_5 text; got model_type={model_type!r}"
    )


def lora_available_targets(cfg: DecoderConfig) -> tuple[str, ...]:
    """Canonical LoRA target names a model family exposes."""
    mlp = ("language.mlp.gate_proj", "language.mlp.up_proj", "language.mlp.down_proj")
    if cfg.family == "qwen3":
        attn = tuple(f"language.self_attn.{p}" for p in ("q_proj", "k_proj", "v_proj", "o_proj"))
        targets = attn + mlp
    else:
        targets = (
            tuple(f"language.full_attn.{p}" for p in ("q_proj", "k_proj", "v_proj", "o_proj"))
            + tuple(
                f"language.linear_attn.{p}" for p in ("q_proj", "k_proj", "v_proj", "in_proj_z", "out_proj")
            )
            + mlp
        )
    if cfg.has_vision:
        depth = int(cfg.extra["vision_config"].get("depth") or 0)
        targets += ("visual.merger.linear_fc1", "visual.merger.linear_fc2")
        targets += tuple(
            f"visual.blocks.{i}.{p}"
            for i in range(depth)
            for p in ("attn.qkv", "attn.proj", "mlp.linear_fc1", "mlp.linear_fc2")
        )
    return targets
