"""Runtime boundary between the GRASPO loop and a model adapter.

The trainer talks only to this protocol (reference: runtime.py:42-268):
``generate_groups`` / ``generate_sample_groups`` produce ``NativeGeneration``
records, ``sequence_log_probs`` scores sequences, ``train_batch`` /
``train_batch_sft`` run optimizer steps, ``save_checkpoint`` /
``load_checkpoint`` persist per-rank state.  The adapter class is loaded from
``graspoflow.adapter`` ("module:Class"), or from the ``GRASPO_ADAPTER``
environment variable when set (the reference documents that variable but
never reads it).
"""

from __future__ import annotations

import importlib
import os
import sys
from dataclasses import dataclass
from pathlib import Path
from typing import Any, Protocol

from graspo_b200.core.buffer import Experience
from graspo_b200.core.completion import ParsedCompletion
from graspo_b200.core.schema import GraspoConfig, Sample

FORBIDDEN_RUNTIME_MODULES = (
    "megatron",
    "nemo_rl",
    "vllm",
    "ray",
    "deepspeed",
    "accelerate",
    "transformer_engine",
    "apex",
)


@dataclass(slots=True)
class NativeGeneration:
    sequences: Any
    attention_mask: Any
    action_mask: Any
    completions: list[str]
    prompt_len: int = 0
    metadata: dict[str, Any] | None = None


class GraspoFlowRuntimeProtocol(Protocol):
    def validate(self) -> None: ...
    def setup(self) -> None: ...
    def generate_groups(self, *, message_batches, tool_batches=None, rollout_group_size: int,
                        max_new_tokens: int, temperature: float = 1.0, top_p: float = 1.0,
                        max_prompt_length: int | None = None,
                        chat_template_kwargs: dict[str, Any] | None = None) -> list[NativeGeneration]: ...
    def generate_sample_groups(self, *, samples: list[Any], rollout_group_size: int, max_new_tokens: int,
                               temperature: float = 1.0, top_p: float = 1.0,
                               max_prompt_length: int | None = None,
                               chat_template_kwargs: dict[str, Any] | None = None) -> list[NativeGeneration]: ...
    def parse_completion(self, completion: str, sample: Sample) -> ParsedCompletion: ...
    def sequence_log_probs(self, sequences: Any, attention_mask: Any, metadata: Any | None = None) -> Any: ...
    def train_batch(self, experiences: list[Experience], *, policy_ratio_clip_eps: float,
                    optimize_iterations_per_step: int, max_grad_norm: float) -> dict[str, Any]: ...
    def train_batch_sft(self, sft_batches: list[dict[str, Any]], *, optimize_iterations_per_step: int,
                        max_grad_norm: float) -> dict[str, Any]: ...
    def save_checkpoint(self, path: str | Path, *, trainer_state: dict[str, Any] | None = None) -> None: ...
    def load_checkpoint(self, path: str | Path) -> dict[str, Any] | None: ...
    def close(self) -> None: ...
    def is_primary(self) -> bool: ...


def validate_graspoflow_runtime_config(config: GraspoConfig, flow: Any | None = None) -> None:
    flow = flow or config.graspoflow
    if int(flow.tp_size) < 1:
        raise ValueError("tp_size must be >= 1")
    if int(flow.pp_size) < 1:
        raise ValueError("pp_size must be >= 1")
    if int(flow.dp_size) < 0:
        raise ValueError("dp_size must be >= 0")
    if int(flow.pp_micro_batch_size) < 1:
        raise ValueError("graspoflow.pp_micro_batch_size must be >= 1")
    if int(flow.forward_batch_size) < 1:
        raise ValueError(f"graspoflow.forward_batch_size must be >= 1, got {flow.forward_batch_size}")
    schedule = str(flow.pp_schedule or "simple")
    if schedule not in {"simple", "one_f_one_b", "gpipe", "1f1b"}:
        raise ValueError("graspoflow.pp_schedule must be simple, gpipe or one_f_one_b")
    if schedule in ("one_f_one_b", "1f1b") and int(flow.pp_size) <= 1:
        raise ValueError("one_f_one_b pp_schedule requires pp_size>1")
    if int(flow.pp_max_inflight_microbatches) < 0:
        raise ValueError("graspoflow.pp_max_inflight_microbatches must be >= 0")
    if config.training.resume_from_checkpoint and config.lora.adapter_path:
        raise ValueError("training.resume_from_checkpoint and lora.adapter_path cannot both be set")
    if int(flow.kv_page_size) % 4 or int(flow.kv_page_size) <= 0:
        raise ValueError("graspoflow.kv_page_size must be a positive multiple of 4")


def assert_forbidden_runtime_modules_not_imported() -> None:
    imported = [name for name in FORBIDDEN_RUNTIME_MODULES if name in sys.modules]
    if imported:
        raise RuntimeError("graspoflow runtime must not import forbidden frameworks: " + ", ".join(imported))


class GraspoFlowRuntime:
    """Validates the config, instantiates the adapter and delegates to it."""

    def __init__(self, config: GraspoConfig) -> None:
        self.config = config
        self.graspoflow_config = config.graspoflow
        self._adapter: Any | None = None

    @classmethod
    def from_config(cls, config: GraspoConfig) -> GraspoFlowRuntime:
        return cls(config)

    def validate(self) -> None:
        validate_graspoflow_runtime_config(self.config, self.graspoflow_config)
        assert_forbidden_runtime_modules_not_imported()

    def adapter_path(self) -> str:
        return os.environ.get("GRASPO_ADAPTER") or self.graspoflow_config.adapter

    def setup(self):
        self.validate()
        module_name, sep, class_name = self.adapter_path().partition(":")
        if not sep:
            raise ValueError("graspoflow.adapter must use the 'module:Class' format")
        adapter_cls = getattr(importlib.import_module(module_name), class_name)
        self._adapter = adapter_cls(self.config)
        self._adapter.setup()
        return self._adapter

    @property
    def adapter(self):
        if self._adapter is None:
            raise RuntimeError("GraspoFlowRuntime.setup() has not been called")
        return self._adapter

    def __getattr__(self, name: str):
        # delegate everything else (generate_groups, train_batch, rank, ...)
        if name.startswith("_"):
            raise AttributeError(name)
        return getattr(self.adapter, name)

    def is_primary(self) -> bool:
        return self._adapter.is_primary() if self._adapter is not None else True

    def close(self) -> None:
        if self._adapter is not None:
            self._adapter.close()
