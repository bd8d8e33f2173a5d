"""Single-YAML configuration for a GRASPO run.

Every section is a strict pydantic model (``extra="forbid"``): a misspelt or
unknown key is a load-time error, never a silent default.  The section and key
names, their defaults and the ``output_dir``/``run_name`` auto-naming follow the
reference schema (src/graspo/core/schema.py:14-200) so existing YAML files load
unchanged.  Keys that only this framework understands live under
``graspoflow`` (``dp_size``, ``kernel_backend``, ``benchmark_ignore_eos``,
``advantage_eps``, ``rollout_engine_batch``...) and are documented where they are
declared.
"""

from __future__ import annotations

import datetime
import json
import logging
import warnings
from pathlib import Path
from typing import Any, Literal

from pydantic import BaseModel, ConfigDict, field_validator

from graspo_b200.core.reward import RewardConfig

_STRICT = ConfigDict(extra="forbid")


class LoRAConfig(BaseModel):
    """Adapter hyper-parameters (rank, scale, dropout) and target selection."""

    model_config = _STRICT

    r: int = 16
    alpha: int = 32
    dropout: float = 0.1
    adapter_path: str | None = None
    target_preset: str = "language_safe"
    target_modules: list[str] | None = None
    bias: str = "none"
    task_type: str = "CAUSAL_LM"


class ModelConfig(BaseModel):
    """Where the frozen base model lives and how it is materialised.

    ``trust_remote_code`` and ``attn_implementation`` configure Hugging Face
    model classes in the reference; here the weights are read from the
    safetensors files by this framework's own loader and attention always
    runs on its own kernels, so both keys are accepted (reference YAMLs load
    unchanged) and have no effect.
    """

    model_config = _STRICT

    model_path: str = ""
    trust_remote_code: bool = True
    torch_dtype: str = "bfloat16"
    attn_implementation: str | None = None
    gradient_checkpointing: bool = True
    chat_template_kwargs: dict[str, Any] = {}


class LRSchedulerConfig(BaseModel):
    """Per-optimizer-step learning-rate schedule (constant, cosine or linear)."""

    model_config = _STRICT

    type: str = "constant"
    warmup_steps: int = 0
    min_lr_ratio: float = 0.0


class TrainingConfig(BaseModel):
    """Loop length, rollout/replay sizes, optimizer and sampling knobs."""

    model_config = _STRICT

    output_dir: str = ""
    run_name: str = ""
    seed: int = 42
    max_epochs: int = 100
    max_steps: int = -1
    rollout_group_size: int = 8
    optimize_prompt_batch_size: int = 8
    optimize_iterations_per_step: int = 3
    rollout_max_retries: int = 5
    learning_rate: float = 5e-6
    weight_decay: float = 0.01
    max_grad_norm: float = 1.0
    policy_ratio_clip_eps: float = 0.2
    max_new_tokens: int = 2048
    temperature: float = 1.0
    top_p: float = 1.0
    save_steps: int = -1
    save_checkpoint_every_epoch: bool = True
    perfect_skip_reward_threshold: float = 1.0
    reject_unparseable_groups: bool = True
    resume_from_checkpoint: str | None = None
    lr_scheduler: LRSchedulerConfig = LRSchedulerConfig()

    @property
    def replay_buffer_optimize_threshold(self) -> int:
        """Completions that must be buffered before an optimize step (B x G)."""
        return int(self.optimize_prompt_batch_size) * int(self.rollout_group_size)


class DataConfig(BaseModel):
    model_config = _STRICT

    train_path: str = ""
    max_prompt_length: int = 2048


class GraspoFlowConfig(BaseModel):
    """Parallel layout, rollout engine and logging switches.

    Keys shared with the reference keep its meaning.  Added keys:

    * ``dp_size`` – data-parallel replicas; ``world = tp * pp * dp``.  ``0`` means
      "whatever is left of the world after tp*pp" (the reference has no DP and
      requires ``world == tp * pp``; with ``dp_size=0`` such a world gives dp=1).
    * ``sequence_parallel`` – Megatron sequence parallelism inside the TP group
      (accepted here; the reference rejects ``true``).
    * ``kernel_backend`` – ``"fused"`` runs the sm_100a kernels, ``"eager"`` the
      plain-PyTorch oracle of the same model (used by tests and for comparison).
    * ``benchmark_ignore_eos`` – generate exactly ``max_new_tokens`` per
      completion (fixed work for throughput measurements).
    * ``advantage_eps`` – epsilon of the group-normalised advantage
      ``(r - mean) / (std + eps)``; the reference hard-codes 1e-8.
    * ``rollout_engine_batch`` – maximum rows decoded together by the paged-KV
      engine (0 = all rows of the prompt queue at once).
    * ``pg_timeout_sec`` – process-group timeout so a dead peer ends collectives
      with an error instead of a hang.
    * ``decode_tp_allreduce`` – ``"fused"``: the decode loop's tensor-parallel
      all-reduces run inside the o_proj / down_proj GEMMs (tile push into the
      peers' memory over NVLink) and the following RMSNorm kernel; ``"nccl"``:
      an NCCL all-reduce after each of those GEMMs.
    * ``async_checkpoint`` – intermediate checkpoints (``step_N``, ``epoch_N``)
      are snapshotted to host memory and written by a background thread while
      training continues; the final checkpoint is always written in place.
    """

    model_config = _STRICT

    tp_size: int = 2
    pp_size: int = 1
    adapter: str = "graspo_b200.engine.adapter:Qwen3Adapter"
    placement_strategy: str = "auto"
    layer_ranges: list[list[int]] | None = None
    sequence_parallel: bool = False
    pp_micro_batch_size: int = 1
    forward_batch_size: int = 8
    use_kv_cache_for_rollout: bool = True
    empty_cache_after_rollout_split: bool = False
    empty_cache_before_train: bool = False
    raw_log_enabled: bool = True
    readable_log_enabled: bool = True
    synchronize_cuda_timing: bool = False
    pp_schedule: str = "simple"
    pp_max_inflight_microbatches: int = 0
    # ---- keys added by this framework ----
    dp_size: int = 0
    kernel_backend: Literal["fused", "eager"] = "fused"
    benchmark_ignore_eos: bool = False
    advantage_eps: float = 1e-8
    rollout_engine_batch: int = 0
    kv_page_size: int = 64
    cuda_graph_decode: bool = True
    pg_timeout_sec: float = 600.0
    decode_tp_allreduce: Literal["fused", "nccl"] = "fused"
    async_checkpoint: bool = False

    @field_validator("adapter")
    @classmethod
    def _map_reference_adapter(cls, value: str) -> str:
        # Reference YAMLs name the reference's own adapter classes; both map to
        # this framework's adapter, which dispatches on the checkpoint family.
        if value.startswith("graspo.backends.graspoflow.models."):
            return "graspo_b200.engine.adapter:Qwen3Adapter"
        return value


class ExportConfig(BaseModel):
    model_config = _STRICT

    checkpoint_path: str = ""
    export_format: str = "peft-adapter"
    export_output: str = ""
    final_formats: list[str] = []


class LaunchConfig(BaseModel):
    model_config = _STRICT

    gpus: list[int] | str | None = None
    nproc_per_node: int | None = None
    nnodes: int = 1
    node_rank: int = 0
    master_addr: str = "127.0.0.1"
    master_port: int = 29500
    python: str | None = None
    torchrun: str | None = None
    env: dict[str, str] = {}


class GraspoConfig(BaseModel):
    """Top-level run configuration; validated completely at load time."""

    model_config = _STRICT

    train_method: Literal["graspo", "sft"] = "graspo"
    backend: str = "graspoflow"
    graspoflow: GraspoFlowConfig = GraspoFlowConfig()
    model: ModelConfig = ModelConfig()
    data: DataConfig = DataConfig()
    lora: LoRAConfig = LoRAConfig()
    export: ExportConfig = ExportConfig()
    launch: LaunchConfig = LaunchConfig()
    reward: RewardConfig = RewardConfig()
    training: TrainingConfig = TrainingConfig()

    @classmethod
    def from_yaml(cls, path: str | Path) -> GraspoConfig:
        import yaml

        return cls.from_dict(yaml.safe_load(Path(path).read_text(encoding="utf-8")))

    @classmethod
    def from_dict(cls, data: dict[str, Any] | None) -> GraspoConfig:
        data = dict(data or {})
        unknown = set(data) - set(cls.model_fields) - {"backend_config"}
        if unknown:
            raise ValueError(f"unknown top-level config key(s): {sorted(unknown)}")
        training = dict(data.get("training") or {})
        output_dir = str(training.get("output_dir") or "").strip()
        run_name = str(training.get("run_name") or "").strip()
        if not output_dir:
            run_name = run_name or default_run_name()
            training["output_dir"] = str(Path("outputs") / run_name)
            training["run_name"] = run_name
        elif not run_name:
            training["run_name"] = Path(output_dir).name
        return cls(
            train_method=data.get("train_method", "graspo"),
            backend=data.get("backend", "graspoflow"),
            graspoflow=GraspoFlowConfig(**_graspoflow_section(data)),
            model=ModelConfig(**(data.get("model") or {})),
            data=DataConfig(**(data.get("data") or {})),
            lora=LoRAConfig(**(data.get("lora") or {})),
            export=ExportConfig(**(data.get("export") or {})),
            launch=LaunchConfig(**(data.get("launch") or {})),
            reward=RewardConfig(**(data.get("reward") or {})),
            training=TrainingConfig(**training),
        )


class Sample(BaseModel):
    """One validated JSONL record: prompt messages, targets, optional tools."""

    model_config = ConfigDict(extra="forbid", frozen=True)

    messages: list[dict[str, Any]]
    targets: list[dict[str, Any]]
    tools: list[dict[str, Any]] | None = None
    metadata: dict[str, Any] = {}
    media: list[dict[str, Any]] = []

    @property
    def expects_tool_calls(self) -> bool:
        """True when any target's output carries ``tool_calls``."""
        return any(
            isinstance(t, dict)
            and isinstance(t.get("output"), dict)
            and t["output"].get("tool_calls") is not None
            for t in self.targets
        )

    @property
    def prompt_preview(self) -> str:
        lines = []
        for message in self.messages:
            text = content_preview(message.get("content", ""))
            lines.append(f"{message.get('role', 'user')}: {text}")
        return "\n\n".join(line for line in lines if line)

    def to_json(self) -> str:
        return json.dumps(self.model_dump(), ensure_ascii=False)


_RUN_NAME: list[str] = []


def default_run_name() -> str:
    """``graspo_YYYYmmdd_HHMMSS``, fixed for the life of the process.

    Caching matters under torchrun: every worker resolves the same name as long
    as they share the launcher's environment variable ``GRASPO_RUN_NAME`` or
    start within the same second.
    """
    import os

    if not _RUN_NAME:
        env = os.environ.get("GRASPO_RUN_NAME")
        _RUN_NAME.append(env or datetime.datetime.now().strftime("graspo_%Y%m%d_%H%M%S"))
    return _RUN_NAME[0]


def _graspoflow_section(data: dict[str, Any]) -> dict[str, Any]:
    if data.get("graspoflow"):
        return dict(data["graspoflow"])
    legacy = data.get("backend_config")
    if isinstance(legacy, dict) and legacy.get("graspoflow"):
        msg = "backend_config.graspoflow is deprecated; move the section to top-level 'graspoflow'"
        warnings.warn(msg, FutureWarning, stacklevel=3)
        logging.getLogger("graspo.config").warning(msg)
        return dict(legacy["graspoflow"])
    return {}


def content_preview(content: Any) -> str:
    """Readable text for a message's content; media items become placeholders."""
    if isinstance(content, str):
        return content
    if not isinstance(content, list):
        return str(content or "")
    parts: list[str] = []
    for item in content:
        if isinstance(item, dict):
            kind = str(item.get("type") or "").lower()
            if kind == "text":
                parts.append(str(item.get("text") or ""))
            elif kind in ("image", "image_url"):
                parts.append("<image>")
            elif kind in ("video", "video_url"):
                parts.append("<video>")
            else:
                parts.append(f"<{kind or 'content'}>")
        else:
            parts.append(str(item))
    return "\n".join(p for p in parts if p)
