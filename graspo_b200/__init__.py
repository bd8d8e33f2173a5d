"""graspo_b200: a Blackwell-native (sm_100a) GRASPO trainer.

GRASPO fine-tunes LoRA adapters on a frozen Qwen-family decoder with
group-relative policy optimisation over a rule-based structured reward.  The
public surface mirrors the reference trainer (YAML schema, JSONL data format,
``graspo launch|export|validate-reward`` CLI, per-rank LoRA checkpoints with
PEFT export); the execution layer is PyTorch plus hand-written sm_100a CUDA
kernels and NCCL/NVLink collectives.
"""

__version__ = "0.1.0"

from graspo_b200.core import (  # noqa: F401
    ClassifyResult,
    Experience,
    GraspoConfig,
    GraspoReward,
    GRASPOLoss,
    GroupDecision,
    ReplayBuffer,
    RewardConfig,
    Sample,
    classify_group,
    dict_compare_score,
    group_advantages,
    load_jsonl,
    resolve_lora_target_modules,
    setup_logging,
)
