"""Pure-CPU core: config, data, reward, decisions, losses, replay buffer.

Nothing in this package touches a GPU, a process group or the filesystem
beyond reading the files it is asked to read.
"""

from graspo_b200.core.buffer import Experience, ReplayBuffer
from graspo_b200.core.compare import CompareResult, dict_compare_score
from graspo_b200.core.completion import ParsedCompletion, raw_parsed_completion
from graspo_b200.core.data import build_sft_target_text, load_jsonl, sample_from_record, write_jsonl
from graspo_b200.core.decisions import (
    GroupDecision,
    GroupSampleDecision,
    classify_group,
    group_advantages,
    has_reward_variance,
    lower_median,
    replay_ready,
)
from graspo_b200.core.logging import setup_logging
from graspo_b200.core.lora_targets import LORA_TARGET_PRESETS, resolve_lora_target_modules
from graspo_b200.core.loss import GRASPOLoss, masked_mean, sft_cross_entropy_loss
from graspo_b200.core.reward import GraspoReward, RewardConfig, RewardResult
from graspo_b200.core.schema import GraspoConfig, Sample
from graspo_b200.core.tool_parser import parse_qwen_tool_completion

ClassifyResult = GroupSampleDecision

__all__ = [
    "ClassifyResult",
    "CompareResult",
    "Experience",
    "GRASPOLoss",
    "GraspoConfig",
    "GraspoReward",
    "GroupDecision",
    "GroupSampleDecision",
    "LORA_TARGET_PRESETS",
    "ParsedCompletion",
    "ReplayBuffer",
    "RewardConfig",
    "RewardResult",
    "Sample",
    "build_sft_target_text",
    "classify_group",
    "dict_compare_score",
    "group_advantages",
    "has_reward_variance",
    "load_jsonl",
    "lower_median",
    "masked_mean",
    "parse_qwen_tool_completion",
    "raw_parsed_completion",
    "replay_ready",
    "resolve_lora_target_modules",
    "sample_from_record",
    "setup_logging",
    "sft_cross_entropy_loss",
    "write_jsonl",
]
