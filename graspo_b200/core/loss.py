"""Reference (plain PyTorch, any device) formulations of the training losses.

These are the numerical oracles for the fused sm_100a kernels in
``graspo_b200.ops``:

* GRPO / PPO-clip: ``ratio = exp(lp - old)``,
  ``loss_t = -min(ratio*A, clip(ratio, 1-eps, 1+eps)*A)``, masked mean over the
  tokens of each sequence, then mean over sequences; no KL or entropy term
  (reference: src/graspo/core/graspo_loss.py:10-63).
* SFT: shifted token cross-entropy with ``ignore_index=-100``
  (reference: src/graspo/core/sft_loss.py:12-34).
"""

from __future__ import annotations

import torch
from torch import nn
from torch.nn import functional as F


def masked_mean(tensor: torch.Tensor, mask: torch.Tensor | None, dim: int | None = None) -> torch.Tensor:
    if mask is None:
        return tensor.mean(dim=dim)
    mask = mask.to(tensor.dtype)
    return (tensor * mask).sum(dim=dim) / mask.sum(dim=dim).clamp_min(1)


def grpo_token_loss(
    log_probs: torch.Tensor,
    old_log_probs: torch.Tensor,
    advantages: torch.Tensor,
    clip_eps: float,
) -> torch.Tensor:
    ratio = torch.exp(log_probs - old_log_probs)
    unclipped = ratio * advantages
    clipped = ratio.clamp(1.0 - clip_eps, 1.0 + clip_eps) * advantages
    return -torch.minimum(unclipped, clipped)


class GRASPOLoss(nn.Module):
    def __init__(self, policy_ratio_clip_eps: float = 0.2) -> None:
        super().__init__()
        self.policy_ratio_clip_eps = float(policy_ratio_clip_eps)

    def forward(
        self,
        log_probs: torch.Tensor,
        old_log_probs: torch.Tensor,
        advantages: torch.Tensor,
        action_mask: torch.Tensor,
    ) -> torch.Tensor:
        per_token = grpo_token_loss(log_probs, old_log_probs, advantages, self.policy_ratio_clip_eps)
        return masked_mean(per_token, action_mask, dim=-1).mean()


def sequence_log_probs_from_logits(logits: torch.Tensor, output_ids: torch.Tensor) -> torch.Tensor:
    return torch.log_softmax(logits.float(), dim=-1).gather(-1, output_ids.unsqueeze(-1)).squeeze(-1)


def sft_cross_entropy_loss(
    logits: torch.Tensor, labels: torch.Tensor, *, ignore_index: int = -100
) -> torch.Tensor:
    shifted = logits[:, :-1].reshape(-1, logits.shape[-1])
    targets = labels[:, 1:].reshape(-1)
    return F.cross_entropy(shifted, targets, ignore_index=ignore_index)
