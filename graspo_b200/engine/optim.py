"""Flat-buffer AdamW with global gradient clipping and a per-step LR schedule.

All LoRA parameters of a rank live in one fp32 buffer, so one reduction
computes the gradient norm and one kernel applies clipping + AdamW.  The
global norm counts every parameter once: tensors replicated across the TP
group contribute ``sumsq / tp`` on each TP rank before the TP and PP
all-reduces.  The clip coefficient and the "skip this step if the loss or
the norm is not finite" decision are taken on the device, so a step needs
no host synchronisation.  Semantics match ``torch.optim.AdamW`` (decoupled
weight decay) preceded by ``clip_grad_norm_`` (reference:
qwen35_36/training.py:435-441).
"""

from __future__ import annotations

import math

import torch
import torch.distributed as dist

from graspo_b200.models.lora import LoRAAdapter


def lr_lambda(kind: str, warmup: int, total: int, min_ratio: float):
    """Multiplier of the base LR at optimizer step ``s`` (reference: transformer_adapter.py:133-187)."""
    if kind == "constant":
        return lambda s: 1.0
    decay = max(1, total - warmup)

    def cosine(s: int) -> float:
        if s < warmup:
            return s / max(1, warmup)
        progress = min((s - warmup) / decay, 1.0)
        return min_ratio + (1 - min_ratio) * 0.5 * (1 + math.cos(math.pi * progress))

    def linear(s: int) -> float:
        if s < warmup:
            return s / max(1, warmup)
        progress = min((s - warmup) / decay, 1.0)
        return min_ratio + (1 - min_ratio) * (1 - progress)

    if kind == "cosine":
        return cosine
    if kind == "linear":
        return linear
    raise ValueError(f"unsupported lr_scheduler.type: {kind} (constant, cosine, linear)")


class FlatAdamW:
    def __init__(
        self,
        adapter: LoRAAdapter,
        *,
        lr: float,
        weight_decay: float,
        betas: tuple[float, float] = (0.9, 0.999),
        eps: float = 1e-8,
        schedule=None,
        ps=None,
    ) -> None:
        self.adapter = adapter
        self.base_lr = float(lr)
        self.weight_decay = float(weight_decay)
        self.betas = betas
        self.eps = eps
        self.schedule = schedule or (lambda s: 1.0)
        self.ps = ps
        dev = adapter.params.device
        self.exp_avg = torch.zeros_like(adapter.params)
        self.exp_avg_sq = torch.zeros_like(adapter.params)
        self.step_count = 0
        self.skipped = torch.zeros(1, dtype=torch.int32, device=dev)
        self.last_sumsq = torch.zeros(1, dtype=torch.float32, device=dev)

    @property
    def lr(self) -> float:
        return self.base_lr * self.schedule(self.step_count)

    def zero_grad(self) -> None:
        self.adapter.grads.zero_()

    def global_sumsq(self) -> torch.Tensor:
        g = self.adapter.grads
        rep = self.adapter.replicated_numel
        tp = self.ps.tp_size if self.ps is not None else 1
        out = torch.zeros(2, dtype=torch.float32, device=g.device)
        if g.is_cuda:
            from graspo_b200.ops._ext import ext

            if rep:
                ext().grad_sumsq(g[:rep], out[0:1])
            if g.numel() > rep:
                ext().grad_sumsq(g[rep:], out[1:2])
        else:
            out[0] = g[:rep].pow(2).sum()
            out[1] = g[rep:].pow(2).sum()
        total = (out[0] / tp + out[1]).reshape(1)
        if self.ps is not None and self.ps.distributed:
            for group, size in ((self.ps.tp_group, self.ps.tp_size), (self.ps.pp_group, self.ps.pp_size)):
                if size > 1:
                    dist.all_reduce(total, group=group)
        return total

    def step(self, max_grad_norm: float, loss: torch.Tensor | None = None) -> torch.Tensor:
        """Clip + AdamW; returns the (device) pre-clip gradient norm."""
        self.step_count += 1
        sumsq = self.global_sumsq()
        self.last_sumsq = sumsq
        lr = self.base_lr * self.schedule(self.step_count - 1)
        b1, b2 = self.betas
        p, g = self.adapter.params, self.adapter.grads
        if p.is_cuda:
            from graspo_b200.ops._ext import ext

            ext().adamw(p, g, self.exp_avg, self.exp_avg_sq, lr, b1, b2, self.eps, self.weight_decay,
                        self.step_count, sumsq, float(max_grad_norm), loss, self.skipped)
        else:
            finite = bool(torch.isfinite(sumsq).all()) and (loss is None or bool(torch.isfinite(loss).all()))
            if finite:
                norm = sumsq.sqrt()
                coef = torch.clamp(max_grad_norm / (norm + 1e-6), max=1.0) if max_grad_norm > 0 else 1.0
                gc = g * coef
                p.mul_(1 - lr * self.weight_decay)
                self.exp_avg.mul_(b1).add_(gc, alpha=1 - b1)
                self.exp_avg_sq.mul_(b2).addcmul_(gc, gc, value=1 - b2)
                bc1 = 1 - b1 ** self.step_count
                bc2 = 1 - b2 ** self.step_count
                denom = (self.exp_avg_sq.sqrt() / math.sqrt(bc2)).add_(self.eps)
                p.addcdiv_(self.exp_avg, denom, value=-lr / bc1)
            else:
                self.skipped += 1
        self.adapter.invalidate()
        return sumsq.sqrt()

    def state_dict(self) -> dict:
        return {
            "exp_avg": self.exp_avg.detach().cpu(),
            "exp_avg_sq": self.exp_avg_sq.detach().cpu(),
            "step": self.step_count,
            "base_lr": self.base_lr,
            "weight_decay": self.weight_decay,
            "betas": list(self.betas),
            "eps": self.eps,
        }

    def load_state_dict(self, state: dict) -> None:
        self.exp_avg.copy_(state["exp_avg"].to(self.exp_avg.device))
        self.exp_avg_sq.copy_(state["exp_avg_sq"].to(self.exp_avg_sq.device))
        self.step_count = int(state["step"])
