"""Tensor- and sequence-parallel autograd operators (Megatron f / g pairs).

* ``copy_to_tp`` (f): identity forward, all-reduce backward -- placed before
  every column-parallel linear so the replicated residual stream receives the
  full input gradient.  The reference has only the g half (its all-reduce has
  an identity backward, reference: tensor_utils.py:146-164), which leaves the
  residual gradients partial on each TP rank; this pair is the corrected form.
* ``reduce_from_tp`` (g): all-reduce forward, identity backward -- after every
  row-parallel linear.
* Sequence parallel: ``gather_from_sp`` (all-gather over the token dim forward,
  reduce-scatter backward) before column-parallel linears and
  ``reduce_scatter_to_sp`` (reduce-scatter forward, all-gather backward) after
  row-parallel linears; norms and residuals then run on 1/tp of the tokens.
"""

from __future__ import annotations

import torch
import torch.distributed as dist


def _size(group) -> int:
    if group is None or not (dist.is_available() and dist.is_initialized()):
        return 1
    return dist.get_world_size(group)


def _all_reduce(x: torch.Tensor, group) -> torch.Tensor:
    if _size(group) == 1:
        return x
    x = x.contiguous()
    dist.all_reduce(x, op=dist.ReduceOp.SUM, group=group)
    return x


class _CopyToTP(torch.autograd.Function):
    @staticmethod
    def forward(ctx, x, group):
        ctx.group = group
        return x

    @staticmethod
    def backward(ctx, grad):
        return _all_reduce(grad.clone(), ctx.group), None


class _ReduceFromTP(torch.autograd.Function):
    @staticmethod
    def forward(ctx, x, group):
        return _all_reduce(x.clone(), group)

    @staticmethod
    def backward(ctx, grad):
        return grad, None


def _all_gather_dim0(x: torch.Tensor, group) -> torch.Tensor:
    world = _size(group)
    if world == 1:
        return x
    x = x.contiguous()
    out = torch.empty((world * x.shape[0], *x.shape[1:]), dtype=x.dtype, device=x.device)
    dist.all_gather_into_tensor(out, x, group=group)
    return out


def _reduce_scatter_dim0(x: torch.Tensor, group) -> torch.Tensor:
    world = _size(group)
    if world == 1:
        return x
    if x.shape[0] % world:
        raise ValueError(f"token dim {x.shape[0]} not divisible by TP={world}")
    x = x.contiguous()
    out = torch.empty((x.shape[0] // world, *x.shape[1:]), dtype=x.dtype, device=x.device)
    dist.reduce_scatter_tensor(out, x, op=dist.ReduceOp.SUM, group=group)
    return out


class _GatherFromSP(torch.autograd.Function):
    @staticmethod
    def forward(ctx, x, group):
        ctx.group = group
        return _all_gather_dim0(x, group)

    @staticmethod
    def backward(ctx, grad):
        return _reduce_scatter_dim0(grad, ctx.group), None


class _ReduceScatterToSP(torch.autograd.Function):
    @staticmethod
    def forward(ctx, x, group):
        ctx.group = group
        return _reduce_scatter_dim0(x, group)

    @staticmethod
    def backward(ctx, grad):
        return _all_gather_dim0(grad, ctx.group), None


def copy_to_tp(x: torch.Tensor, group) -> torch.Tensor:
    return x if _size(group) == 1 else _CopyToTP.apply(x, group)


def reduce_from_tp(x: torch.Tensor, group) -> torch.Tensor:
    return x if _size(group) == 1 else _ReduceFromTP.apply(x, group)


def gather_from_sp(x: torch.Tensor, group) -> torch.Tensor:
    return x if _size(group) == 1 else _GatherFromSP.apply(x, group)


def reduce_scatter_to_sp(x: torch.Tensor, group) -> torch.Tensor:
    return x if _size(group) == 1 else _ReduceScatterToSP.apply(x, group)


def all_reduce_(x: torch.Tensor, group, op=None) -> torch.Tensor:
    """In-place all-reduce (no autograd) that is a no-op for a single rank."""
    if _size(group) > 1:
        dist.all_reduce(x, op=op or dist.ReduceOp.SUM, group=group)
    return x
