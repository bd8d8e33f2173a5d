"""Autograd entry points of the hybrid-decoder kernels (csrc/hybrid_ops.cu).

Reference counterpart: the DeltaNet mixer's causal conv1d + SiLU, its gated
RMSNorm and the gated attention's sigmoid output gate, PyTorch ops in the
reference (src/graspo/backends/graspoflow/models/common/layers.py:358-633).

On CUDA tensors each op is one forward and one backward kernel (fp32
arithmetic, one rounding per stored value; frozen weights get no gradient).
On the CPU the same functions compute with PyTorch ops; the CPU tests use
them as the reference semantics.
"""

from __future__ import annotations

import torch
import torch.nn.functional as F

from graspo_b200.ops._ext import ext


def _conv_silu_torch(x: torch.Tensor, prev: torch.Tensor | None, w: torch.Tensor) -> torch.Tensor:
    K = w.shape[1]
    xt = x.transpose(1, 2)
    ext_in = torch.cat([prev, xt], -1) if prev is not None else F.pad(xt, (K - 1, 0))
    return F.silu(F.conv1d(ext_in, w[:, None, :], groups=x.shape[2])).transpose(1, 2)


class _ConvSilu(torch.autograd.Function):
    @staticmethod
    def forward(ctx, x, prev, w):
        y = torch.empty_like(x)
        ext().conv_silu_fwd(x, prev, w, y)
        ctx.save_for_backward(x, prev if prev is not None else torch.empty(0, device=x.device), w)
        ctx.has_prev = prev is not None
        return y

    @staticmethod
    def backward(ctx, dy):
        x, prev, w = ctx.saved_tensors
        dx = torch.empty_like(x)
        ext().conv_silu_bwd(x, prev if ctx.has_prev else None, w, dy.contiguous(), dx)
        return dx, None, None


def conv_silu(x: torch.Tensor, prev: torch.Tensor | None, w: torch.Tensor) -> torch.Tensor:
    """silu(causal depthwise conv1d) over channels-last ``x`` [B, S, C] with weight ``w`` [C, K];
    ``prev`` [B, C, K-1] holds the inputs before position 0 (zeros when None)."""
    if not x.is_cuda:
        return _conv_silu_torch(x, prev, w)
    return _ConvSilu.apply(x.contiguous(), None if prev is None else prev.contiguous().to(x.dtype),
                           w.contiguous().to(x.dtype))


def _gated_rmsnorm_torch(x, z, w, eps):
    xf = x.float()
    y = (xf * torch.rsqrt(xf.pow(2).mean(-1, keepdim=True) + eps)).to(x.dtype)
    return (w * y * F.silu(z.float())).to(x.dtype)


class _GatedRMSNorm(torch.autograd.Function):
    @staticmethod
    def forward(ctx, x, z, w, eps):
        y = torch.empty_like(x)
        ext().gated_rmsnorm_fwd(x, z, w, y, eps)
        ctx.save_for_backward(x, z, w)
        ctx.eps = eps
        return y

    @staticmethod
    def backward(ctx, dy):
        x, z, w = ctx.saved_tensors
        dx, dz = torch.empty_like(x), torch.empty_like(z)
        ext().gated_rmsnorm_bwd(x, z, w, dy.contiguous(), dx, dz, ctx.eps)
        return dx, dz, None, None


def gated_rmsnorm(x: torch.Tensor, z: torch.Tensor, w: torch.Tensor, eps: float) -> torch.Tensor:
    """``w * rmsnorm(x) * silu(z)`` per row of the last dimension (fp32 statistics)."""
    if not x.is_cuda:
        return _gated_rmsnorm_torch(x, z, w, eps)
    z = z.to(x.dtype).contiguous()
    return _GatedRMSNorm.apply(x.contiguous(), z, w.to(x.dtype).contiguous(), float(eps))


class _SigmoidGate(torch.autograd.Function):
    @staticmethod
    def forward(ctx, o, g):
        y = torch.empty_like(o)
        ext().sigmoid_gate_fwd(o, g, y)
        ctx.save_for_backward(o, g)
        return y

    @staticmethod
    def backward(ctx, dy):
        o, g = ctx.saved_tensors
        do, dg = torch.empty_like(o), torch.empty_like(g)
        ext().sigmoid_gate_bwd(o, g, dy.contiguous(), do, dg)
        return do, dg


def sigmoid_gate(o: torch.Tensor, g: torch.Tensor) -> torch.Tensor:
    """``o * sigmoid(g)`` (the gated attention's output gate)."""
    if not o.is_cuda:
        return o * torch.sigmoid(g)
    return _SigmoidGate.apply(o.contiguous(), g.to(o.dtype).contiguous())
