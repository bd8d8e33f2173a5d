"""Hybrid-decoder kernels (csrc/hybrid_ops.cu) against fp32 PyTorch references:
causal conv1d + SiLU (with and without a carried state), the gated RMSNorm and
the sigmoid output gate, forward values and input gradients."""

import pytest
import torch
import torch.nn.functional as F

pytestmark = pytest.mark.gpu


def _rel(a, b):
    return (a.float() - b.float()).abs().max().item() / (b.float().abs().max().item() + 1e-6)


@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float32])
@pytest.mark.parametrize("with_prev", [False, True])
def test_conv_silu_matches_reference(dtype, with_prev):
    from graspo_b200.ops.hybrid import conv_silu

    B, S, C, K = 3, 37, 96, 4
    g = torch.Generator(device="cuda").manual_seed(1)
    x = torch.randn(B, S, C, device="cuda", generator=g).to(dtype).requires_grad_(True)
    w = (torch.randn(C, K, device="cuda", generator=g) * 0.5).to(dtype)
    prev = torch.randn(B, C, K - 1, device="cuda", generator=g).to(dtype) if with_prev else None
    y = conv_silu(x, prev, w)
    dy = torch.randn_like(y)
    (y.float() * dy.float()).sum().backward()
    xr = x.detach().float().requires_grad_(True)
    xt = xr.transpose(1, 2)
    ext_in = torch.cat([prev.float(), xt], -1) if with_prev else F.pad(xt, (K - 1, 0))
    yr = F.silu(F.conv1d(ext_in, w.float()[:, None, :], groups=C)).transpose(1, 2)
    (yr * dy.float()).sum().backward()
    tol = 1e-2 if dtype == torch.bfloat16 else 1e-5
    assert _rel(y, yr) < tol
    assert _rel(x.grad, xr.grad) < 2 * tol


@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float32])
def test_gated_rmsnorm_matches_reference(dtype):
    from graspo_b200.ops.hybrid import gated_rmsnorm

    rows, D, eps = 50, 128, 1e-6
    g = torch.Generator(device="cuda").manual_seed(2)
    x = torch.randn(rows, D, device="cuda", generator=g).to(dtype).requires_grad_(True)
    z = torch.randn(rows, D, device="cuda", generator=g).to(dtype).requires_grad_(True)
    w = (1 + 0.1 * torch.randn(D, device="cuda", generator=g)).to(dtype)
    y = gated_rmsnorm(x, z, w, eps)
    dy = torch.randn_like(y)
    (y.float() * dy.float()).sum().backward()
    xr, zr = x.detach().float().requires_grad_(True), z.detach().float().requires_grad_(True)
    yr = w.float() * (xr * torch.rsqrt(xr.pow(2).mean(-1, keepdim=True) + eps)) * F.silu(zr)
    (yr * dy.float()).sum().backward()
    tol = 2e-2 if dtype == torch.bfloat16 else 1e-5
    assert _rel(y, yr) < tol
    assert _rel(x.grad, xr.grad) < 2 * tol
    assert _rel(z.grad, zr.grad) < 2 * tol


def test_sigmoid_gate_matches_reference():
    from graspo_b200.ops.hybrid import sigmoid_gate

    g = torch.Generator(device="cuda").manual_seed(3)
    o = torch.randn(7, 300, device="cuda", generator=g).bfloat16().requires_grad_(True)
    gate = torch.randn(7, 300, device="cuda", generator=g).bfloat16().requires_grad_(True)
    y = sigmoid_gate(o, gate)
    dy = torch.randn_like(y)
    (y.float() * dy.float()).sum().backward()
    orf, gr = o.detach().float().requires_grad_(True), gate.detach().float().requires_grad_(True)
    yr = orf * torch.sigmoid(gr)
    (yr * dy.float()).sum().backward()
    assert _rel(y, yr) < 1e-2
    assert _rel(o.grad, orf.grad) < 2e-2
    assert _rel(gate.grad, gr.grad) < 2e-2
