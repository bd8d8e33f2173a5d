"""The kernel-path selected-token log-prob head (tcgen05 GEMM with the
(max, sum-exp) epilogue forward, softmax-grad epilogue backward) against an
fp32 PyTorch reference, values and input gradients, on a ragged token count."""

import pytest
import torch


@pytest.mark.gpu
def test_selected_token_logprobs_matches_fp32():
    from graspo_b200.ops.head import selected_token_logprobs

    g = torch.Generator().manual_seed(0)
    T, H, V = 333, 256, 1024
    h = (torch.randn(T, H, generator=g) * 0.5).to(torch.bfloat16).cuda()
    w = (torch.randn(V, H, generator=g) * 0.1).to(torch.bfloat16).cuda()
    tgt = torch.randint(0, V, (T,), generator=g).cuda()
    up = torch.randn(T, generator=g).cuda()
    hk = h.clone().requires_grad_(True)
    lp = selected_token_logprobs(hk, w, tgt, chunk_tokens=128)
    (lp * up).sum().backward()
    hr = h.float().clone().requires_grad_(True)
    logits = hr @ w.float().T
    ref = logits.gather(-1, tgt[:, None]).squeeze(-1) - torch.logsumexp(logits, -1)
    (ref * up).sum().backward()
    assert lp.shape == (T,) and lp.dtype == torch.float32
    assert (lp - ref).abs().max().item() < 2e-3
    # the backward's softmax-grad chunk is stored in bf16
    err = (hk.grad.float() - hr.grad).abs().max().item()
    assert err < 2e-2 * hr.grad.abs().max().item(), err


@pytest.mark.gpu
@pytest.mark.parametrize("rows", [5, 200])
def test_vocab_logits_matches_fp32(rows):
    from graspo_b200.ops.head import vocab_logits

    g = torch.Generator().manual_seed(rows)
    h = (torch.randn(rows, 256, generator=g) * 0.5).to(torch.bfloat16).cuda()
    w = (torch.randn(1024, 256, generator=g) * 0.1).to(torch.bfloat16).cuda()
    out = vocab_logits(h, w)
    ref = h.float() @ w.float().T
    assert out.dtype == torch.float32 and out.shape == (rows, 1024)
    assert (out - ref).abs().max().item() < 1e-3
