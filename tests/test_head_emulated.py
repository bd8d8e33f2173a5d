"""The selected-token log-prob head's host logic (row padding to whole tiles,
backward chunking, ragged token counts) on the emulated kernels, against an
fp32 PyTorch reference."""

import torch


def test_head_padding_and_chunking_on_emulated_kernels():
    from graspo_b200.ops.emulate import use_emulation
    from graspo_b200.ops.head import _SelectedTokenLogprob

    g = torch.Generator().manual_seed(2)
    T, H, V = 301, 128, 512
    h = (torch.randn(T, H, generator=g) * 0.5).to(torch.bfloat16)
    w = (torch.randn(V, H, generator=g) * 0.1).to(torch.bfloat16)
    tgt = torch.randint(0, V, (T,), generator=g)
    up = torch.randn(T, generator=g)
    with use_emulation():
        hk = h.clone().requires_grad_(True)
        lp = _SelectedTokenLogprob.apply(hk, w, tgt, 128)      # three backward chunks of 128 padded rows
        (lp * up).sum().backward()
    hr = h.float().clone().requires_grad_(True)
    logits = hr @ w.float().T
    ref = logits.gather(-1, tgt[:, None]).squeeze(-1) - torch.logsumexp(logits, -1)
    (ref * up).sum().backward()
    assert lp.shape == (T,)
    assert (lp - ref).abs().max().item() < 1e-3
    assert (hk.grad.float() - hr.grad).abs().max().item() < 2e-2 * hr.grad.abs().max().item()


def test_vocab_logits_on_emulated_kernels():
    from graspo_b200.ops import head
    from graspo_b200.ops.emulate import use_emulation

    g = torch.Generator().manual_seed(3)
    w = (torch.randn(512, 128, generator=g) * 0.1).to(torch.bfloat16)
    for rows in (5, 200):
        h = (torch.randn(rows, 128, generator=g) * 0.5).to(torch.bfloat16)
        with use_emulation():
            ok = head.kernel_head_ok
            head.kernel_head_ok = lambda a, b: True          # CPU tensors through the emulated GEMM
            try:
                out = head.vocab_logits(h, w)
            finally:
                head.kernel_head_ok = ok
        assert out.shape == (rows, 512) and (out - h.float() @ w.float().T).abs().max().item() < 1e-3
