"""The fused tensor-parallel reduction of prefill / training on one GPU.

The GEMM's slot push and ``tp_reduce`` are checked with every "rank" in this
GPU's memory (two receive slots and a counter in local tensors): the push
writes the same tile into every destination slot (all-reduce) or each row
into its owner's slot (reduce-scatter), counts the remote destinations'
elements, and ``tp_reduce`` sums the slots in rank order.  The last test makes
the bounded wait run out on a counter that nothing increments and checks that
the error word turns into ``KernelTimeout``.  The two-GPU version (real peers)
is in tests/test_multigpu.py.
"""

import pytest
import torch

pytestmark = pytest.mark.gpu


def _rand(*shape, scale=1.0):
    return (torch.randn(*shape, device="cuda") * scale).bfloat16()


def _push_kwargs(slots, ctr, scatter_rows=0, self_rank=0):
    n = slots.shape[0]
    out_tab = torch.tensor([slots[q].data_ptr() for q in range(n)], dtype=torch.int64)
    sig_tab = torch.tensor([0 if q == self_rank else ctr.data_ptr() + 8 * q for q in range(n)], dtype=torch.int64)
    return {"push_out": out_tab, "push_sig": sig_tab, "push_self": self_rank, "push_rows": scatter_rows}


@pytest.mark.parametrize("M,N,K", [(300, 512, 256), (128, 4096, 64), (513, 1024, 320)])
def test_slot_push_all_reduce_layout(M, N, K):
    from graspo_b200.ops._ext import check_errors
    from graspo_b200.ops.gemm import gemm

    a, w, r = _rand(M, K, scale=0.5), _rand(N, K, scale=0.5), _rand(M, N)
    slots = torch.full((2, M, N), float("nan"), device="cuda", dtype=torch.bfloat16)
    ctr = torch.zeros(2, device="cuda", dtype=torch.int64)
    gemm(a, w, slots[0], residual=r, push=_push_kwargs(slots, ctr))
    torch.cuda.synchronize()
    check_errors()
    ref = a.float() @ w.float().T + r.float()
    err = (slots[0].float() - ref).abs().max().item() / ref.abs().max().item()
    assert err < 1e-2, err
    assert torch.equal(slots[0], slots[1]), "every destination receives the same bits"
    assert int(ctr[1].item()) == M * N and int(ctr[0].item()) == 0


def test_slot_push_reduce_scatter_rows():
    from graspo_b200.ops._ext import check_errors
    from graspo_b200.ops.gemm import gemm

    M, N, K, ranks = 384, 1024, 192, 4
    rows = M // ranks
    a, w = _rand(M, K, scale=0.5), _rand(N, K, scale=0.5)
    slots = torch.full((ranks, rows, N), float("nan"), device="cuda", dtype=torch.bfloat16)
    ctr = torch.zeros(ranks, device="cuda", dtype=torch.int64)
    gemm(a, w, slots[1], push=_push_kwargs(slots, ctr, scatter_rows=rows, self_rank=1))
    torch.cuda.synchronize()
    check_errors()
    ref = (a.float() @ w.float().T).view(ranks, rows, N)
    err = (slots.float() - ref).abs().max().item() / ref.abs().max().item()
    assert err < 1e-2, err
    assert [int(c) for c in ctr.tolist()] == [rows * N, 0, rows * N, rows * N]


def test_slot_push_dgrad_layout_with_residual():
    """The dgrad form: dy @ W with W read as stored (MN-major B) plus the LoRA path as a residual."""
    from graspo_b200.ops._ext import check_errors
    from graspo_b200.ops.gemm import gemm

    T, n_out, k_in = 256, 768, 512
    dy, W, tmp = _rand(T, n_out, scale=0.5), _rand(n_out, k_in, scale=0.5), _rand(T, k_in)
    slots = torch.zeros(2, T, k_in, device="cuda", dtype=torch.bfloat16)
    ctr = torch.zeros(2, device="cuda", dtype=torch.int64)
    gemm(dy, W, slots[0], b_mn=True, residual=tmp, push=_push_kwargs(slots, ctr))
    torch.cuda.synchronize()
    check_errors()
    ref = dy.float() @ W.float() + tmp.float()
    assert (slots[1].float() - ref).abs().max().item() / ref.abs().max().item() < 1e-2
    assert int(ctr[1].item()) == T * k_in


def test_tp_reduce_sums_slots_in_rank_order():
    from graspo_b200.ops._ext import check_errors, err_word, ext

    rows, H, ranks = 777, 4096, 3
    slots = _rand(ranks, rows, H)
    res = _rand(rows, H)
    ctr = torch.tensor([12345], device="cuda", dtype=torch.int64)
    out = torch.empty(rows, H, device="cuda", dtype=torch.bfloat16)
    srcs = torch.tensor([slots[q].data_ptr() for q in range(ranks)], dtype=torch.int64)
    ext().tp_reduce(srcs, ctr.data_ptr(), 12345, res, out, H, err_word(out.device), 0)
    torch.cuda.synchronize()
    check_errors()
    want = ((slots[0].float() + slots[1].float()) + slots[2].float()) + res.float()
    assert torch.equal(out, want.bfloat16())


def test_tp_reduce_wait_runs_out_and_raises():
    """A counter that nothing increments: the wait gives up after ~1 ms of SM
    clocks, records kErrPeerTimeout, writes nothing, and check_errors raises."""
    from graspo_b200.ops._ext import ERROR_NAMES, KernelTimeout, check_errors, err_word, ext

    rows, H = 64, 512
    slots = _rand(2, rows, H)
    ctr = torch.zeros(1, device="cuda", dtype=torch.int64)
    out = torch.zeros(rows, H, device="cuda", dtype=torch.bfloat16)
    srcs = torch.tensor([slots[0].data_ptr(), slots[1].data_ptr()], dtype=torch.int64)
    word = err_word(out.device)
    ext().tp_reduce(srcs, ctr.data_ptr(), 1, None, out, H, word, 2_000_000)
    torch.cuda.synchronize()
    assert ERROR_NAMES.get(int(word[0].item()), "").lower().find("peer") >= 0
    with pytest.raises(KernelTimeout):
        check_errors()
    assert int(out.abs().sum().item()) == 0, "a timed-out reduction writes nothing"
    # the context stays usable: the same call with the counter satisfied works
    ctr.fill_(1)
    ext().tp_reduce(srcs, ctr.data_ptr(), 1, None, out, H, word, 2_000_000)
    torch.cuda.synchronize()
    check_errors()
    assert torch.equal(out, (slots[0].float() + slots[1].float()).bfloat16())
