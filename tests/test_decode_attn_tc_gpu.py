"""Paged decode attention on tcgen05 / TMA (csrc/decode_attn_tc.cu) against an fp32 oracle.

Covers the shared-prompt mode (prompt keys attended once per group for all of
its rows, the rows' own keys split) and the plain split mode, page sizes 16 and
64, 4 and 8 query heads per KV head, left-padded prompts, rows of different
lengths, and two calls in a row (the arrival counters must be left at zero).
"""

import math

import pytest
import torch

pytestmark = pytest.mark.gpu


def _oracle(q, kp, vp, bt, start, length, scale):
    rows, nq, D = q.shape
    nkv = kp.shape[1]
    G = nq // nkv
    out = torch.empty(rows, nq, D, device=q.device)
    for r in range(rows):
        keys = torch.cat([kp[int(p)] for p in bt[r]], 1)[:, int(start[r]) : int(length[r])].float()
        vals = torch.cat([vp[int(p)] for p in bt[r]], 1)[:, int(start[r]) : int(length[r])].float()
        qq = q[r].float().view(nkv, G, D)
        out[r] = (torch.softmax(qq @ keys.transpose(1, 2) * scale, -1) @ vals).reshape(nq, D)
    return out.view(rows, nq * D)


def _case(seed, *, groups, group_rows, nkv, G, page, P, gen_cap):
    g = torch.Generator(device="cuda").manual_seed(seed)
    gc = torch.Generator().manual_seed(seed)
    rows, nq, D = groups * group_rows, nkv * G, 128
    pp, gp = P // page, -(-gen_cap // page)
    num_pages = groups * pp + rows * gp + 3
    kp = torch.randn(num_pages, nkv, page, D, device="cuda", generator=g).bfloat16()
    vp = torch.randn(num_pages, nkv, page, D, device="cuda", generator=g).bfloat16()
    q = torch.randn(rows, nq, D, device="cuda", generator=g).bfloat16()
    perm = torch.randperm(num_pages, generator=gc)
    bt = torch.empty(rows, pp + gp, dtype=torch.int32)
    for r in range(rows):
        grp = r // group_rows
        bt[r, :pp] = perm[grp * pp : (grp + 1) * pp]
        base = groups * pp + r * gp
        bt[r, pp:] = perm[base : base + gp]
    start = torch.empty(rows, dtype=torch.int32)
    length = torch.empty(rows, dtype=torch.int32)
    for grp in range(groups):
        s0 = int(torch.randint(0, max(1, P // 2), (1,), generator=gc))
        for j in range(group_rows):
            r = grp * group_rows + j
            start[r] = s0
            length[r] = P + int(torch.randint(1, gen_cap + 1, (1,), generator=gc))
    return q, kp, vp, bt.cuda(), start.cuda(), length.cuda()


@pytest.mark.parametrize("page,G,prefix,splits", [(64, 4, True, 2), (16, 4, True, 3), (64, 8, True, 1),
                                                  (64, 4, False, 3), (16, 8, False, 1)])
def test_decode_attention_tcgen05_matches_oracle(page, G, prefix, splits):
    from graspo_b200.ops._ext import check_errors, err_word, ext

    groups, group_rows, nkv, P, gen_cap = 3, 4, 2, 192, 200
    scale = 1.0 / math.sqrt(128)
    scratch = None
    for call in range(2):
        q, kp, vp, bt, start, length = _case(10 * page + G + call, groups=groups, group_rows=group_rows, nkv=nkv,
                                             G=G, page=page, P=P, gen_cap=gen_cap)
        rows, nq = q.shape[0], q.shape[1]
        slots = splits + (1 if prefix else 0)
        if scratch is None:
            scratch = torch.zeros(rows * nq * slots * 130 + rows * nkv, device="cuda")
        out = torch.full((rows, nq * 128), float("nan"), device="cuda", dtype=torch.bfloat16)
        ext().paged_decode_attention_tc(q, kp, vp, bt, start, length, out, scale, splits, scratch,
                                        P if prefix else 0, group_rows, 1, err_word(q.device))
        torch.cuda.synchronize()
        check_errors()
        want = _oracle(q, kp, vp, bt, start, length, scale)
        err = (out.float() - want).abs().max().item() / want.abs().max().item()
        assert err < 2e-2, f"call {call}: max rel err {err}"
        counters = scratch[rows * nq * slots * 130 :].view(torch.int32)
        assert int(counters.abs().sum().item()) == 0, "arrival counters must be left at zero"


def test_decode_attention_tcgen05_prompt_splits_and_long_rows():
    """Two prompt slices per group and rows that use their whole capacity."""
    from graspo_b200.ops._ext import check_errors, err_word, ext

    groups, group_rows, nkv, G, page, P, gen_cap = 2, 8, 4, 4, 64, 512, 384
    q, kp, vp, bt, start, length = _case(3, groups=groups, group_rows=group_rows, nkv=nkv, G=G, page=page, P=P,
                                         gen_cap=gen_cap)
    length[0] = P + gen_cap
    rows, nq = q.shape[0], q.shape[1]
    splits, psplits = 2, 2
    scratch = torch.zeros(rows * nq * (splits + psplits) * 130 + rows * nkv, device="cuda")
    out = torch.empty(rows, nq * 128, device="cuda", dtype=torch.bfloat16)
    scale = 1.0 / math.sqrt(128)
    ext().paged_decode_attention_tc(q, kp, vp, bt, start, length, out, scale, splits, scratch, P, group_rows,
                                    psplits, err_word(q.device))
    torch.cuda.synchronize()
    check_errors()
    want = _oracle(q, kp, vp, bt, start, length, scale)
    assert (out.float() - want).abs().max().item() / want.abs().max().item() < 2e-2
