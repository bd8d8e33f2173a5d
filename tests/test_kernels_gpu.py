"""Numerics of the sm_100a kernels against plain PyTorch fp32 references."""

import math

import pytest
import torch

pytestmark = pytest.mark.gpu


def _ext():
    from graspo_b200.ops._ext import ext

    return ext()


def _rand(*shape, scale=1.0, dtype=torch.bfloat16):
    return (torch.randn(*shape, device="cuda") * scale).to(dtype)


def _close(out, ref, tol):
    err = (out.float() - ref.float()).abs().max().item()
    den = ref.float().abs().max().item() + 1e-6
    assert err / den < tol, f"max rel err {err / den:.3e} (abs {err:.3e})"


@pytest.fixture(autouse=True)
def _seed():
    torch.manual_seed(0)
    yield
    from graspo_b200.ops._ext import check_errors

    torch.cuda.synchronize()
    check_errors()


@pytest.mark.parametrize("m,n,k", [(128, 256, 64), (300, 520, 512), (1000, 1536, 1024), (64, 4096, 4096)])
def test_gemm_store(m, n, k):
    from graspo_b200.ops.gemm import gemm

    a, b = _rand(m, k), _rand(n, k)
    out = gemm(a, b)
    _close(out, a.float() @ b.float().T, 2e-2)


@pytest.mark.parametrize("bn", [64, 128, 256])
def test_gemm_tile_widths_and_residual(bn):
    from graspo_b200.ops.gemm import gemm

    a, b, r = _rand(384, 256), _rand(640, 256), _rand(384, 640)
    out = gemm(a, b, residual=r, bn=bn)
    _close(out, a.float() @ b.float().T + r.float(), 2e-2)


def test_gemm_lora_extension():
    from graspo_b200.ops.gemm import gemm

    m, n, k, r = 257, 384, 512, 48
    x, w = _rand(m, k), _rand(n, k)
    A, B = _rand(r, k, scale=0.05), _rand(n, r, scale=0.05)
    s = 2.0
    u = torch.zeros(m, 64, device="cuda", dtype=torch.bfloat16)
    u[:, :r] = ((x.float() @ A.float().T) * s).bfloat16()
    bpad = torch.zeros(n, 64, device="cuda", dtype=torch.bfloat16)
    bpad[:, :r] = B
    out = gemm(x, w, ext_ab=(u, bpad))
    ref = x.float() @ w.float().T + u[:, :r].float() @ B.float().T
    _close(out, ref, 2e-2)


def test_gemm_swiglu():
    from graspo_b200.ops.gemm import gemm

    m, i, k = 200, 384, 256
    x, wg, wu = _rand(m, k), _rand(i, k, scale=0.1), _rand(i, k, scale=0.1)
    inter = torch.stack([wg, wu], dim=1).reshape(2 * i, k).contiguous()
    aux = torch.empty(m, 2 * i, device="cuda", dtype=torch.bfloat16)
    out = gemm(x, inter, epilogue="swiglu", aux=aux)
    g, u = x.float() @ wg.float().T, x.float() @ wu.float().T
    _close(out, torch.nn.functional.silu(g) * u, 3e-2)
    _close(aux.view(m, i, 2)[..., 0], g, 2e-2)


@pytest.mark.parametrize("splits", [1, 3])
def test_gemm_atomic_split_k(splits):
    from graspo_b200.ops.gemm import gemm

    a, b = _rand(130, 768), _rand(300, 768)
    out = gemm(a, b, epilogue="atomic", splits=splits)
    _close(out, a.float() @ b.float().T, 1e-2)


@pytest.mark.parametrize("bn", [64, 128, 256])
def test_gemm_b_mn_major(bn):
    """dY @ W with the weight read as stored ([N_out, K_in], MN-major B), with and without a K-extension."""
    from graspo_b200.ops.gemm import gemm

    dy, w = _rand(300, 448), _rand(448, 200)
    out = gemm(dy, w, b_mn=True, bn=bn)
    _close(out, dy.float() @ w.float(), 1e-2)
    du, a = _rand(300, 64), _rand(64, 200)
    out2 = gemm(dy, w, b_mn=True, bn=bn, ext_ab=(du, a))
    _close(out2, dy.float() @ w.float() + du.float() @ a.float(), 1e-2)


@pytest.mark.parametrize("swap", [False, True])
def test_gemm_both_mn_major_split_k(swap):
    """Contraction over the shared leading (token) dimension: A^T B, fp32 split-K atomics."""
    from graspo_b200.ops.gemm import gemm

    x, du = _rand(1000, 320), _rand(1000, 64)
    ref = x.float().T @ du.float()                       # [320, 64]
    out = torch.zeros(64, 320, device="cuda") if swap else torch.zeros(320, 64, device="cuda")
    gemm(x, du, out, epilogue="atomic", splits=3, a_mn=True, b_mn=True, swap=swap)
    _close(out, ref.T if swap else ref, 1e-2)


@pytest.mark.parametrize("tokens", [8, 64, 100])
@pytest.mark.parametrize("epilogue", ["store", "atomic", "store_f32"])
def test_gemm_swap(tokens, epilogue):
    from graspo_b200.ops.gemm import gemm

    w, x = _rand(384, 512), _rand(tokens, 512)
    out = gemm(w, x, swap=True, epilogue=epilogue, splits=2 if epilogue == "atomic" else 1)
    _close(out, x.float() @ w.float().T, 2e-2)


def test_gemm_swap_swiglu_and_residual():
    from graspo_b200.ops.gemm import gemm

    i, k, t = 256, 256, 40
    wg, wu, x = _rand(i, k, scale=0.1), _rand(i, k, scale=0.1), _rand(t, k)
    inter = torch.stack([wg, wu], dim=1).reshape(2 * i, k).contiguous()
    out = gemm(inter, x, swap=True, epilogue="swiglu")
    ref = torch.nn.functional.silu(x.float() @ wg.float().T) * (x.float() @ wu.float().T)
    _close(out, ref, 3e-2)
    w, r = _rand(384, k), _rand(t, 384)
    _close(gemm(w, x, swap=True, residual=r), x.float() @ w.float().T + r.float(), 2e-2)


@pytest.mark.parametrize("t,splits,i", [(64, 3, 640), (40, 2, 640), (100, 4, 640), (64, 3, 10000)])
def test_gemm_swap_swiglu_split_k(t, splits, i):
    """Split-K SwiGLU: per-split fp32 partial tiles, the last split of each tile
    applies the activation; counters are left zeroed for the next call.  With
    more tiles than SMs (i = 10000) only the last wave's tiles are split."""
    from graspo_b200.ops.gemm import gemm

    k = 1024
    wg, wu, x = _rand(i, k, scale=0.05), _rand(i, k, scale=0.05), _rand(t, k)
    a2, b2 = _rand(2 * i, 64, scale=0.05), _rand(t, 64, scale=0.5)    # LoRA-style K extension
    inter = torch.stack([wg, wu], dim=1).reshape(2 * i, k).contiguous()
    full = x.float() @ inter.float().T + b2.float() @ a2.float().T
    ref = torch.nn.functional.silu(full[:, 0::2]) * full[:, 1::2]
    ws = torch.empty(splits * t * 2 * i, device="cuda")
    ctr = torch.zeros(-(-2 * i // 128) * -(-t // 64), device="cuda", dtype=torch.int32)
    for _ in range(3):
        out = gemm(inter, x, swap=True, epilogue="swiglu", ext_ab=(a2, b2), splits=splits, aux=ws, tile_ctr=ctr)
        _close(out, ref, 3e-2)
        assert int(ctr.abs().sum()) == 0
    one = gemm(inter, x, swap=True, epilogue="swiglu", ext_ab=(a2, b2))
    _close(out, one.float(), 2e-2)


def test_gemm_lse_and_softmax_grad():
    from graspo_b200.ops.gemm import gemm

    t, v, h = 300, 1000, 256
    x, w = _rand(t, h), _rand(v, h, scale=0.2)
    tgt = torch.randint(0, v, (t,), device="cuda")
    nblk = (v + 255) // 256
    part = torch.empty(t, nblk, 2, device="cuda")
    tl = torch.empty(t, device="cuda")
    gemm(x, w, epilogue="lse", aux=part.view(t, nblk * 2), targets=tgt, tgt_logit=tl, bn=256)
    lse, logp = torch.empty(t, device="cuda"), torch.empty(t, device="cuda")
    _ext().lse_combine(part, tl, lse, logp)
    logits = x.float() @ w.float().T
    ref = torch.log_softmax(logits, -1).gather(1, tgt[:, None]).squeeze(1)
    assert (logp - ref).abs().max().item() < 2e-2
    g = torch.randn(t, device="cuda")
    dl = gemm(x, w, epilogue="softmax_grad", targets=tgt, row_lse=lse, row_scale=g)
    ref_dl = g[:, None] * (torch.nn.functional.one_hot(tgt, v).float() - torch.softmax(logits, -1))
    _close(dl, ref_dl, 3e-2)


def _rmsnorm_ref(x, w, eps):
    xf = x.float()
    return xf * torch.rsqrt(xf.pow(2).mean(-1, keepdim=True) + eps) * w.float()


@pytest.mark.parametrize("delta_dtype", [None, torch.bfloat16, torch.float32])
def test_add_rmsnorm(delta_dtype):
    h, w = _rand(37, 4096), _rand(4096, scale=0.1) + 1
    y = torch.empty_like(h)
    hout = torch.empty_like(h)
    A = _rand(48, 4096, scale=0.02)
    U = torch.empty(37, 64, device="cuda", dtype=torch.bfloat16)
    delta = None if delta_dtype is None else _rand(37, 4096).to(delta_dtype)
    ref_in = h.float() + (delta.float() if delta is not None else 0)
    ref_in = ref_in.bfloat16()
    dcopy = delta.clone() if delta is not None else None
    _ext().add_rmsnorm(h, delta, hout if delta is not None else None, w, y, None, A, U, 2.0, 1e-6)
    ref = _rmsnorm_ref(ref_in, w, 1e-6)
    _close(y, ref, 2e-2)
    _close(U[:, :48], 2.0 * ref.bfloat16().float() @ A.float().T, 3e-2)
    assert U[:, 48:].abs().max().item() == 0
    if delta_dtype is torch.float32:
        assert delta.abs().max().item() == 0, "fp32 workspace must be zeroed after use"
    if dcopy is not None:
        _close(hout, ref_in, 1e-2)


@pytest.mark.parametrize("r,R", [(16, 32), (64, 128), (5, 7)])
def test_add_rmsnorm_lora_b_u_and_down(r, R):
    """fp32 split-K delta with U columns after H: x' = h + delta + B U, then the
    norm and U' = s y A^T; LoRA rows stream through the shared-memory ring."""
    from graspo_b200.ops._ext import check_errors, err_word

    rows, H = 37, 4096
    h, w = _rand(rows, H), _rand(H, scale=0.1) + 1
    bt = _rand(r, H, scale=0.05)                       # B^T [r, H]
    u = torch.randn(rows, r, device="cuda")
    delta = torch.zeros(rows, H + 64, device="cuda")
    delta[:, :H] = torch.randn(rows, H, device="cuda")
    delta[:, H:H + r] = u
    ref_in = (h.float() + delta[:, :H] + u @ bt.float()).bfloat16()
    A = _rand(R, H, scale=0.02)
    U = torch.full((rows, 128), 7.0, device="cuda", dtype=torch.bfloat16)
    zt = torch.ones(rows, 24, device="cuda")
    y, hout = torch.empty_like(h), torch.empty_like(h)
    _ext().add_rmsnorm(h, delta, hout, w, y, None, A, U, 2.0, 1e-6, bt, r, err=err_word(h.device), zero_tail=zt)
    torch.cuda.synchronize()
    check_errors()
    _close(hout, ref_in, 1e-2)
    ref = _rmsnorm_ref(ref_in, w, 1e-6)
    _close(y, ref, 2e-2)
    _close(U[:, :R], 2.0 * ref.bfloat16().float() @ A.float().T, 3e-2)
    assert R == U.shape[1] or U[:, R:].abs().max().item() == 0
    assert delta.abs().max().item() == 0 and zt.abs().max().item() == 0


def test_rmsnorm_bwd():
    x = _rand(19, 1024).requires_grad_(False)
    w = _rand(1024, scale=0.1) + 1
    dy = _rand(19, 1024)
    xf = x.float().requires_grad_(True)
    _rmsnorm_ref(xf, w, 1e-6).backward(dy.float())
    dx = torch.empty_like(x)
    _ext().rmsnorm_bwd(dy, x, w, None, None, dx, 1e-6)
    _close(dx, xf.grad, 2e-2)


def _rope_ref(x, pos, inv_freq):
    f = pos.float()[:, None] * inv_freq[None, :]
    emb = torch.cat([f, f], -1)
    cos, sin = emb.cos()[:, None, :], emb.sin()[:, None, :]
    x1, x2 = x[..., :64], x[..., 64:]
    rot = torch.cat([-x2, x1], -1)
    return x * cos + rot * sin


def test_qk_norm_rope_and_bwd():
    T, nq, nkv, D = 23, 4, 2, 128
    qkv = _rand(T, (nq + 2 * nkv) * D)
    qw, kw = _rand(D, scale=0.1) + 1, _rand(D, scale=0.1) + 1
    inv_freq = 1.0 / (1e6 ** (torch.arange(0, D, 2, device="cuda", dtype=torch.float32) / D))
    pos = torch.randint(0, 3000, (T,), device="cuda")
    q = torch.empty(T, nq, D, device="cuda", dtype=torch.bfloat16)
    k = torch.empty(T, nkv, D, device="cuda", dtype=torch.bfloat16)
    v = torch.empty_like(k)
    _ext().qk_norm_rope(qkv, qw, kw, inv_freq, pos, q, k, v, None, None, None, nq, nkv, 64, 1e-6)
    x = qkv.float().view(T, nq + 2 * nkv, D).requires_grad_(True)
    qr = _rope_ref(_rmsnorm_ref(x[:, :nq], qw, 1e-6), pos, inv_freq)
    kr = _rope_ref(_rmsnorm_ref(x[:, nq:nq + nkv], kw, 1e-6), pos, inv_freq)
    _close(q, qr, 2e-2)
    _close(k, kr, 2e-2)
    _close(v, x[:, nq + nkv:], 1e-2)
    dq, dk, dv = _rand(T, nq, D), _rand(T, nkv, D), _rand(T, nkv, D)
    (qr * dq.float()).sum().add_((kr * dk.float()).sum()).add_((x[:, nq + nkv:] * dv.float()).sum()).backward()
    dqkv = torch.empty_like(qkv)
    _ext().qk_norm_rope_bwd(dq, dk, dv, qkv, qw, kw, inv_freq, pos, dqkv, nq, nkv, 1e-6)
    _close(dqkv, x.grad.view(T, -1), 3e-2)


def test_swiglu_bwd_lora_down_embedding_transpose():
    gu, dh = _rand(33, 2 * 96), _rand(33, 96)
    dgu = torch.empty_like(gu)
    _ext().swiglu_bwd(gu, dh, dgu)
    x = gu.float().view(33, 96, 2).requires_grad_(True)
    (torch.nn.functional.silu(x[..., 0]) * x[..., 1] * dh.float()).sum().backward()
    _close(dgu, x.grad.view(33, -1), 2e-2)

    xx, A = _rand(10, 3072), _rand(40, 3072, scale=0.05)
    U = torch.empty(10, 64, device="cuda", dtype=torch.bfloat16)
    _ext().lora_down(xx, A, U, 0.5)
    _close(U[:, :40], 0.5 * xx.float() @ A.float().T, 2e-2)

    table, ids = _rand(100, 64), torch.randint(0, 100, (17,), device="cuda")
    out = torch.empty(17, 64, device="cuda", dtype=torch.bfloat16)
    _ext().embedding(ids, table, out)
    assert torch.equal(out, table[ids])

    m = _rand(70, 45)
    t = torch.empty(45, 70, device="cuda", dtype=torch.bfloat16)
    _ext().transpose_bf16(m, t)
    assert torch.equal(t, m.T)


@pytest.mark.parametrize("page,G", [(16, 4), (64, 4), (64, 8), (128, 2)])
def test_paged_decode_attention(page, G):
    rows, nkv, D = 6, 2, 128
    nq = nkv * G
    lens = torch.tensor([5, 16, 17, 40, 33, 64], device="cuda", dtype=torch.int32) * (page // 16)
    starts = torch.tensor([0, 3, 0, 7, 1, 0], device="cuda", dtype=torch.int32) * (page // 16)
    max_pages = 4
    num_pages = rows * max_pages
    perm = torch.randperm(num_pages, device="cuda").int().view(rows, max_pages)
    kp, vp = _rand(num_pages, nkv, page, D), _rand(num_pages, nkv, page, D)
    q = _rand(rows, nq, D)
    out = torch.empty(rows, nq * D, device="cuda", dtype=torch.bfloat16)
    scale = 1 / math.sqrt(D)
    _ext().paged_decode_attention(q, kp, vp, perm, starts, lens, out, scale, 1, None)
    scratch = torch.zeros(rows * nq * 3 * (D + 2) + rows * nkv, device="cuda")
    out3 = torch.empty_like(out)
    for _ in range(2):  # the split path resets its counters: a second launch must agree
        _ext().paged_decode_attention(q, kp, vp, perm, starts, lens, out3, scale, 3, scratch)
        _close(out3, out, 1e-2)
    for r in range(rows):
        L = int(lens[r])
        s0 = int(starts[r])
        keys = torch.cat([kp[perm[r, p]] for p in range(max_pages)], dim=1)[:, s0:L]  # [nkv, L, D]
        vals = torch.cat([vp[perm[r, p]] for p in range(max_pages)], dim=1)[:, s0:L]
        kk = keys.float().repeat_interleave(nq // nkv, 0)
        vv = vals.float().repeat_interleave(nq // nkv, 0)
        att = torch.softmax(q[r].float()[:, None, :] @ kk.transpose(1, 2) * scale, -1) @ vv
        _close(out[r].view(nq, D), att.squeeze(1), 2e-2)


@pytest.mark.parametrize("G,R", [(4, 4), (4, 8), (8, 8), (2, 3)])
def test_paged_decode_attention_shared_prefix(G, R):
    """Prompt pages shared by the R rows of a group, attended once per group."""
    nkv, D, page, P = 2, 128, 64, 192
    nq = nkv * G
    groups = 2
    rows = groups * R
    gen_pages = 3
    prompt_pages = P // page
    num_pages = groups * prompt_pages + rows * gen_pages
    kp, vp = _rand(num_pages, nkv, page, D), _rand(num_pages, nkv, page, D)
    bt = torch.empty(rows, prompt_pages + gen_pages, dtype=torch.int32)
    for r in range(rows):
        grp = r // R
        bt[r, :prompt_pages] = torch.arange(grp * prompt_pages, (grp + 1) * prompt_pages)
        base = groups * prompt_pages + r * gen_pages
        bt[r, prompt_pages:] = torch.arange(base, base + gen_pages)
    bt = bt.cuda()
    start = torch.tensor([7] * R + [0] * R, device="cuda", dtype=torch.int32)
    # every row's keys fit its block table (prompt pages + gen_pages)
    lens = torch.tensor([P + 1 + (gen_pages * page - 1) * r // (rows - 1) for r in range(rows)], device="cuda",
                        dtype=torch.int32)
    assert int(lens.max()) <= bt.shape[1] * page
    q = _rand(rows, nq, D)
    scale = 1 / math.sqrt(D)
    splits = 2
    ref = torch.empty(rows, nq * D, device="cuda", dtype=torch.bfloat16)
    scratch = torch.zeros(rows * nq * 3 * (D + 2) + rows * nkv, device="cuda")
    _ext().paged_decode_attention(q, kp, vp, bt, start, lens, ref, scale, 3, scratch)
    out = torch.empty_like(ref)
    pscr = torch.zeros(rows * nq * (splits + 4 * 2) * (D + 2) + rows * nkv, device="cuda")
    for _ in range(2):
        _ext().paged_decode_attention(q, kp, vp, bt, start, lens, out, scale, splits, pscr, P, R, 2)
        _close(out, ref, 1e-2)
    for r in range(rows):
        keys = torch.cat([kp[bt[r, p]] for p in range(bt.shape[1])], dim=1)[:, int(start[r]) : int(lens[r])]
        vals = torch.cat([vp[bt[r, p]] for p in range(bt.shape[1])], dim=1)[:, int(start[r]) : int(lens[r])]
        kk = keys.float().repeat_interleave(G, 0)
        vv = vals.float().repeat_interleave(G, 0)
        att = torch.softmax(q[r].float()[:, None, :] @ kk.transpose(1, 2) * scale, -1) @ vv
        _close(out[r].view(nq, D), att.squeeze(1), 2e-2)


def _attn_reference(q, k, v, start, end, B, S, scale):
    """fp32 reference of causal attention over per-row valid ranges."""
    from graspo_b200.ops import emulate

    T, nq, D = q.shape
    out = torch.empty(T, nq, D, device=q.device)
    lse = torch.empty(T, nq, device=q.device)
    emulate.flash_attn_fwd(q, k, v, out, lse, start, end, B, S, scale)
    return out, lse


@pytest.mark.parametrize("S,G", [(96, 2), (300, 4), (64, 1), (520, 8)])
def test_flash_attention_forward_tcgen05(S, G):
    from graspo_b200.ops._ext import check_errors, err_word

    B, nkv, D = 3, 2, 128
    nq = nkv * G
    T = B * S
    q, k, v = _rand(T, nq, D), _rand(T, nkv, D), _rand(T, nkv, D)
    start = torch.tensor([0, 17, 5], device="cuda", dtype=torch.int32)
    end = torch.tensor([S, S, S - 23], device="cuda", dtype=torch.int32)
    scale = 1 / math.sqrt(D)
    out = torch.empty(T, nq, D, device="cuda", dtype=torch.bfloat16)
    lse = torch.empty(T, nq, device="cuda")
    _ext().flash_attn_fwd_tc(q, k, v, out, lse, start, end, B, S, scale, err_word(q.device))
    torch.cuda.synchronize()
    check_errors()
    ref, ref_lse = _attn_reference(q, k, v, start, end, B, S, scale)
    _close(out, ref, 2e-2)
    assert (lse - ref_lse).abs().max().item() < 2e-2


def _attn_grads_reference(q, k, v, dout, start, end, B, S, G, scale):
    """Autograd of the fp32 reference: (dq, dk, dv)."""
    T, nq, D = q.shape
    nkv = k.shape[1]
    qf, kf, vf = (t.float().requires_grad_(True) for t in (q, k, v))
    idx = torch.arange(S, device="cuda")
    valid = (idx[None] >= start[:, None]) & (idx[None] < end[:, None])
    allowed = valid[:, None, :] & valid[:, :, None] & (idx[:, None] >= idx[None, :])[None]
    qh = qf.view(B, S, nq, D).transpose(1, 2)
    kh = kf.view(B, S, nkv, D).transpose(1, 2).repeat_interleave(G, 1)
    vh = vf.view(B, S, nkv, D).transpose(1, 2).repeat_interleave(G, 1)
    s = (qh @ kh.transpose(-1, -2) * scale).masked_fill(~allowed[:, None], float("-inf"))
    p = torch.softmax(s, -1).nan_to_num(0.0)
    o = (p @ vh) * valid[:, None, :, None]
    o.transpose(1, 2).reshape(T, nq, D).mul(dout.float()).sum().backward()
    return qf.grad, kf.grad, vf.grad


@pytest.mark.parametrize("S,G", [(96, 2), (300, 4), (64, 1), (520, 8), (384, 4)])
def test_flash_attention_backward_tcgen05(S, G):
    from graspo_b200.ops._ext import check_errors, err_word

    B, nkv, D = 3, 2, 128
    nq = nkv * G
    T = B * S
    q, k, v = _rand(T, nq, D), _rand(T, nkv, D), _rand(T, nkv, D)
    start = torch.tensor([0, 17, 5], device="cuda", dtype=torch.int32)
    end = torch.tensor([S, S, S - 23], device="cuda", dtype=torch.int32)
    scale = 1 / math.sqrt(D)
    out = torch.empty(T, nq, D, device="cuda", dtype=torch.bfloat16)
    lse = torch.empty(T, nq, device="cuda")
    _ext().flash_attn_fwd_tc(q, k, v, out, lse, start, end, B, S, scale, err_word(q.device))
    dout = _rand(T, nq, D)
    rq, rk, rv = _attn_grads_reference(q, k, v, dout, start, end, B, S, G, scale)
    dq, dk, dv = torch.full_like(q, float("nan")), torch.full_like(k, float("nan")), torch.full_like(v, float("nan"))
    for _ in range(2):  # a second run must not depend on leftovers of the first
        _ext().flash_attn_bwd_tc(dout, q, k, v, out, lse, dq, dk, dv, start, end, B, S, scale, err_word(q.device))
        torch.cuda.synchronize()
        check_errors()
        _close(dq, rq, 3e-2)
        _close(dk, rk, 3e-2)
        _close(dv, rv, 3e-2)


def test_sample_append_greedy_and_distribution():
    rows, V = 4, 50
    logits = torch.randn(rows, V, device="cuda")
    state = dict(
        next_ids=torch.zeros(rows, dtype=torch.long, device="cuda"),
        slot=torch.full((rows,), 9, dtype=torch.long, device="cuda"),
        pos=torch.zeros(rows, dtype=torch.long, device="cuda"),
        kv_len=torch.zeros(rows, dtype=torch.int32, device="cuda"),
        finished=torch.zeros(rows, dtype=torch.uint8, device="cuda"),
        out=torch.zeros(rows, 4, dtype=torch.long, device="cuda"),
    )
    _ext().sample_append(logits, 0.0, 1.0, 1, state["next_ids"], state["slot"], state["pos"], state["kv_len"],
                         state["finished"], state["out"], 10, -1, 0, False, None)
    assert torch.equal(state["next_ids"], logits.argmax(-1))
    assert torch.equal(state["out"][:, 0], logits.argmax(-1))
    assert int(state["slot"][0]) == 10 and int(state["kv_len"][0]) == 11
    # distribution: many independent rows of the same logits
    n = 4000
    lg = torch.log(torch.tensor([0.5, 0.3, 0.15, 0.05], device="cuda")).repeat(n, 1)
    ids = torch.zeros(n, dtype=torch.long, device="cuda")
    slot = torch.zeros(n, dtype=torch.long, device="cuda")
    _ext().sample_append(lg, 1.0, 1.0, 123, ids, slot, torch.zeros_like(slot), torch.zeros(n, dtype=torch.int32, device="cuda"),
                         torch.zeros(n, dtype=torch.uint8, device="cuda"), torch.zeros(n, 1, dtype=torch.long, device="cuda"),
                         1, -1, 0, False, None)
    freq = torch.bincount(ids, minlength=4).float() / n
    assert (freq - torch.tensor([0.5, 0.3, 0.15, 0.05], device="cuda")).abs().max() < 0.03
    # top-p 0.7 keeps only the two most likely tokens
    _ext().sample_append(lg, 1.0, 0.7, 7, ids, slot, torch.zeros_like(slot), torch.zeros(n, dtype=torch.int32, device="cuda"),
                         torch.zeros(n, dtype=torch.uint8, device="cuda"), torch.zeros(n, 1, dtype=torch.long, device="cuda"),
                         1, -1, 0, False, None)
    assert int(ids.max()) <= 1


def test_grpo_loss_matches_reference():
    from graspo_b200.core.loss import GRASPOLoss

    B, S = 5, 37
    lp = (torch.randn(B, S, device="cuda") * 0.1 - 2).requires_grad_(True)
    old = lp.detach() + torch.randn(B, S, device="cuda") * 0.3
    adv = torch.randn(B, 1, device="cuda").expand(B, S).contiguous()
    mask = torch.rand(B, S, device="cuda") > 0.3
    ref = GRASPOLoss(0.2)(lp, old, adv, mask)
    ref.backward()
    loss = torch.zeros(1, device="cuda")
    dlp = torch.empty(B, S, device="cuda")
    _ext().grpo_loss(lp.detach(), old, adv, mask.to(torch.uint8), 0.2, 1.0, loss, dlp, None)
    assert abs(loss.item() - ref.item()) < 1e-5
    _close(dlp, lp.grad, 1e-4)


def test_adamw_matches_torch():
    n = 1000
    p0 = torch.randn(n, device="cuda")
    grads = [torch.randn(n, device="cuda") * 3 for _ in range(3)]
    ref = p0.clone().requires_grad_(True)
    opt = torch.optim.AdamW([ref], lr=1e-3, weight_decay=0.01)
    p, m, v = p0.clone(), torch.zeros(n, device="cuda"), torch.zeros(n, device="cuda")
    for step, g in enumerate(grads, start=1):
        ref.grad = g.clone()
        torch.nn.utils.clip_grad_norm_([ref], 1.0)
        opt.step()
        ss = torch.zeros(1, device="cuda")
        _ext().grad_sumsq(g, ss)
        _ext().adamw(p, g, m, v, 1e-3, 0.9, 0.999, 1e-8, 0.01, step, ss, 1.0, None, None)
    _close(p, ref.detach(), 1e-5)


@pytest.mark.parametrize("temperature", [1.0, 0.0])
def test_split_sampler_matches_single_pass(temperature):
    """The split sampler draws the same noise per vocabulary entry as the one-CTA-per-row sampler,
    so both pick the same tokens and leave the same decode state."""
    rows, V = 5, 151936
    logits = torch.randn(rows, V, device="cuda") * 2

    def state():
        return dict(next_ids=torch.zeros(rows, dtype=torch.long, device="cuda"),
                    slot=torch.arange(rows, device="cuda", dtype=torch.long) + 40,
                    pos=torch.zeros(rows, dtype=torch.long, device="cuda"),
                    kv_len=torch.zeros(rows, dtype=torch.int32, device="cuda"),
                    finished=torch.zeros(rows, dtype=torch.uint8, device="cuda"),
                    out=torch.zeros(rows, 64, dtype=torch.long, device="cuda"))

    from graspo_b200.ops._ext import check_errors, err_word

    a, b = state(), state()
    chunk = 15196
    nch = -(-V // chunk)
    scratch = torch.zeros(rows * (1 + 2 * nch) + 2, device="cuda")
    for step in range(3):
        _ext().sample_append(logits, temperature, 1.0, 11, a["next_ids"], a["slot"], a["pos"], a["kv_len"],
                             a["finished"], a["out"], 32, -1, 0, True, None)
        _ext().sample_append_split(logits, temperature, 11, b["next_ids"], b["slot"], b["pos"], b["kv_len"],
                                   b["finished"], b["out"], 32, -1, 0, True, 0, scratch, chunk, err_word())
    torch.cuda.synchronize()
    check_errors()
    for k in a:
        assert torch.equal(a[k], b[k]), k
    assert int(scratch[:rows].view(torch.int32).abs().sum().item()) == 0, "row counters are left at zero"


def test_dropout_statistics():
    x = torch.ones(100000, device="cuda", dtype=torch.bfloat16)
    y = torch.empty_like(x)
    _ext().dropout(x, y, 0.1, 5, 3, None)
    kept = (y != 0).float().mean().item()
    assert abs(kept - 0.9) < 0.01
    assert abs(y[y != 0].float().mean().item() - 1 / 0.9) < 1e-2
    y2 = torch.empty_like(x)
    _ext().dropout(x, y2, 0.1, 5, 3, None)
    assert torch.equal(y, y2), "same seed and stream must regenerate the same mask"


def test_dropout_tail_add_and_streams():
    n = 100003  # not a multiple of the 8-element vectors
    x = (torch.randn(n, device="cuda") + 3).bfloat16()
    a = torch.randn(n, device="cuda").bfloat16()
    y0, y = torch.empty_like(x), torch.empty_like(x)
    _ext().dropout(x, y0, 0.25, 9, 1, None)
    _ext().dropout(x, y, 0.25, 9, 1, a)
    keep = y0 != 0
    assert abs(keep.float().mean().item() - 0.75) < 0.01
    want = (x.float() * keep.float() * (1.0 / 0.75) + a.float()).bfloat16()
    assert torch.equal(y, want), "the added variant applies the same mask"
    tail = (x[-3:].float() * keep[-3:].float() * (1.0 / 0.75)).bfloat16()
    assert torch.equal(y0[-3:], tail), "the tail elements are masked and scaled like the rest"
    y3 = torch.empty_like(x)
    _ext().dropout(x, y3, 0.25, 9, 2, None)
    assert ((y3 != 0) != keep).float().mean().item() > 0.2, "another stream id draws another mask"


@pytest.mark.parametrize("dk,dv", [(64, 64), (128, 128), (128, 96)])
def test_gated_delta_step_matches_recurrence(dk, dv):
    from graspo_b200.models.qwen35 import l2norm, recurrent_gated_delta

    B, h = 3, 5
    q = (l2norm(torch.randn(B, h, dk, device="cuda")) / dk ** 0.5).float()
    k = l2norm(torch.randn(B, h, dk, device="cuda")).float()
    v = torch.randn(B, h, dv, device="cuda")
    g = -torch.rand(B, h, device="cuda")
    beta = torch.rand(B, h, device="cuda")
    state = torch.randn(B, h, dk, dv, device="cuda") * 0.1
    ref_state = state.clone()
    ref = recurrent_gated_delta(q, k, v, g, beta, ref_state)
    out = torch.empty(B, h, dv, device="cuda")
    for _ in range(1):
        _ext().gated_delta_step(q, k, v, g, beta, state, out)
    _close(out, ref, 1e-4)
    _close(state, ref_state, 1e-4)


def test_kernel_checks_flag_and_decode_attention_with_error_word():
    """The loaded build reports whether index checks are compiled in; the decode
    attention accepts the error word either way and leaves it clear on valid input."""
    from graspo_b200.ops._ext import check_errors, err_word

    assert isinstance(_ext().kernel_checks(), bool)
    rows, nq, nkv, D, page = 4, 8, 2, 128, 64
    kp = _rand(8, nkv, page, D)
    vp = _rand(8, nkv, page, D)
    bt = torch.arange(8, device="cuda", dtype=torch.int32).view(rows, 2)
    q = _rand(rows, nq, D)
    start = torch.zeros(rows, device="cuda", dtype=torch.int32)
    ln = torch.full((rows,), 100, device="cuda", dtype=torch.int32)
    out = torch.empty(rows, nq * D, device="cuda", dtype=torch.bfloat16)
    scratch = torch.zeros(rows * nq * 2 * (D + 2) + rows * nkv, device="cuda")
    _ext().paged_decode_attention(q, kp, vp, bt, start, ln, out, 1 / math.sqrt(D), 2, scratch, err=err_word(q.device))
    torch.cuda.synchronize()
    check_errors()
