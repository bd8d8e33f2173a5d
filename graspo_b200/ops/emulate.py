"""Plain-PyTorch emulation of every kernel-library entry point.

Same names and signatures as ``graspo_b200._C``; results are computed with
ordinary tensor operations in fp32 and stored in the caller's buffers.  It
exists for CPU tests of the fused orchestration code (layouts, LoRA
K-extension, split-K workspaces, paged cache bookkeeping): with
``use_emulation()`` active, ``ext()`` returns this module, so the fused
model, rollout engine and optimizer run on a machine without a GPU and can be
compared with the eager oracle.  It is never used on a GPU run.
"""

from __future__ import annotations

import contextlib
import math

import torch

EPI_STORE, EPI_SWIGLU, EPI_ATOMIC, EPI_LSE, EPI_STORE_F32, EPI_SOFTMAX_GRAD = range(6)


def _f(x):
    return x.float()


def gemm_tc(A, B, A2, B2, C, R, aux, targets, tgt_logit, row_lse, row_scale, epilogue, swap, bn, splits, err,
            max_ctas, push_dst=None, push_flag=None, tile_ctr=None, layout=0, push_out=None, push_sig=None,
            push_self=0, push_rows=0, push_fence_once=0):
    if push_dst is not None or push_out is not None:
        raise NotImplementedError("the peer-memory tile push needs GPUs")
    a_mn, b_mn = bool(layout & 2), bool(layout & 1)

    def op(a, b):
        return (_f(a).T if a_mn else _f(a)) @ (_f(b) if b_mn else _f(b).T)

    acc = op(A, B)
    if A2 is not None:
        acc = acc + op(A2, B2)
    if swap:
        acc = acc.T  # [tokens, features]
    M, N = acc.shape
    if epilogue == EPI_STORE:
        if R is not None:
            acc = acc + _f(R)
        C.copy_(acc.to(C.dtype))
    elif epilogue == EPI_STORE_F32:
        C.copy_(acc)
    elif epilogue == EPI_ATOMIC:
        C.add_(acc)
    elif epilogue == EPI_SWIGLU:
        pre = acc.to(torch.bfloat16).float()
        g, u = pre[:, 0::2], pre[:, 1::2]
        C.copy_((torch.nn.functional.silu(g) * u).to(C.dtype))
        if aux is not None and not (swap and splits > 1):  # split-K swap: aux is the kernel's workspace
            aux.copy_(acc.to(aux.dtype))
    elif epilogue == EPI_LSE:
        nblk = math.ceil(N / bn)
        part = aux.view(M, nblk, 2)
        for b in range(nblk):
            blk = acc[:, b * bn : (b + 1) * bn]
            mx = blk.max(-1).values
            part[:, b, 0] = mx
            part[:, b, 1] = torch.exp(blk - mx[:, None]).sum(-1)
        t = targets.long()
        inside = (t >= 0) & (t < N)
        tgt_logit.copy_(torch.where(inside, acc.gather(1, t.clamp(0, N - 1)[:, None]).squeeze(1), tgt_logit))
    elif epilogue == EPI_SOFTMAX_GRAD:
        t = targets.long()
        onehot = torch.zeros_like(acc)
        inside = (t >= 0) & (t < N)
        onehot[inside, t[inside]] = 1.0
        C.copy_((row_scale[:, None] * (onehot - torch.exp(acc - row_lse[:, None]))).to(C.dtype))
    else:
        raise ValueError(epilogue)


def add_rmsnorm(h, delta, h_out, w, y, rstd, lora_a, lora_u, scale, eps, delta_lora_b=None, delta_lora_r=0,
                peer_src=None, peer_sync=None, peer_expected=0, err=None, zero_tail=None):
    if peer_src is not None:
        raise NotImplementedError("the peer-memory sum needs GPUs")
    if zero_tail is not None:
        zero_tail.zero_()
    x = _f(h)
    H = h.shape[-1]
    if delta is not None:
        d = _f(delta[..., :H])
        if delta_lora_b is not None:  # B^T [r, H]
            u = _f(delta[..., H : H + delta_lora_r])
            d = d + u @ _f(delta_lora_b[:delta_lora_r])
        x = x + d
        x = x.to(torch.bfloat16).float() if h.dtype == torch.bfloat16 else x
        h_out.copy_(x.to(h_out.dtype))
        if delta.dtype == torch.float32:
            delta.zero_()
    r = torch.rsqrt(x.pow(2).mean(-1) + eps)
    if rstd is not None:
        rstd.copy_(r)
    out = (x * r[:, None] * _f(w)).to(y.dtype)
    y.copy_(out)
    if lora_a is not None:
        u = (_f(out) @ _f(lora_a).T) * scale
        lora_u.zero_()
        lora_u[:, : lora_a.shape[0]] = u.to(lora_u.dtype)


def rmsnorm_bwd(dy, x, w, rstd, dres, dx, eps):
    xf = _f(x).requires_grad_(True)
    with torch.enable_grad():
        y = xf * torch.rsqrt(xf.pow(2).mean(-1, keepdim=True) + eps) * _f(w)
        (g,) = torch.autograd.grad(y, xf, _f(dy))
    if dres is not None:
        g = g + _f(dres)
    dx.copy_(g.to(dx.dtype))


def _rope(x, pos, inv_freq):
    f = pos.float()[:, None] * inv_freq[None, :]
    emb = torch.cat([f, f], -1)[:, None, :]
    half = x.shape[-1] // 2
    rot = torch.cat([-x[..., half:], x[..., :half]], -1)
    return x * emb.cos() + rot * emb.sin()


def _head_norm(x, w, eps):
    return (x * torch.rsqrt(x.pow(2).mean(-1, keepdim=True) + eps) * _f(w)).to(torch.bfloat16).float()


def qk_norm_rope(qkv, q_w, k_w, inv_freq, pos, q_out, k_out, v_out, block_table, row_of_token, slot, nq, nkv,
                 page_size, eps, lora_b=None, lora_r=0, err=None):
    T = qkv.shape[0]
    D = q_out.shape[-1]
    W = (nq + 2 * nkv) * D
    x = _f(qkv[:, :W])
    if lora_b is not None:  # B^T [3r, W] of the block-diagonal B
        u = _f(qkv[:, W : W + 3 * lora_r])
        x = x + u @ _f(lora_b[: 3 * lora_r])
    x = x.view(T, nq + 2 * nkv, D)
    if qkv.dtype == torch.float32:
        x = x.to(torch.bfloat16).float()
        qkv[:, :W].zero_()
    q = _rope(_head_norm(x[:, :nq], q_w, eps), pos, inv_freq)
    k = _rope(_head_norm(x[:, nq : nq + nkv], k_w, eps), pos, inv_freq)
    v = x[:, nq + nkv :]
    q_out.copy_(q.to(q_out.dtype).view_as(q_out))
    if block_table is None:
        k_out.copy_(k.to(k_out.dtype).view_as(k_out))
        v_out.copy_(v.to(v_out.dtype).view_as(v_out))
        return
    for t in range(T):
        row = int(row_of_token[t])
        s = int(slot[t])
        page = int(block_table[row, s // page_size])
        k_out[page, :, s % page_size] = k[t].to(k_out.dtype)
        v_out[page, :, s % page_size] = v[t].to(v_out.dtype)


def qk_norm_rope_bwd(dq, dk, dv, qkv, q_w, k_w, inv_freq, pos, dqkv, nq, nkv, eps):
    T, D = qkv.shape[0], dq.shape[-1]
    x = _f(qkv).view(T, nq + 2 * nkv, D).requires_grad_(True)
    with torch.enable_grad():
        xf = x.float()
        q = _rope(xf[:, :nq] * torch.rsqrt(xf[:, :nq].pow(2).mean(-1, keepdim=True) + eps) * _f(q_w), pos, inv_freq)
        k = _rope(xf[:, nq:nq + nkv] * torch.rsqrt(xf[:, nq:nq + nkv].pow(2).mean(-1, keepdim=True) + eps) * _f(k_w),
                  pos, inv_freq)
        out = (q * _f(dq)).sum() + (k * _f(dk)).sum() + (xf[:, nq + nkv:] * _f(dv)).sum()
        (g,) = torch.autograd.grad(out, x)
    dqkv.copy_(g.reshape(T, -1).to(dqkv.dtype))


def swiglu_bwd(gu, dh, dgu):
    g, u = _f(gu)[:, 0::2], _f(gu)[:, 1::2]
    d = _f(dh)
    sig = torch.sigmoid(g)
    out = torch.empty_like(_f(gu))
    out[:, 0::2] = d * u * sig * (1 + g * (1 - sig))
    out[:, 1::2] = d * g * sig
    dgu.copy_(out.to(dgu.dtype))


def lora_down(x, A, U, scale):
    U.zero_()
    U[:, : A.shape[0]] = ((_f(x) @ _f(A).T) * scale).to(U.dtype)


def embedding(ids, table, out):
    out.copy_(table[ids.long().clamp(0, table.shape[0] - 1)])


def paged_decode_attention(q, k_pool, v_pool, block_table, start, length, out, scale, splits, scratch,
                           prefix_len=0, group_rows=1, prefix_splits=1, err=None):
    rows, nq, D = q.shape
    nkv, page = k_pool.shape[1], k_pool.shape[2]
    G = nq // nkv
    for r in range(rows):
        s0, s1 = int(start[r]), int(length[r])
        pages = [int(block_table[r, p]) for p in range(block_table.shape[1])]
        keys = torch.cat([k_pool[p] for p in pages], 1)[:, s0:s1].float()  # [nkv, L, D]
        vals = torch.cat([v_pool[p] for p in pages], 1)[:, s0:s1].float()
        qq = q[r].float().view(nkv, G, D)
        att = torch.softmax(qq @ keys.transpose(1, 2) * scale, -1) @ vals
        out[r] = att.reshape(-1).to(out.dtype)


class _Gen:
    def __init__(self, seed):
        self.g = torch.Generator().manual_seed(int(seed) & ((1 << 62) - 1))


def _flash_scores(q, k, start, end, B, S, scale):
    T, nq, D = q.shape
    G = nq // k.shape[1]
    qh = _f(q).view(B, S, nq, D).transpose(1, 2)
    kh = _f(k).view(B, S, -1, D).transpose(1, 2).repeat_interleave(G, 1)
    idx = torch.arange(S, device=q.device)
    st, en = start.long()[:, None], end.long()[:, None]
    valid = (idx[None] >= st) & (idx[None] < en)                      # [B, S]
    allowed = valid[:, None, :] & (idx[None, :, None] >= idx[None, None, :]) & valid[:, :, None]
    s = (qh @ kh.transpose(-1, -2)) * scale
    return s.masked_fill(~allowed[:, None], float("-inf")), valid


def flash_attn_fwd(q, k, v, out, lse, start, end, B, S, scale):
    T, nq, D = q.shape
    G = nq // k.shape[1]
    s, valid = _flash_scores(q, k, start, end, B, S, scale)
    m = s.amax(-1, keepdim=True).clamp_min(-1e30)
    p = torch.exp(s - m)
    z = p.sum(-1, keepdim=True)
    vh = _f(v).view(B, S, -1, D).transpose(1, 2).repeat_interleave(G, 1)
    o = (p / z.clamp_min(1e-30)) @ vh                                  # [B, nq, S, D]
    o = o * valid[:, None, :, None]
    out.copy_(o.transpose(1, 2).reshape(T, nq, D).to(out.dtype))
    l2 = ((m + torch.log(z.clamp_min(1e-30))) / math.log(2.0)).squeeze(-1)  # log2 domain, [B, nq, S]
    l2 = torch.where(valid[:, None], l2, torch.zeros_like(l2))
    lse.copy_(l2.transpose(1, 2).reshape(T, nq))


def flash_attn_fwd_tc(q, k, v, out, lse, start, end, B, S, scale, err):
    flash_attn_fwd(q, k, v, out, lse, start, end, B, S, scale)


def flash_attn_bwd_tc(dout, q, k, v, out, lse, dq, dk, dv, start, end, B, S, scale, err):
    flash_attn_bwd(dout, q, k, v, out, lse, dq, dk, dv, start, end, B, S, scale)


def flash_attn_bwd(dout, q, k, v, out, lse, dq, dk, dv, start, end, B, S, scale):
    T, nq, D = q.shape
    nkv = k.shape[1]
    G = nq // nkv
    s, valid = _flash_scores(q, k, start, end, B, S, scale)
    l2 = lse.view(B, S, nq).transpose(1, 2)[..., None] * math.log(2.0)
    p = torch.exp(s - l2).masked_fill(~valid[:, None, :, None], 0.0)
    doh = _f(dout).view(B, S, nq, D).transpose(1, 2)
    oh = _f(out).view(B, S, nq, D).transpose(1, 2)
    vh = _f(v).view(B, S, nkv, D).transpose(1, 2).repeat_interleave(G, 1)
    qh = _f(q).view(B, S, nq, D).transpose(1, 2)
    kh = _f(k).view(B, S, nkv, D).transpose(1, 2).repeat_interleave(G, 1)
    dvh = p.transpose(-1, -2) @ doh
    dp = doh @ vh.transpose(-1, -2)
    dd = (doh * oh).sum(-1, keepdim=True)
    ds = p * (dp - dd) * scale
    dqh = ds @ kh
    dkh = ds.transpose(-1, -2) @ qh
    dq.copy_(dqh.transpose(1, 2).reshape(T, nq, D).to(dq.dtype))
    dk.copy_(dkh.view(B, nkv, G, S, D).sum(2).transpose(1, 2).reshape(T, nkv, D).to(dk.dtype))
    dv.copy_(dvh.view(B, nkv, G, S, D).sum(2).transpose(1, 2).reshape(T, nkv, D).to(dv.dtype))


def sample_append(logits, temperature, top_p, seed, next_ids, slot, pos, kv_len, finished, out_tokens, prompt_slots,
                  eos_id, pad_id, ignore_eos, active):
    rows = logits.shape[0]
    for r in range(rows):
        lg = logits[r].float()
        if temperature > 0:
            g = torch.Generator().manual_seed((int(seed) * 1000003 + r * 7919 + int(slot[r])) & ((1 << 62) - 1))
            u = torch.rand(lg.shape, generator=g).clamp_(1e-20, 1 - 1e-7)
            x = lg / temperature
            if top_p < 1:
                p = torch.softmax(x, -1)
                sp, si = torch.sort(p, descending=True)
                keep = (sp.cumsum(0) - sp) < top_p
                mask = torch.zeros_like(p, dtype=torch.bool)
                mask[si[keep]] = True
                x = x.masked_fill(~mask, float("-inf"))
            tok = int((x - torch.log(-torch.log(u))).argmax())
        else:
            tok = int(lg.argmax())
        live = (active is None or bool(active[r])) and not bool(finished[r])
        if not live:
            tok = pad_id
        s = int(slot[r])
        col = s + 1 - prompt_slots
        if 0 <= col < out_tokens.shape[1]:
            out_tokens[r, col] = tok
        if live and not ignore_eos and tok == eos_id:
            finished[r] = 1
        next_ids[r] = tok
        slot[r] = s + 1
        pos[r] = pos[r] + 1
        kv_len[r] = s + 2


def lse_combine(partials, tgt, lse, logp):
    m = partials[..., 0]
    s = partials[..., 1]
    mx = m.max(-1).values
    total = (s * torch.exp(m - mx[:, None])).sum(-1)
    lse.copy_(mx + total.log())
    logp.copy_(tgt - lse)


def grpo_loss(logp, old_logp, adv, mask, clip_eps, grad_scale, loss, dlogp, stats):
    m = mask.bool().float()
    r = torch.exp(logp - old_logp)
    u1, u2 = r * adv, r.clamp(1 - clip_eps, 1 + clip_eps) * adv
    per = -torch.minimum(u1, u2)
    cnt = m.sum(-1).clamp_min(1)
    B = logp.shape[0]
    loss.add_(((per * m).sum(-1) / cnt).sum() / B)
    d = torch.where(u1 <= u2, -r * adv, torch.zeros_like(r))
    dlogp.copy_(d * m * grad_scale / (cnt[:, None] * B))


def dropout(x, y, p, seed, stream_id, add):
    g = torch.Generator().manual_seed((int(seed) * 131 + int(stream_id)) & ((1 << 62) - 1))
    keep = (torch.rand(x.shape, generator=g) >= p).to(torch.float32)
    out = _f(x) * keep / (1 - p)
    if add is not None:
        out = out + _f(add)
    y.copy_(out.to(y.dtype))


def grad_sumsq(g, out):
    out.add_(g.float().pow(2).sum())


def adamw(p, g, m, v, lr, b1, b2, eps, wd, step, sumsq, max_norm, loss, skipped):
    ss = float(sumsq.reshape(-1)[0])
    if not math.isfinite(ss) or (loss is not None and not bool(torch.isfinite(loss).all())):
        if skipped is not None:
            skipped += 1
        return
    coef = min(1.0, max_norm / (math.sqrt(ss) + 1e-6)) if max_norm > 0 else 1.0
    gc = g * coef
    p.mul_(1 - lr * wd)
    m.mul_(b1).add_(gc, alpha=1 - b1)
    v.mul_(b2).addcmul_(gc, gc, value=1 - b2)
    bc1, bc2 = 1 - b1**step, 1 - b2**step
    p.addcdiv_(m, v.sqrt() / math.sqrt(bc2) + eps, value=-lr / bc1)


def transpose_bf16(inp, out):
    out.copy_(inp.T)


@contextlib.contextmanager
def use_emulation():
    """Route ``ext()`` to this module for the duration of the block."""
    import sys

    from graspo_b200.ops import _ext

    saved = _ext._C
    _ext._C = sys.modules[__name__]
    _ext._ERR.clear()
    try:
        yield
    finally:
        _ext._C = saved


def kernel_checks():
    return False


def tp_reduce(srcs, counter, expected, residual, out, ld_src, err, spin_limit=0):
    raise NotImplementedError("the fused tensor-parallel reduction reads peer memory and needs GPUs")


def lse_push(partials, tgt, dst, sig, self_rank):
    raise NotImplementedError("the vocab-parallel log-prob exchange writes peer memory and needs GPUs")


def lse_merge(srcs, counter, expected, lse, logp, err, spin_limit=0):
    raise NotImplementedError("the vocab-parallel log-prob exchange reads peer memory and needs GPUs")


def paged_decode_attention_tc(q, k_pool, v_pool, block_table, start, length, out, scale, splits, scratch,
                              prefix_len, group_rows, prefix_splits, err):
    paged_decode_attention(q, k_pool, v_pool, block_table, start, length, out, scale, splits, scratch)


def sample_append_split(logits, temperature, seed, next_ids, slot, pos, kv_len, finished, out_tokens, prompt_slots,
                        eos_id, pad_id, ignore_eos, vocab_start, scratch, chunk, err, exch_dst=None, exch_sig=None,
                        exch_self=0, exch_slots=0, exch_arrivals=0, spin_limit=0):
    if exch_dst is not None:
        raise NotImplementedError("the vocab-parallel sampler exchange writes peer memory and needs GPUs")
    sample_append(logits, temperature, 1.0, seed, next_ids, slot, pos, kv_len, finished, out_tokens, prompt_slots,
                  eos_id, pad_id, ignore_eos, None)
