"""Prefill / training attention over padded batches (sm_100a flash attention).

Reference counterpart: SDPA with a boolean causal + padding mask
(src/graspo/backends/graspoflow/models/common/layers_qwen3.py:252-257,
src/graspo/backends/graspoflow/tensor_utils.py:452-468).

Layout: q [T, nq, D], k/v [T, nkv, D] with T = B*S tokens; ``meta.key_mask``
marks valid tokens.  A row's valid tokens form one contiguous range
[start, end) -- left padding before the prompt, right padding after EOS --
and each valid query attends causally to the valid keys of its own row.
Padding queries produce zero output and receive zero gradient; nothing
downstream consumes them (loss masks exclude them and no valid query attends
to a padding key).

Both directions run on tcgen05 kernels (csrc/flash_attn_tc.cu): the forward
keeps S and O in TMEM and P in swizzled shared memory; the backward walks, per
128-key tile, every query tile and head of the GQA group with S^T / dP^T, dQ,
dK and dV in TMEM (dQ is added into an fp32 buffer with vector atomics).  The
forward also returns the per-(token, head) log-sum-exp (log2 domain, fp32),
which the backward uses to rebuild the probabilities without a second softmax
pass (FlashAttention-2, Dao 2023).  GQA is handled inside the kernels: a query
head reads KV head ``h // (nq // nkv)``.  On the CPU the entry points run their
emulation (graspo_b200/ops/emulate.py), used by the CPU tests.
Head dim 128 (every Qwen3 size) is the supported kernel shape.
"""

from __future__ import annotations

import torch

from graspo_b200.ops._ext import err_word, ext


def row_ranges(meta) -> tuple[torch.Tensor, torch.Tensor]:
    """int32 [B] start / end of each row's valid range, computed on device once per meta."""
    cached = getattr(meta, "_row_ranges", None)
    if cached is not None:
        return cached
    m = meta.key_mask.bool()
    S = m.shape[1]
    any_ = m.any(-1)
    first = m.int().argmax(-1)
    last = S - 1 - m.flip(-1).int().argmax(-1)
    start = torch.where(any_, first, torch.zeros_like(first)).int().contiguous()
    end = torch.where(any_, last + 1, torch.zeros_like(last)).int().contiguous()
    object.__setattr__(meta, "_row_ranges", (start, end))
    return start, end


def _check(q: torch.Tensor) -> None:
    if q.is_cuda and q.shape[-1] != 128:
        raise NotImplementedError(f"flash attention kernel supports head_dim 128, got {q.shape[-1]}")


def attention_forward(q, k, v, meta, scale: float, need_ctx: bool = False):
    """Returns (out [T, nq*D], lse [T, nq] or None)."""
    _check(q)
    T, nq, D = q.shape
    start, end = row_ranges(meta)
    out = torch.empty(T, nq * D, device=q.device, dtype=q.dtype)
    lse = torch.empty(T, nq, device=q.device, dtype=torch.float32)
    ext().flash_attn_fwd_tc(q.contiguous(), k.contiguous(), v.contiguous(), out.view(T, nq, D), lse, start, end,
                            meta.B, meta.S, float(scale), err_word(q.device))
    return out, (lse if need_ctx else None)


def attention_backward(dout, q, k, v, out, ctx, meta, scale: float):
    """dout / out [T, nq*D]; ctx is the forward's log-sum-exp.  Returns dq, dk, dv."""
    _check(q)
    T, nq, D = q.shape
    start, end = row_ranges(meta)
    if ctx is None:
        _, ctx = attention_forward(q, k, v, meta, scale, need_ctx=True)
    dq = torch.empty_like(q)
    dk = torch.empty_like(k)
    dv = torch.empty_like(v)
    args = (dout.contiguous().view(T, nq, D), q.contiguous(), k.contiguous(), v.contiguous(),
            out.contiguous().view(T, nq, D), ctx.contiguous(), dq, dk, dv, start, end, meta.B, meta.S, float(scale))
    ext().flash_attn_bwd_tc(*args, err_word(q.device))
    return dq, dk, dv
