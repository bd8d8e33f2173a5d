"""Prefill / training attention over padded batches.

Layout: q [T, nq, D], k/v [T, nkv, D] with T = B*S tokens; ``meta.key_mask``
marks valid tokens (left padding before the prompt, right padding after
EOS).  Each valid query attends causally to valid keys of its own row.  A
padding query attends only to itself, so every softmax row is non-empty; its
output is never consumed (loss masks exclude it, and no valid query attends
to padding keys).

This module currently runs the attention through
``torch.nn.functional.scaled_dot_product_attention`` (a library kernel) while
the sm_100a flash-attention kernel is developed; the decode-time attention
over the paged cache is already a hand-written kernel.
"""

from __future__ import annotations

import torch
import torch.nn.functional as F


def _mask(meta) -> torch.Tensor:
    cached = getattr(meta, "_sdpa_mask", None)
    if cached is not None:
        return cached
    S = meta.S
    dev = meta.key_mask.device
    causal = torch.ones(S, S, dtype=torch.bool, device=dev).tril()
    allowed = causal[None] & meta.key_mask[:, None, :]
    allowed |= torch.eye(S, dtype=torch.bool, device=dev)[None]
    mask = allowed[:, None]
    object.__setattr__(meta, "_sdpa_mask", mask)
    return mask


def _heads(x: torch.Tensor, B: int, S: int) -> torch.Tensor:
    return x.view(B, S, x.shape[1], x.shape[2]).transpose(1, 2)


def attention_forward(q, k, v, meta, scale: float, need_ctx: bool = False):
    B, S = meta.B, meta.S
    out = F.scaled_dot_product_attention(
        _heads(q, B, S), _heads(k, B, S), _heads(v, B, S), attn_mask=_mask(meta), scale=scale,
        enable_gqa=q.shape[1] != k.shape[1],
    )
    return out.transpose(1, 2).reshape(B * S, -1), None


def attention_backward(dout, q, k, v, out, ctx, meta, scale: float):
    B, S = meta.B, meta.S
    with torch.enable_grad():
        qh = _heads(q, B, S).detach().requires_grad_(True)
        kh = _heads(k, B, S).detach().requires_grad_(True)
        vh = _heads(v, B, S).detach().requires_grad_(True)
        o = F.scaled_dot_product_attention(qh, kh, vh, attn_mask=_mask(meta), scale=scale,
                                           enable_gqa=q.shape[1] != k.shape[1])
        dq, dk, dv = torch.autograd.grad(o, (qh, kh, vh), dout.view(B, S, -1, q.shape[2]).transpose(1, 2))
    return (dq.transpose(1, 2).reshape_as(q).contiguous(), dk.transpose(1, 2).reshape_as(k).contiguous(),
            dv.transpose(1, 2).reshape_as(v).contiguous())
