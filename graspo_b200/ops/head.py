"""Selected-token log-probabilities over a full vocabulary on the kernel path.

``selected_token_logprobs(h, weight, targets)`` returns ``log softmax(h @ weight^T)[t, targets[t]]``
for normed hidden states ``h`` [T, H] and a vocabulary projection ``weight`` [V, H]
(both bf16, on the GPU), as an autograd function of ``h``:

* forward: one tcgen05 GEMM over the vocabulary whose epilogue keeps, per block
  of 256 vocabulary columns, each row's running (max, sum of exp) and picks up
  its target logit; ``lse_combine`` merges the blocks.  The [T, V] logits are
  never stored (fp32 accumulation, as in an fp32 matmul of the bf16 inputs);
* backward: per chunk of tokens the same GEMM recomputes the logits and its
  epilogue writes ``g * (onehot(target) - softmax)`` in bf16, which a second
  GEMM multiplies by ``weight``.

``vocab_logits(h, weight)`` gives the fp32 logits of a few rows (sampling):
the same GEMM with an fp32 store, the vocabulary on the MMA rows when there
are at most 128 tokens.

The reference computes fp32 logits chunk by chunk and takes gather - logsumexp
(src/graspo/backends/graspoflow/tensor_utils.py:167-186).  The families whose
decoder is a PyTorch module (the Qwen3.5 hybrid) use this for their LM head;
the dense family's fused path calls the same GEMM epilogues directly.
"""

from __future__ import annotations

import torch

from graspo_b200.ops._ext import ext
from graspo_b200.ops.gemm import gemm

_BLOCK = 256  # vocabulary columns per (max, sum-exp) partial
_ROWS = 128   # token rows are padded to whole GEMM tiles


def kernel_head_ok(h: torch.Tensor, weight: torch.Tensor) -> bool:
    """Shapes and types the kernels take: bf16 CUDA tensors whose hidden and
    vocabulary sizes are whole 64-wide GEMM K tiles."""
    return (h.is_cuda and weight.is_cuda and h.dtype == torch.bfloat16 and weight.dtype == torch.bfloat16
            and h.shape[-1] == weight.shape[1] and h.shape[-1] % 64 == 0 and weight.shape[0] % 64 == 0)


class _SelectedTokenLogprob(torch.autograd.Function):
    @staticmethod
    def forward(ctx, h, weight, targets, chunk_tokens):
        T, V = h.shape[0], weight.shape[0]
        pad = (-T) % _ROWS
        if pad:
            h = torch.cat([h, h.new_zeros(pad, h.shape[1])])
            targets = torch.cat([targets, targets.new_zeros(pad)])
        Tp = T + pad
        nblk = (V + _BLOCK - 1) // _BLOCK
        part = torch.empty(Tp, nblk, 2, device=h.device, dtype=torch.float32)
        tl = torch.zeros(Tp, device=h.device, dtype=torch.float32)
        gemm(h, weight, torch.empty(0, device=h.device), epilogue="lse", aux=part.view(Tp, nblk * 2),
             targets=targets, tgt_logit=tl, bn=_BLOCK)
        lse = torch.empty(Tp, device=h.device, dtype=torch.float32)
        logp = torch.empty(Tp, device=h.device, dtype=torch.float32)
        ext().lse_combine(part, tl, lse, logp)
        ctx.save_for_backward(h, weight, targets, lse)
        ctx.rows, ctx.chunk = T, int(chunk_tokens)
        return logp[:T]

    @staticmethod
    def backward(ctx, g):
        h, weight, targets, lse = ctx.saved_tensors
        Tp = h.shape[0]
        scale = torch.zeros(Tp, device=h.device, dtype=torch.float32)
        scale[: ctx.rows] = g.float()
        dh = torch.empty_like(h)
        step = max(_ROWS, ctx.chunk // _ROWS * _ROWS)
        for t0 in range(0, Tp, step):
            t1 = min(Tp, t0 + step)
            dlog = gemm(h[t0:t1], weight, epilogue="softmax_grad", targets=targets[t0:t1],
                        row_lse=lse[t0:t1].contiguous(), row_scale=scale[t0:t1].contiguous())
            gemm(dlog, weight, dh[t0:t1], b_mn=True)
            del dlog
        return dh[: ctx.rows], None, None, None


def selected_token_logprobs(h: torch.Tensor, weight: torch.Tensor, targets: torch.Tensor, *,
                            chunk_tokens: int = 8192) -> torch.Tensor:
    """log p(targets) [T] (fp32) of ``h`` [T, H] under the vocabulary projection ``weight`` [V, H]."""
    if not kernel_head_ok(h, weight):
        raise ValueError("selected_token_logprobs takes bf16 CUDA tensors with H and V multiples of 64")
    if h.shape[0] == 0:
        return (h.sum(-1) * 0).float()                    # no tokens: an empty result tied to h
    return _SelectedTokenLogprob.apply(h.contiguous(), weight.contiguous(), targets.reshape(-1).long().contiguous(),
                                       chunk_tokens)


def vocab_logits(h: torch.Tensor, weight: torch.Tensor) -> torch.Tensor:
    """fp32 logits ``h @ weight^T`` [T, V] (bf16 operands, fp32 accumulation and store)."""
    if not kernel_head_ok(h, weight):
        raise ValueError("vocab_logits takes bf16 CUDA tensors with H and V multiples of 64")
    h = h.contiguous()
    if h.shape[0] <= _ROWS:
        return gemm(weight.contiguous(), h, swap=True, epilogue="store_f32")
    return gemm(h, weight.contiguous(), epilogue="store_f32")
