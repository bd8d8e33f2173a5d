"""Python face of the tcgen05 GEMM (csrc/gemm_tc.cu).

Reference counterpart: the LoRA linears ``y = x W^T + s (drop(x) A^T) B^T``
(src/graspo/backends/graspoflow/lora.py:208-213) and the LM head / log-prob
chunks (src/graspo/backends/graspoflow/tensor_utils.py:167-186), cuBLAS there.

``gemm(a, b)`` computes ``a @ b.T`` for row-major bf16 ``a [M, K]`` and
``b [N, K]`` with fp32 accumulation, plus optional fused pieces:

* ``ext=(a2, b2)``: extends the reduction with ``a2 @ b2.T`` (LoRA: ``a2`` is
  ``s * x A^T`` zero-padded to a multiple of 64 columns, ``b2`` the padded B).
* ``residual``: adds a bf16 tensor to the result.
* ``epilogue``: ``store`` (bf16), ``store_f32``, ``atomic`` (fp32 +=, allows
  split-K), ``swiglu`` (b rows interleave gate/up; output N/2 columns),
  ``lse`` (row log-sum-exp partials + target logits), ``softmax_grad``.
* ``splits`` > 1 with ``swiglu`` in swap mode: split-K whose partial tiles go to
  ``aux`` (fp32, ``splits x tokens x features``) and whose last split per
  tile applies the activation; ``tile_ctr`` is a zeroed int32 counter per
  output tile (left zeroed by the kernel).
* ``swap=True``: ``a`` is the weight ``[N_out, K]`` and ``b`` the activations
  ``[T, K]``; the result is stored as ``[T, N_out]``.  This is the decode
  shape: tokens fill the narrow N side of the tensor-core tile.
* ``b_mn=True``: ``b`` is given as ``[K, N]`` (read MN-major by the tensor
  cores, no transpose) -- e.g. ``gemm(dy, W, b_mn=True)`` is ``dy @ W`` for
  the frozen weight as stored; ``a_mn=True`` likewise takes ``a`` as
  ``[K, M]`` (with both set the product contracts over the shared leading
  dimension, e.g. LoRA gradients over tokens).
"""

from __future__ import annotations

import torch

from graspo_b200.ops._ext import err_word, ext

EPILOGUES = {"store": 0, "swiglu": 1, "atomic": 2, "lse": 3, "store_f32": 4, "softmax_grad": 5}


def pick_bn(n: int, swap: bool) -> int:
    if swap:
        if n <= 32:
            return 32
        if n <= 64:
            return 64
        return 128
    if n >= 1024:
        return 256
    if n >= 128:
        return 128
    return 64


def gemm(
    a: torch.Tensor,
    b: torch.Tensor,
    out: torch.Tensor | None = None,
    *,
    ext_ab: tuple[torch.Tensor, torch.Tensor] | None = None,
    residual: torch.Tensor | None = None,
    epilogue: str = "store",
    aux: torch.Tensor | None = None,
    targets: torch.Tensor | None = None,
    tgt_logit: torch.Tensor | None = None,
    row_lse: torch.Tensor | None = None,
    row_scale: torch.Tensor | None = None,
    swap: bool = False,
    bn: int | None = None,
    splits: int = 1,
    max_ctas: int = 0,
    push=None,
    tile_ctr: torch.Tensor | None = None,
    a_mn: bool = False,
    b_mn: bool = False,
) -> torch.Tensor:
    epi = EPILOGUES[epilogue]
    M = a.shape[1] if a_mn else a.shape[0]
    N = b.shape[1] if b_mn else b.shape[0]
    if swap:
        out_shape = (N, M // 2 if epilogue == "swiglu" else M)
    else:
        out_shape = (M, N // 2 if epilogue == "swiglu" else N)
    narrow = N
    if out is None:
        dtype = torch.float32 if epilogue in ("atomic", "store_f32") else torch.bfloat16
        if epilogue == "lse":
            out = torch.empty(0, device=a.device, dtype=torch.float32)
        else:
            out = (torch.zeros if epilogue == "atomic" else torch.empty)(out_shape, device=a.device, dtype=dtype)
    a2 = b2 = None
    if ext_ab is not None:
        a2, b2 = ext_ab
        if swap:
            # the extension pairs with (a, b) in the same roles
            pass
    bn = bn or pick_bn(narrow, swap)
    if b_mn:
        bn = max(bn, 64)
    # push: the decode all-reduce site (PeerReduce) or the slot-push tables of a
    # prefill / training site (TPAllReduce.begin's keyword arguments)
    kw = push.gemm_kwargs() if hasattr(push, "gemm_kwargs") else dict(push or {})
    if tile_ctr is not None:
        kw["tile_ctr"] = tile_ctr
    layout = (2 if a_mn else 0) | (1 if b_mn else 0)
    ext().gemm_tc(
        a, b, a2, b2, out, residual, aux, targets, tgt_logit, row_lse, row_scale,
        epi, swap, bn, splits, err_word(a.device), max_ctas, **kw, layout=layout,
    )
    return out


def lse_partials_shape(m: int, n: int, bn: int = 256) -> tuple[int, int, int]:
    return (m, (n + bn - 1) // bn, 2)
