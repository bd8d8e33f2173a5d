"""Fused sm_100a execution of the Qwen3 decoder (forward, backward, log-probs).

Reference counterpart: the Qwen3 layer stack and its checkpointed recompute
(src/graspo/backends/graspoflow/models/common/layers_qwen3.py, models/qwen3/model.py:338-347)
and the vocab-chunked selected-token log-prob (tensor_utils.py:167-186).

Per decoder layer the forward is ~10 kernels:

    add_rmsnorm -> [dropout] -> U = x A^T (tcgen05, N=64) -> QKV GEMM with the
    LoRA update folded into its K loop -> qk_norm_rope -> attention ->
    O GEMM (+LoRA, + residual in the epilogue) -> add_rmsnorm ->
    gate/up GEMM (+LoRA, SwiGLU epilogue) -> down GEMM (+LoRA, + residual)

Training uses whole-layer recomputation: the forward keeps only each layer's
input; the backward re-runs the layer keeping its intermediates, then runs
the backward kernels.  LoRA gradients are tensor-core reductions over tokens
(``dB = dY^T U``, ``dA = s * dU^T X``) written straight into the adapter's
flat fp32 gradient buffer.  Under tensor parallelism the input gradients of
column-parallel projections are all-reduced over the TP group (the conjugate
of the forward all-reduce after row-parallel projections).  On B200s both
directions overlap the transfer with the GEMM: the row-parallel GEMM runs in
row chunks into this rank's receive slot, the copy engines send each finished
chunk to the other ranks over NVLink on a side stream, and ``tp_reduce`` sums
the slots in rank order once the peers' chunks have arrived
(``parallel/symm.py`` TPAllReduce.gemm_reduce); with sequence parallelism each
chunk goes only to the rank that owns its tokens (reduce-scatter).

The selected-token log-prob never materialises logits: the LM-head GEMM's
epilogue emits per-tile (max, sum-exp) partials, a small kernel merges them
(and, with a vocab-parallel head, an all-reduce merges the TP shards); the
backward recomputes each logit tile and writes ``g * (onehot - softmax)``
directly from the epilogue.
"""

from __future__ import annotations

import math
from dataclasses import dataclass

import torch
import torch.distributed as dist

from graspo_b200.models.qwen3 import LayerWeights, Qwen3Model
from graspo_b200.ops import attention as attn_ops
from graspo_b200.ops._ext import ext
from graspo_b200.ops.gemm import gemm

# dropout stream ids: layer * 8 + site
_DROP_SITES = {"qkv": 0, "o": 1, "gu": 2, "down": 3}


def _tp_all_reduce(x: torch.Tensor, group) -> torch.Tensor:
    if group is not None and dist.is_initialized() and dist.get_world_size(group) > 1:
        dist.all_reduce(x, group=group)
    return x


def _sp_gather(x: torch.Tensor, group) -> torch.Tensor:
    """All-gather token shards [T/tp, ...] -> [T, ...] (sequence parallel)."""
    world = dist.get_world_size(group)
    out = torch.empty((world * x.shape[0], *x.shape[1:]), dtype=x.dtype, device=x.device)
    dist.all_gather_into_tensor(out, x.contiguous(), group=group)
    return out


def _sp_scatter(x: torch.Tensor, group) -> torch.Tensor:
    """Reduce-scatter partial sums [T, ...] -> this rank's token shard [T/tp, ...]."""
    world = dist.get_world_size(group)
    out = torch.empty((x.shape[0] // world, *x.shape[1:]), dtype=x.dtype, device=x.device)
    dist.reduce_scatter_tensor(out, x.contiguous(), op=dist.ReduceOp.SUM, group=group)
    return out


def _grad_splits(rows: int, sms: int = 148) -> int:
    """Split-K factor for a token-contracted LoRA gradient with ``rows`` output rows."""
    tiles = max(1, -(-rows // 128))
    return max(1, min(16, round(2 * sms / tiles)))


@dataclass
class AttnMeta:
    """Token layout of a padded batch: B sequences of S tokens, flattened."""

    B: int
    S: int
    key_mask: torch.Tensor      # [B, S] bool, valid tokens
    pos: torch.Tensor           # [B*S] int64 rope positions

    @staticmethod
    def from_mask(mask: torch.Tensor) -> "AttnMeta":
        m = mask.bool()
        pos = (m.long().cumsum(-1) - 1).masked_fill(~m, 0)
        return AttnMeta(B=m.shape[0], S=m.shape[1], key_mask=m, pos=pos.reshape(-1).contiguous())


class LayerSaved:
    __slots__ = ("x", "xn", "rstd1", "xd", "u_qkv", "qkv", "q", "k", "v", "attn", "attn_d", "u_o",
                 "x1", "xn2", "rstd2", "xd2", "u_gu", "gu", "act", "act_d", "u_d", "attn_ctx")


class AttnCache:
    """Values of a layer's training forward kept for the backward's recompute.

    Level 1: the q/k/v projection output, the attention output and its
    log-sum-exp (the recompute skips the q/k/v GEMM and the flash-attention
    forward).  Level 2 adds the residual after attention and the gate/up
    pre-activations with the SwiGLU output (it also skips the o and gate/up
    GEMMs).  Cached values are the forward's own tensors, so the gradients do
    not change."""

    __slots__ = ("qkv", "attn", "lse", "x1", "gu", "act", "mlp")

    def __init__(self, mlp: bool = False) -> None:
        self.qkv = self.attn = self.lse = None
        self.x1 = self.gu = self.act = None
        self.mlp = mlp


def _cache_attention_mode() -> str:
    import os

    return os.environ.get("GRASPO_CACHE_ATTN", "auto").strip().lower()


class FusedQwen3:
    """Kernel-path forward / backward of the Qwen3 decoder.

    With ``sequence_parallel`` (and TP > 1) the residual stream, the norms and
    the residual adds hold 1/tp of the tokens on each TP rank: the input of a
    column-parallel projection is all-gathered over the tokens, the output of a
    row-parallel projection is reduce-scattered (instead of all-reduced), and
    the backward pass mirrors both (Megatron sequence parallelism).
    """

    def __init__(self, model: Qwen3Model, sequence_parallel: bool = False) -> None:
        self.m = model
        self.C = ext()
        self.eps = model.cfg.rms_norm_eps
        self.scale = 1.0 / math.sqrt(model.D)
        self.sp = bool(sequence_parallel) and model.ps.tp_size > 1
        self._tp_red = None

    def tp_reducer(self):
        """The fused GEMM + all-reduce / reduce-scatter sites (CUDA with TP > 1), made on first use.

        On the CPU (gloo process groups in tests) the collectives stay library calls."""
        m = self.m
        if m.ps.tp_size == 1 or m.device.type != "cuda" or not dist.is_initialized():
            return None
        if self._tp_red is None:
            from graspo_b200.parallel.symm import TPAllReduce

            self._tp_red = TPAllReduce(m.ps.tp_group, m.device, m.cfg.hidden_size)
        return self._tp_red

    # ------------------------------------------------------------ sequence parallel
    def sp_shard(self, x: torch.Tensor) -> torch.Tensor:
        """This rank's token shard of a replicated [T, ...] tensor (identity without SP)."""
        if not self.sp:
            return x
        tp, r = self.m.ps.tp_size, self.m.ps.tp_rank
        n = x.shape[0] // tp
        return x[r * n : (r + 1) * n].contiguous()

    def sp_gather(self, x: torch.Tensor) -> torch.Tensor:
        return _sp_gather(x, self.m.ps.tp_group) if self.sp else x

    # ------------------------------------------------------------ helpers
    def _dropout(self, x, site: str, layer: int, seed: int, train: bool):
        p = self.m.lora.dropout
        if not train or p <= 0:
            return x
        y = torch.empty_like(x)
        self.C.dropout(x, y, p, seed, layer * 8 + _DROP_SITES[site], None)
        return y

    def _layouts(self, lw: LayerWeights):
        return self.m.lora.layer_layouts(lw.index, self.m.sizes)

    # ------------------------------------------------------------ forward
    def layer_forward(self, lw: LayerWeights, x: torch.Tensor, meta: AttnMeta, *, train: bool = False,
                      seed: int = 0, save: bool = False, kv_sink=None, keep: AttnCache | None = None,
                      cache: AttnCache | None = None, need_out: bool = True):
        """One decoder layer.  ``keep`` receives this forward's attention values;
        ``cache`` supplies them instead of recomputing (backward recompute);
        ``need_out=False`` skips the down projection, whose output the backward
        does not read (its inputs are saved)."""
        m, C, L = self.m, self.C, self._layouts(lw)
        tp_group = m.ps.tp_group
        tp = m.ps.tp_size
        sp = self.sp
        s = LayerSaved() if save else None
        xn = torch.empty_like(x)
        rstd1 = torch.empty(x.shape[0], device=x.device, dtype=torch.float32)
        C.add_rmsnorm(x, None, None, lw.ln1, xn, rstd1, None, None, 1.0, self.eps)
        if sp:
            xn = _sp_gather(xn, tp_group)
        T = xn.shape[0]
        ext_qkv = None
        if "a_qkv" in L:
            xd = self._dropout(xn, "qkv", lw.index, seed, train)
            u_qkv = gemm(xd, L["a_qkv"], bn=64)
            ext_qkv = (u_qkv, L["b_qkv"])
        qkv = cache.qkv if cache is not None else gemm(xn, lw.w_qkv, ext_ab=ext_qkv)
        q = torch.empty(T, m.nq, m.D, device=x.device, dtype=xn.dtype)
        k = torch.empty(T, m.nkv, m.D, device=x.device, dtype=xn.dtype)
        v = torch.empty_like(k)
        C.qk_norm_rope(qkv, lw.q_norm, lw.k_norm, m.inv_freq, meta.pos, q, k, v, None, None, None, m.nq, m.nkv, 0,
                       self.eps)
        if kv_sink is not None:
            kv_sink(lw.index, k, v)
        if cache is not None:
            attn, ctx = cache.attn, cache.lse
        else:
            attn, ctx = attn_ops.attention_forward(q, k, v, meta, self.scale, need_ctx=save or keep is not None)
        if keep is not None:
            keep.qkv, keep.attn, keep.lse = qkv, attn, ctx
        mlp_cached = cache is not None and cache.x1 is not None
        ext_o = None
        if "a_o" in L:
            attn_d = self._dropout(attn, "o", lw.index, seed, train)
            u_o = gemm(attn_d, L["a_o"], bn=64)
            ext_o = (u_o, L["b_o"])
        x1 = torch.empty_like(x)
        xn2 = torch.empty_like(x)
        rstd2 = torch.empty(x.shape[0], device=x.device, dtype=torch.float32)
        if mlp_cached:
            # every TP rank takes this branch (the cache level is agreed across the group)
            x1 = cache.x1
            C.add_rmsnorm(x1, None, None, lw.ln2, xn2, rstd2, None, None, 1.0, self.eps)
        elif tp == 1:
            gemm(attn, lw.w_o, x1, ext_ab=ext_o, residual=x)
            C.add_rmsnorm(x1, None, None, lw.ln2, xn2, rstd2, None, None, 1.0, self.eps)
        elif self.tp_reducer() is not None:
            # the o_proj GEMM's row chunks go to every rank as they finish; x1 = x + sum
            def o_rows(rows, dst):
                gemm(attn[rows], lw.w_o, dst, ext_ab=(ext_o[0][rows], ext_o[1]) if ext_o else None)

            x1 = self.tp_reducer().gemm_reduce(o_rows, T, scatter=sp, residual=x)
            C.add_rmsnorm(x1, None, None, lw.ln2, xn2, rstd2, None, None, 1.0, self.eps)
        else:
            o = gemm(attn, lw.w_o, ext_ab=ext_o)
            o = _sp_scatter(o, tp_group) if sp else _tp_all_reduce(o, tp_group)
            C.add_rmsnorm(x, o, x1, lw.ln2, xn2, rstd2, None, None, 1.0, self.eps)
        if sp:
            xn2 = _sp_gather(xn2, tp_group)
        ext_gu = None
        if "a_gu" in L:
            xd2 = self._dropout(xn2, "gu", lw.index, seed, train)
            u_gu = gemm(xd2, L["a_gu"], bn=64)
            ext_gu = (u_gu, L["b_gu"])
        keep_mlp = keep is not None and keep.mlp
        if mlp_cached:
            gu, act = cache.gu, cache.act
        else:
            gu = (torch.empty(T, 2 * m.inter_local, device=x.device, dtype=xn2.dtype) if save or keep_mlp
                  else None)
            act = gemm(xn2, lw.w_gu, ext_ab=ext_gu, epilogue="swiglu", aux=gu)
        if keep_mlp:
            keep.x1, keep.gu, keep.act = x1, gu, act
        ext_d = None
        if "a_down" in L:
            act_d = self._dropout(act, "down", lw.index, seed, train)
            u_d = gemm(act_d, L["a_down"], bn=64)
            ext_d = (u_d, L["b_down"])
        if not need_out:
            x2 = None  # every TP rank skips the same GEMM and collective
        elif tp == 1:
            x2 = gemm(act, lw.w_down, ext_ab=ext_d, residual=x1)
        elif self.tp_reducer() is not None:
            def down_rows(rows, dst):
                gemm(act[rows], lw.w_down, dst, ext_ab=(ext_d[0][rows], ext_d[1]) if ext_d else None)

            x2 = self.tp_reducer().gemm_reduce(down_rows, T, scatter=sp, residual=x1)
        else:
            d = gemm(act, lw.w_down, ext_ab=ext_d)
            d = _sp_scatter(d, tp_group) if sp else _tp_all_reduce(d, tp_group)
            x2 = (x1.float() + d.float()).to(x.dtype)
        if save:
            s.x, s.xn, s.rstd1, s.qkv, s.q, s.k, s.v, s.attn = x, xn, rstd1, qkv, q, k, v, attn
            s.x1, s.xn2, s.rstd2, s.gu, s.act, s.attn_ctx = x1, xn2, rstd2, gu, act, ctx
            s.xd = xd if ext_qkv else None
            s.u_qkv = ext_qkv[0] if ext_qkv else None
            s.attn_d = attn_d if ext_o else None
            s.u_o = ext_o[0] if ext_o else None
            s.xd2 = xd2 if ext_gu else None
            s.u_gu = ext_gu[0] if ext_gu else None
            s.act_d = act_d if ext_d else None
            s.u_d = ext_d[0] if ext_d else None
        return x2, s

    # ------------------------------------------------------------ backward
    def _lora_linear_backward(self, dy, w, saved_u, saved_xd, b_ext, a_ext, site, layer, seed, train,
                              reduce: str | None = None):
        """d(input) of y = x W^T + U B^T with U = drop(x) (sA)^T, plus LoRA grads.

        Every operand is read as stored: ``W`` [N, K], ``B`` [N, 64k] and ``sA``
        [64k, K] are the MN-major B operand of ``dy @ W`` / ``dy @ B`` /
        ``du @ sA``, and the gradients contract over tokens with both operands
        MN-major (split-K fp32 atomics), so no transposed copy is made.
        ``reduce`` ("all" or "scatter") sums d(input) over the TP group: on CUDA
        the dgrad runs in row chunks whose results the copy engines send to the
        peers while the next chunk computes (``TPAllReduce.gemm_reduce``), an
        NCCL / gloo collective follows it elsewhere.
        Returns (dx, db_full [N, 64k] fp32, da_full [64k, K] fp32) -- the
        gradient w.r.t. the padded layouts (caller scatters into parameters).
        """
        red = self.tp_reducer() if reduce is not None else None
        du = tmp = None
        if saved_u is not None:
            du = gemm(dy, b_ext, b_mn=True, bn=64)            # [T, 64k]
            if train and self.m.lora.dropout > 0:
                # the LoRA path's dgrad, masked like the forward, enters the
                # frozen dgrad's epilogue as a residual
                tmp = self._dropout(gemm(du, a_ext, b_mn=True), site, layer, seed, train)

        def dgrad_rows(rows, dst):
            if saved_u is None:
                gemm(dy[rows], w, dst, b_mn=True)
            elif tmp is not None:
                gemm(dy[rows], w, dst, b_mn=True, residual=tmp[rows])
            else:
                gemm(dy[rows], w, dst, b_mn=True, ext_ab=(du[rows], a_ext))

        if red is not None:
            # the dgrad's row chunks go to every rank (or their owner) as they finish
            dx = red.gemm_reduce(dgrad_rows, dy.shape[0], scatter=reduce == "scatter")
        else:
            dx = torch.empty(dy.shape[0], w.shape[1], device=dy.device, dtype=dy.dtype)
            dgrad_rows(slice(0, dy.shape[0]), dx)
        del tmp
        db = da = None
        if saved_u is not None:
            n_out, width, k_in = dy.shape[1], saved_u.shape[1], saved_xd.shape[1]
            db = torch.zeros(n_out, width, device=dy.device, dtype=torch.float32)
            gemm(dy, saved_u, db, epilogue="atomic", a_mn=True, b_mn=True, bn=64, splits=_grad_splits(n_out))
            da = torch.zeros(width, k_in, device=dy.device, dtype=torch.float32)
            gemm(saved_xd, du, da, epilogue="atomic", a_mn=True, b_mn=True, bn=64, swap=True,
                 splits=_grad_splits(k_in))
        if red is None and reduce == "scatter":
            dx = _sp_scatter(dx, self.m.ps.tp_group)
        elif red is None and reduce == "all":
            dx = _tp_all_reduce(dx, self.m.ps.tp_group)
        return dx, db, da

    def _scatter_grads(self, layer: int, group: str, db, da) -> None:
        ad = self.m.lora
        r, s = ad.r, ad.scaling
        if group == "qkv":
            rows = [("q", self.m.q_local), ("k", self.m.kv_local), ("v", self.m.kv_local)]
            row = 0
            for slot, (kind, n) in enumerate(rows):
                mod = ad.module(layer, kind)
                if mod is not None:
                    mod.b_grad += db[row : row + n, slot * r : (slot + 1) * r]
                    mod.a_grad += s * da[slot * r : (slot + 1) * r]
                row += n
        elif group == "gu":
            for slot, kind in enumerate(("gate", "up")):
                mod = ad.module(layer, kind)
                if mod is not None:
                    mod.b_grad += db[slot::2, slot * r : (slot + 1) * r]
                    mod.a_grad += s * da[slot * r : (slot + 1) * r]
        else:
            mod = ad.module(layer, group)
            if mod is not None:
                mod.b_grad += db[:, :r]
                mod.a_grad += s * da[:r]

    def layer_backward(self, lw: LayerWeights, s: LayerSaved, dx2: torch.Tensor, meta: AttnMeta, *,
                       train: bool, seed: int) -> torch.Tensor:
        m, C, L = self.m, self.C, self._layouts(lw)
        tp_group = m.ps.tp_group
        li = lw.index
        sp = self.sp
        # --- down projection (SP: its output gradient is gathered over the tokens)
        dy2 = _sp_gather(dx2, tp_group) if sp else dx2
        dact, db, da = self._lora_linear_backward(dy2, lw.w_down, s.u_d, s.act_d, L.get("b_down"),
                                                  L.get("a_down"), "down", li, seed, train)
        if db is not None:
            self._scatter_grads(li, "down", db, da)
        # --- SwiGLU
        dgu = torch.empty_like(s.gu)
        C.swiglu_bwd(s.gu, dact, dgu)
        del dact
        # --- gate/up
        tp_reduce = None if m.ps.tp_size == 1 else ("scatter" if sp else "all")
        dxn2, db, da = self._lora_linear_backward(dgu, lw.w_gu, s.u_gu, s.xd2, L.get("b_gu"), L.get("a_gu"),
                                                  "gu", li, seed, train, reduce=tp_reduce)
        if db is not None:
            self._scatter_grads(li, "gu", db, da)
        del dgu, dy2
        dx1 = torch.empty_like(dx2)
        C.rmsnorm_bwd(dxn2, s.x1, lw.ln2, s.rstd2, dx2, dx1, self.eps)
        # --- o projection
        dy1 = _sp_gather(dx1, tp_group) if sp else dx1
        dattn, db, da = self._lora_linear_backward(dy1, lw.w_o, s.u_o, s.attn_d, L.get("b_o"), L.get("a_o"),
                                                   "o", li, seed, train)
        if db is not None:
            self._scatter_grads(li, "o", db, da)
        # --- attention
        dq, dk, dv = attn_ops.attention_backward(dattn, s.q, s.k, s.v, s.attn, s.attn_ctx, meta, self.scale)
        dqkv = torch.empty_like(s.qkv)
        C.qk_norm_rope_bwd(dq, dk, dv, s.qkv, lw.q_norm, lw.k_norm, m.inv_freq, meta.pos, dqkv, m.nq, m.nkv, self.eps)
        del dq, dk, dv
        # --- qkv projection
        dxn, db, da = self._lora_linear_backward(dqkv, lw.w_qkv, s.u_qkv, s.xd, L.get("b_qkv"), L.get("a_qkv"),
                                                 "qkv", li, seed, train, reduce=tp_reduce)
        if db is not None:
            self._scatter_grads(li, "qkv", db, da)
        dx = torch.empty_like(dx2)
        C.rmsnorm_bwd(dxn, s.x, lw.ln1, s.rstd1, dx1, dx, self.eps)
        return dx

    # ------------------------------------------------------------ stages
    def embed(self, ids: torch.Tensor) -> torch.Tensor:
        out = torch.empty(ids.numel(), self.m.cfg.hidden_size, device=ids.device, dtype=self.m.dtype)
        self.C.embedding(ids.reshape(-1).contiguous(), self.m.embed, out)
        return out

    def attention_cache_bytes(self, tokens: int, level: int = 1) -> int:
        """Device bytes that caching every local layer's values at ``level``
        (1: attention, 2: attention and MLP) costs for ``tokens``."""
        m = self.m
        qkv_w = (m.nq + 2 * m.nkv) * m.D
        per_token = 2 * qkv_w + 2 * m.nq * m.D + 4 * m.nq
        if level >= 2:
            per_token += 2 * (m.cfg.hidden_size + 3 * m.inter_local)
        return len(m.layers) * tokens * per_token

    def _cache_level(self, tokens: int, device: torch.device) -> int:
        """0, 1 or 2 (``GRASPO_CACHE_ATTN``: ``auto`` picks the highest level
        that leaves room for one layer's backward; ``1`` / ``2`` force a level,
        ``0`` disables).  TP ranks agree on the lowest level any of them picked,
        because level 2 skips the row-parallel projections and their collectives."""
        mode = _cache_attention_mode()
        if mode in ("0", "off", "false") or not self.m.layers:
            level = 0
        elif mode in ("1", "on", "true"):
            level = 1
        elif mode in ("2", "full", "mlp"):
            level = 2
        elif device.type != "cuda":
            level = 0
        else:
            free, _ = torch.cuda.mem_get_info(device)
            free += torch.cuda.memory_reserved(device) - torch.cuda.memory_allocated(device)
            m = self.m
            # head-room for one layer's backward: its saved activations and gradients
            per_layer_bwd = tokens * 2 * (6 * m.cfg.hidden_size + 4 * (m.nq + 2 * m.nkv) * m.D + 6 * m.inter_local)
            room = free - 2 * per_layer_bwd - (4 << 30)
            level = 2 if room > self.attention_cache_bytes(tokens, 2) else (
                1 if room > self.attention_cache_bytes(tokens, 1) else 0)
        ps = self.m.ps
        if ps.tp_size > 1 and dist.is_available() and dist.is_initialized():
            t = torch.tensor([level], device=ps.device, dtype=torch.int32)
            dist.all_reduce(t, op=dist.ReduceOp.MIN, group=ps.tp_group)
            level = int(t.item())
        return level

    def _cache_attention(self, tokens: int, device: torch.device) -> bool:
        return self._cache_level(tokens, device) > 0

    def stage_forward(self, x: torch.Tensor, meta: AttnMeta, *, train=False, seed=0, keep_inputs=False):
        """Run this rank's layers; returns (out, [per-layer (input, AttnCache or None)] if keep_inputs).

        With ``keep_inputs`` forward values are kept for the backward's
        recompute when they fit in free device memory (``GRASPO_CACHE_ATTN``:
        ``auto`` (default), ``1`` attention values, ``2`` attention and MLP
        values, ``0`` none; see ``AttnCache``)."""
        inputs = []
        T = x.shape[0] * (self.m.ps.tp_size if self.sp else 1)
        level = self._cache_level(T, x.device) if keep_inputs else 0
        for lw in self.m.layers:
            keep = AttnCache(mlp=level >= 2) if level else None
            x_in = x
            x, _ = self.layer_forward(lw, x, meta, train=train, seed=seed, keep=keep)
            if keep_inputs:
                inputs.append((x_in, keep))
        return x, inputs

    def stage_backward(self, inputs, dout: torch.Tensor, meta: AttnMeta, *, train=True, seed=0,
                       on_layer_done=None):
        """Recompute-and-backprop through this rank's layers; returns d(input).

        ``inputs`` (from ``stage_forward``) is consumed: each layer's entry is
        released once its backward ran.  ``on_layer_done(layer)`` runs after a
        layer's LoRA gradients are complete (the data-parallel gradient push)."""
        g = dout
        for lw in reversed(self.m.layers):
            x, cache = inputs.pop()
            _, saved = self.layer_forward(lw, x, meta, train=train, seed=seed, save=True, cache=cache,
                                          need_out=False)
            del x, cache
            g = self.layer_backward(lw, saved, g, meta, train=train, seed=seed)
            del saved
            if on_layer_done is not None:
                on_layer_done(lw.index)
        if inputs:
            raise ValueError("stage_backward: more saved inputs than local layers")
        return g

    # ------------------------------------------------------------ head
    def final_norm(self, x: torch.Tensor):
        xn = torch.empty_like(x)
        rstd = torch.empty(x.shape[0], device=x.device, dtype=torch.float32)
        self.C.add_rmsnorm(x, None, None, self.m.norm, xn, rstd, None, None, 1.0, self.eps)
        return xn, rstd

    def token_logprobs(self, h: torch.Tensor, targets: torch.Tensor):
        """log p(targets) from normed hidden h [T, H] -> (logp [T], lse [T])."""
        m = self.m
        T = h.shape[0]
        bn = 256
        nblk = (m.vocab_local + bn - 1) // bn
        local_t = (targets - m.vocab_start).contiguous()
        part = torch.empty(T, nblk, 2, device=h.device, dtype=torch.float32)
        tl = torch.zeros(T, device=h.device, dtype=torch.float32)
        gemm(h, m.lm_head, torch.empty(0, device=h.device), epilogue="lse", aux=part.view(T, nblk * 2),
             targets=local_t, tgt_logit=tl, bn=bn)
        red = self.tp_reducer()
        if red is not None:
            # vocab shards merged through peer memory (no library collective)
            lse, logp = red.lse_exchange(part, tl)
            return logp, lse
        lse = torch.empty(T, device=h.device, dtype=torch.float32)
        logp = torch.empty(T, device=h.device, dtype=torch.float32)
        self.C.lse_combine(part, tl, lse, logp)
        group = m.ps.tp_group
        if m.ps.tp_size > 1:
            # merge vocab shards: lse = log sum_r exp(lse_r); target logit lives on one shard
            lses = torch.empty(m.ps.tp_size * T, device=h.device, dtype=torch.float32)
            dist.all_gather_into_tensor(lses, lse.contiguous(), group=group)
            lses = lses.view(m.ps.tp_size, T)
            _tp_all_reduce(tl, group)
            lse = torch.logsumexp(lses, 0)
            logp = tl - lse
        return logp, lse

    def token_logprobs_backward(self, h: torch.Tensor, targets: torch.Tensor, lse: torch.Tensor,
                                g: torch.Tensor, chunk_tokens: int = 32768) -> torch.Tensor:
        """d(normed hidden) for upstream grads g [T] of the selected log-probs.

        ``h`` holds every token; with SP the result is this rank's token shard
        (reduce-scattered instead of all-reduced over the vocabulary shards)."""
        m = self.m
        T, H = h.shape
        dh = torch.empty_like(h)
        local_t = (targets - m.vocab_start).contiguous()
        # without SP the vocab shards' partial d(hidden) are summed by the fused
        # GEMM + all-reduce, chunk by chunk
        red = self.tp_reducer() if not self.sp else None
        for t0 in range(0, T, chunk_tokens):
            t1 = min(T, t0 + chunk_tokens)
            dlog = gemm(h[t0:t1], m.lm_head, epilogue="softmax_grad", targets=local_t[t0:t1],
                        row_lse=lse[t0:t1].contiguous(), row_scale=g[t0:t1].contiguous())
            if red is not None:
                red.gemm_reduce(lambda rows, dst: gemm(dlog[rows], m.lm_head, dst, b_mn=True), t1 - t0,
                                out=dh[t0:t1])
            else:
                gemm(dlog, m.lm_head, dh[t0:t1], b_mn=True)
            del dlog
        if red is not None:
            return dh
        if self.sp:
            return _sp_scatter(dh, m.ps.tp_group)
        _tp_all_reduce(dh, m.ps.tp_group)
        return dh
