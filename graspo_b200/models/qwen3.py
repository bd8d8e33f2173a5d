"""Qwen3 dense decoder: weight container + eager (autograd) execution.

Architecture (reference: models/common/layers_qwen3.py:24-351, qwen3/model.py):
embedding -> N x [RMSNorm -> q/k/v (GQA) -> per-head QK RMSNorm -> RoPE ->
causal attention -> o_proj -> residual -> RMSNorm -> SwiGLU MLP -> residual]
-> final RMSNorm -> LM head.

Weights are stored in the layouts the sm_100a kernels consume:

* ``w_qkv [q_local + 2*kv_local, H]`` -- q, k, v rows of this TP rank stacked,
* ``w_o [H, q_local]``, ``w_down [H, I_local]`` -- row-parallel shards,
* ``w_gu [2*I_local, H]`` -- gate and up rows *interleaved* (row 2j = gate j,
  row 2j+1 = up j) so one GEMM tile holds matching pairs and SwiGLU runs in
  its epilogue,
* ``lm_head [V_local, H]`` -- vocab-parallel: each TP rank holds V/tp rows
  (the reference replicates the full head on every rank),
* transposed copies (``*_t``) for the backward pass, built on demand: base
  weights are frozen, and 180 GB of HBM makes a K-major copy cheaper than a
  transposing GEMM.

The eager executor below is plain PyTorch (any device / dtype) and serves as
the oracle for the fused path and as the CPU/gloo execution path.
"""

from __future__ import annotations

import math
from dataclasses import dataclass

import torch
import torch.nn.functional as F

from graspo_b200.core.lora_targets import lora_target_enabled
from graspo_b200.models.config import DecoderConfig
from graspo_b200.models.loader import SafetensorIndex, shard_bounds
from graspo_b200.models.lora import LoRAAdapter, LoRAModule
from graspo_b200.parallel.state import ParallelState
from graspo_b200.parallel.tp import copy_to_tp, reduce_from_tp

KINDS = ("q", "k", "v", "o", "gate", "up", "down")
_TARGET = {
    "q": "language.self_attn.q_proj",
    "k": "language.self_attn.k_proj",
    "v": "language.self_attn.v_proj",
    "o": "language.self_attn.o_proj",
    "gate": "language.mlp.gate_proj",
    "up": "language.mlp.up_proj",
    "down": "language.mlp.down_proj",
}
_MODULE = {
    "q": "self_attn.q_proj",
    "k": "self_attn.k_proj",
    "v": "self_attn.v_proj",
    "o": "self_attn.o_proj",
    "gate": "mlp.gate_proj",
    "up": "mlp.up_proj",
    "down": "mlp.down_proj",
}


@dataclass
class LayerWeights:
    index: int
    ln1: torch.Tensor
    ln2: torch.Tensor
    q_norm: torch.Tensor
    k_norm: torch.Tensor
    w_qkv: torch.Tensor
    w_o: torch.Tensor
    w_gu: torch.Tensor
    w_down: torch.Tensor
    # the same weights followed by spare rows holding a LoRA A factor (decode
    # GEMMs compute W x and s A x in one pass); w_qkv / w_o / w_down are views
    w_qkv_ext: torch.Tensor | None = None
    w_o_ext: torch.Tensor | None = None
    w_down_ext: torch.Tensor | None = None


class Qwen3Model:
    """Weights and LoRA state of the layers placed on this rank."""

    supports_kv_cache = True

    def __init__(
        self,
        cfg: DecoderConfig,
        loader: SafetensorIndex,
        *,
        ps: ParallelState,
        local_layers: list[int] | None = None,
        include_embed: bool = True,
        include_head: bool = True,
        lora_targets: set[str] | frozenset[str] = frozenset(),
        lora_r: int = 16,
        lora_alpha: float = 32,
        lora_dropout: float = 0.0,
        dtype: torch.dtype = torch.bfloat16,
        device: torch.device | None = None,
        seed: int = 42,
        gradient_checkpointing: bool = True,
    ) -> None:
        self.cfg = cfg
        self.ps = ps
        self.device = device or ps.device
        self.dtype = dtype
        self.gradient_checkpointing = gradient_checkpointing
        tp, tr = ps.tp_size, ps.tp_rank
        if cfg.num_attention_heads % tp or cfg.num_key_value_heads % tp:
            raise ValueError("attention heads and KV heads must be divisible by the TP size")
        if cfg.intermediate_size % tp or cfg.vocab_size % tp:
            raise ValueError("intermediate size and vocab size must be divisible by the TP size")
        self.nq = cfg.num_attention_heads // tp
        self.nkv = cfg.num_key_value_heads // tp
        self.D = cfg.head_dim
        self.q_local = self.nq * self.D
        self.kv_local = self.nkv * self.D
        self.inter_local = cfg.intermediate_size // tp
        self.vocab_local = cfg.vocab_size // tp
        self.vocab_start = tr * self.vocab_local
        self.local_layers = list(range(cfg.num_hidden_layers)) if local_layers is None else list(local_layers)
        self.include_embed = include_embed
        self.include_head = include_head
        self.lora_targets = set(lora_targets)
        pre = cfg.key_prefix
        dev, dt = self.device, dtype

        def load(name: str) -> torch.Tensor:
            return loader.get(name).to(device=dev, dtype=dt)

        def rows(name: str, a: int, b: int) -> torch.Tensor:
            return loader.get_rows(name, a, b).to(device=dev, dtype=dt)

        def cols(name: str, a: int, b: int) -> torch.Tensor:
            return loader.get_cols(name, a, b).to(device=dev, dtype=dt)

        self.embed = load(f"{pre}.embed_tokens.weight") if include_embed else None
        # frozen vision tower on the stage that embeds the tokens; every stage
        # keeps its config (image grids give placeholder counts and positions)
        self.vision = self.vision_cfg = None
        if cfg.has_vision:
            from graspo_b200.models.vision import VisionConfig, VisionTower

            vc = dict(cfg.extra["vision_config"])
            vc.setdefault("out_hidden_size", cfg.hidden_size)
            self.vision_cfg = VisionConfig.from_dict(vc)
            if include_embed:
                self.vision = VisionTower(self.vision_cfg, loader, "model.visual", dtype=dtype, device=self.device)
        self.layers: list[LayerWeights] = []
        modules: list[LoRAModule] = []
        H = cfg.hidden_size
        q0, q1 = shard_bounds(cfg.q_size, tr, tp)
        k0, k1 = shard_bounds(cfg.kv_size, tr, tp)
        i0, i1 = shard_bounds(cfg.intermediate_size, tr, tp)
        for idx in self.local_layers:
            p = f"{pre}.layers.{idx}"
            wq = rows(f"{p}.self_attn.q_proj.weight", q0, q1)
            wk = rows(f"{p}.self_attn.k_proj.weight", k0, k1)
            wv = rows(f"{p}.self_attn.v_proj.weight", k0, k1)
            wg = rows(f"{p}.mlp.gate_proj.weight", i0, i1)
            wu = rows(f"{p}.mlp.up_proj.weight", i0, i1)
            for bias in ("q_proj", "k_proj", "v_proj", "o_proj"):
                if loader.has(f"{p}.self_attn.{bias}.bias"):
                    raise ValueError("attention biases are not supported by this decoder")
            qn = loader.get_optional(f"{p}.self_attn.q_norm.weight")
            kn = loader.get_optional(f"{p}.self_attn.k_norm.weight")
            layer = LayerWeights(
                index=idx,
                ln1=load(f"{p}.input_layernorm.weight"),
                ln2=load(f"{p}.post_attention_layernorm.weight"),
                q_norm=(qn.to(dev, dt) if qn is not None else torch.ones(self.D, device=dev, dtype=dt)),
                k_norm=(kn.to(dev, dt) if kn is not None else torch.ones(self.D, device=dev, dtype=dt)),
                w_qkv=torch.cat([wq, wk, wv], 0).contiguous(),
                w_o=cols(f"{p}.self_attn.o_proj.weight", q0, q1).contiguous(),
                w_gu=torch.stack([wg, wu], 1).reshape(2 * self.inter_local, H).contiguous(),
                w_down=cols(f"{p}.mlp.down_proj.weight", i0, i1).contiguous(),
            )
            del wq, wk, wv, wg, wu
            self.layers.append(layer)
            for kind in KINDS:
                target = _TARGET[kind]
                if not lora_target_enabled(self.lora_targets, target):
                    continue
                col = kind in ("o", "down")
                in_full = {"o": cfg.q_size, "down": cfg.intermediate_size}.get(kind, H)
                out_full = {"q": cfg.q_size, "k": cfg.kv_size, "v": cfg.kv_size, "gate": cfg.intermediate_size,
                            "up": cfg.intermediate_size}.get(kind, H)
                mod = LoRAModule(
                    module_name=f"layers.{idx}.{_MODULE[kind]}",
                    target_name=target,
                    hf_module_path=f"{p}.{_MODULE[kind]}",
                    layer=idx,
                    kind=kind,
                    shard_kind="in" if col else "out",
                    in_full=in_full,
                    out_full=out_full,
                    in_local=in_full // tp if col else in_full,
                    out_local=out_full if col else out_full // tp,
                )
                if col:
                    mod.col_start, mod.col_stop = shard_bounds(in_full, tr, tp)
                else:
                    mod.row_start, mod.row_stop = shard_bounds(out_full, tr, tp)
                modules.append(mod)
        if include_head:
            self.norm = load(f"{pre}.norm.weight")
            name = "lm_head.weight" if loader.has("lm_head.weight") else f"{pre}.embed_tokens.weight"
            self.lm_head = rows(name, self.vocab_start, self.vocab_start + self.vocab_local).contiguous()
        else:
            self.norm = None
            self.lm_head = None
        if self.vision is not None:
            from graspo_b200.models.vision import vision_lora_modules

            modules += vision_lora_modules(self.vision.cfg, self.lora_targets)
        self.lora = LoRAAdapter(
            modules, r=lora_r, alpha=lora_alpha, dropout=lora_dropout, device=dev, seed=seed, tp_rank=tr
        )
        inv = 1.0 / (cfg.rope_theta ** (torch.arange(0, self.D, 2, dtype=torch.float32) / self.D))
        self.inv_freq = inv.to(dev)
        self.sizes = {"hidden": H, "q": self.q_local, "kv": self.kv_local, "inter": self.inter_local}

    # ------------------------------------------------------------------ misc
    def layer_by_index(self, idx: int) -> LayerWeights:
        return self.layers[self.local_layers.index(idx)]

    def ensure_transposed(self) -> None:
        """Kept for callers of earlier versions: backward GEMMs read every weight
        MN-major as stored, so no transposed copies are built."""
        return None

    def ensure_tail_rows(self, tails: dict[str, int]) -> None:
        """Give ``w_qkv`` / ``w_o`` / ``w_down`` ``tails[name]`` spare rows.

        The weight moves into a buffer of ``rows + tail`` rows; the layer keeps
        a view of the first ``rows`` (so every other user is unaffected) and
        ``<name>_ext`` names the whole buffer.  The rollout engine writes the
        scaled LoRA A factor into the spare rows before decoding.
        """
        for lw in self.layers:
            for name, tail in tails.items():
                ext = getattr(lw, f"{name}_ext")
                w = getattr(lw, name)
                if tail <= 0 or (ext is not None and ext.shape[0] == w.shape[0] + tail):
                    continue
                buf = torch.zeros(w.shape[0] + tail, w.shape[1], device=w.device, dtype=w.dtype)
                buf[: w.shape[0]].copy_(w)
                setattr(lw, name, buf[: w.shape[0]])
                setattr(lw, f"{name}_ext", buf)
                del w

    def estimate_kv_cache_bytes(self, *, batch_size: int, sequence_len: int) -> int:
        return batch_size * len(self.local_layers) * 2 * self.nkv * self.D * sequence_len * self.dtype.itemsize

    def lora_state_dict(self) -> dict[str, torch.Tensor]:
        return self.lora.state_dict()

    def lora_tensor_metadata(self) -> list[dict]:
        return self.lora.metadata()

    def lora_target_signature(self) -> dict[str, object]:
        return self.lora.signature()

    def enabled_lora_target_names(self) -> tuple[str, ...]:
        return self.lora.target_names()


# ====================================================================== eager
def position_ids_from_mask(mask: torch.Tensor) -> torch.Tensor:
    """Rope positions: index among the valid tokens of the row (pads get 0)."""
    pos = mask.long().cumsum(-1) - 1
    return pos.masked_fill(~mask.bool(), 0)


def rmsnorm(x: torch.Tensor, w: torch.Tensor, eps: float) -> torch.Tensor:
    xf = x.float()
    return (xf * torch.rsqrt(xf.pow(2).mean(-1, keepdim=True) + eps) * w.float()).to(x.dtype)


def apply_rope(x: torch.Tensor, pos: torch.Tensor, inv_freq: torch.Tensor) -> torch.Tensor:
    """Rotate-half RoPE; x [..., S, heads, D], pos [..., S]."""
    freqs = pos.float()[..., None] * inv_freq
    emb = torch.cat([freqs, freqs], -1)[..., None, :]
    cos, sin = emb.cos(), emb.sin()
    half = x.shape[-1] // 2
    xf = x.float()
    rot = torch.cat([-xf[..., half:], xf[..., :half]], -1)
    return (xf * cos + rot * sin).to(x.dtype)


def masked_attention(q, k, v, key_mask, scale):
    """q [B,S,nq,D], k/v [B,S,nkv,D], key_mask [B,S] -> [B,S,nq*D]; causal.

    Query rows with no valid key (left padding) produce zeros.
    """
    B, S, nq, D = q.shape
    nkv = k.shape[2]
    rep = nq // nkv
    qf = q.float().transpose(1, 2)
    kf = k.float().transpose(1, 2).repeat_interleave(rep, 1)
    vf = v.float().transpose(1, 2).repeat_interleave(rep, 1)
    scores = (qf @ kf.transpose(-1, -2)) * scale
    causal = torch.ones(S, S, dtype=torch.bool, device=q.device).tril()
    allowed = causal[None, None] & key_mask.bool()[:, None, None, :]
    scores = scores.masked_fill(~allowed, float("-inf"))
    probs = torch.softmax(scores, -1)
    probs = torch.nan_to_num(probs, nan=0.0)
    out = probs @ vf
    return out.transpose(1, 2).reshape(B, S, nq * D).to(q.dtype)


class EagerLoRA:
    """Autograd leaves sharing storage with the adapter's fp32 master weights."""

    def __init__(self, adapter: LoRAAdapter, requires_grad: bool) -> None:
        self.adapter = adapter
        self.leaves: dict[str, tuple[torch.Tensor, torch.Tensor]] = {}
        for m in adapter.modules:
            a = m.a.detach().requires_grad_(requires_grad)
            b = m.b.detach().requires_grad_(requires_grad)
            self.leaves[m.module_name] = (a, b)

    def accumulate_grads(self) -> None:
        for m in self.adapter.modules:
            a, b = self.leaves[m.module_name]
            if a.grad is not None:
                m.a_grad.add_(a.grad)
            if b.grad is not None:
                m.b_grad.add_(b.grad)


def _linear_lora(x, w, mod: LoRAModule | None, lora: EagerLoRA | None, scaling, dropout, training):
    y = F.linear(x, w)
    if mod is None or lora is None:
        return y
    a, b = lora.leaves[mod.module_name]
    xin = F.dropout(x, dropout, training) if (training and dropout > 0) else x
    delta = F.linear(F.linear(xin.to(a.dtype), a), b) * scaling
    return y + delta.to(y.dtype)


def eager_layer(model: Qwen3Model, lw: LayerWeights, x, pos, key_mask, lora: EagerLoRA | None, training: bool):
    """One decoder layer, [B, S, H] -> [B, S, H] (TP-aware, no KV cache)."""
    cfg = model.cfg
    ad = model.lora
    group = model.ps.tp_group
    B, S, H = x.shape
    mod = {k: ad.module(lw.index, k) for k in KINDS}
    h = copy_to_tp(rmsnorm(x, lw.ln1, cfg.rms_norm_eps), group)
    q_end, k_end = model.q_local, model.q_local + model.kv_local
    q = _linear_lora(h, lw.w_qkv[:q_end], mod["q"], lora, ad.scaling, ad.dropout, training)
    k = _linear_lora(h, lw.w_qkv[q_end:k_end], mod["k"], lora, ad.scaling, ad.dropout, training)
    v = _linear_lora(h, lw.w_qkv[k_end:], mod["v"], lora, ad.scaling, ad.dropout, training)
    q = rmsnorm(q.view(B, S, model.nq, model.D), lw.q_norm, cfg.rms_norm_eps)
    k = rmsnorm(k.view(B, S, model.nkv, model.D), lw.k_norm, cfg.rms_norm_eps)
    q = apply_rope(q, pos, model.inv_freq)
    k = apply_rope(k, pos, model.inv_freq)
    attn = masked_attention(q, k, v.view(B, S, model.nkv, model.D), key_mask, 1.0 / math.sqrt(model.D))
    o = _linear_lora(attn, lw.w_o, mod["o"], lora, ad.scaling, ad.dropout, training)
    x = x + reduce_from_tp(o, group)
    h2 = copy_to_tp(rmsnorm(x, lw.ln2, cfg.rms_norm_eps), group)
    g = _linear_lora(h2, lw.w_gu[0::2], mod["gate"], lora, ad.scaling, ad.dropout, training)
    u = _linear_lora(h2, lw.w_gu[1::2], mod["up"], lora, ad.scaling, ad.dropout, training)
    d = _linear_lora(F.silu(g) * u, lw.w_down, mod["down"], lora, ad.scaling, ad.dropout, training)
    return x + reduce_from_tp(d, group)


def eager_stage_forward(
    model: Qwen3Model,
    inputs: torch.Tensor,
    attention_mask: torch.Tensor,
    *,
    lora: EagerLoRA | None = None,
    training: bool = False,
    embed_hook=None,
) -> torch.Tensor:
    """Token ids (first stage) or hidden states -> hidden states after local layers.

    The adapter is always applied; pass ``lora`` (with ``requires_grad``) to
    collect its gradients.  ``embed_hook(ids, x)`` may edit the token
    embeddings in place (image features).
    """
    if lora is None:
        lora = EagerLoRA(model.lora, requires_grad=False)
    if model.include_embed:
        x = F.embedding(inputs, model.embed)
        if embed_hook is not None:
            x = embed_hook(inputs, x.reshape(-1, x.shape[-1]).clone()).view_as(x)
    else:
        x = inputs
    pos = position_ids_from_mask(attention_mask)
    for lw in model.layers:
        if training and model.gradient_checkpointing and torch.is_grad_enabled():
            x = torch.utils.checkpoint.checkpoint(
                eager_layer, model, lw, x, pos, attention_mask, lora, training, use_reentrant=False
            )
        else:
            x = eager_layer(model, lw, x, pos, attention_mask, lora, training)
    return x


class _VocabParallelLogProb(torch.autograd.Function):
    """log softmax(h W^T)[y] with W split by vocabulary over the TP group."""

    @staticmethod
    def forward(ctx, h, w_local, targets, vocab_start, group, chunk):
        T = h.shape[0]
        hf = h.float()
        wf = w_local.float()
        V = wf.shape[0]
        local_max = torch.full((T,), float("-inf"), device=h.device)
        for c0 in range(0, V, chunk):
            local_max = torch.maximum(local_max, (hf @ wf[c0 : c0 + chunk].T).amax(-1))
        gmax = local_max.clone()
        if group is not None and torch.distributed.is_initialized() and torch.distributed.get_world_size(group) > 1:
            torch.distributed.all_reduce(gmax, op=torch.distributed.ReduceOp.MAX, group=group)
        sumexp = torch.zeros(T, device=h.device)
        for c0 in range(0, V, chunk):
            sumexp += torch.exp(hf @ wf[c0 : c0 + chunk].T - gmax[:, None]).sum(-1)
        local_t = targets - vocab_start
        in_shard = (local_t >= 0) & (local_t < V)
        idx = local_t.clamp(0, V - 1)
        tgt_logit = (hf * wf[idx]).sum(-1) * in_shard
        if group is not None and torch.distributed.is_initialized() and torch.distributed.get_world_size(group) > 1:
            torch.distributed.all_reduce(sumexp, group=group)
            torch.distributed.all_reduce(tgt_logit, group=group)
        lse = gmax + sumexp.log()
        ctx.save_for_backward(h, w_local, targets, lse)
        ctx.vocab_start, ctx.chunk = vocab_start, chunk
        return tgt_logit - lse

    @staticmethod
    def backward(ctx, grad):
        h, w_local, targets, lse = ctx.saved_tensors
        hf, wf = h.float(), w_local.float()
        V = wf.shape[0]
        dh = torch.zeros_like(hf)
        local_t = targets - ctx.vocab_start
        for c0 in range(0, V, ctx.chunk):
            wc = wf[c0 : c0 + ctx.chunk]
            p = torch.exp(hf @ wc.T - lse[:, None])
            onehot = (local_t[:, None] == torch.arange(c0, c0 + wc.shape[0], device=h.device)[None]).float()
            dh += (grad[:, None] * (onehot - p)) @ wc
        return dh.to(h.dtype), None, None, None, None, None


def eager_token_logprobs(model: Qwen3Model, hidden: torch.Tensor, targets: torch.Tensor, chunk: int = 32768):
    """Selected-token log-probs of ``targets`` from final-layer hidden states.

    hidden [B, S, H] (before the final norm), targets [B, S] -> [B, S] fp32.
    """
    B, S, H = hidden.shape
    h = copy_to_tp(rmsnorm(hidden, model.norm, model.cfg.rms_norm_eps), model.ps.tp_group)
    out = _VocabParallelLogProb.apply(
        h.reshape(B * S, H), model.lm_head, targets.reshape(-1), model.vocab_start, model.ps.tp_group, chunk
    )
    return out.view(B, S)


def eager_sequence_logprobs(model: Qwen3Model, sequences, attention_mask, *, lora=None, training=False):
    """log p(sequences[:, 1:]) under the model, [B, S-1] fp32 (single-stage model)."""
    hidden = eager_stage_forward(model, sequences, attention_mask, lora=lora, training=training)
    return eager_token_logprobs(model, hidden[:, :-1], sequences[:, 1:])
