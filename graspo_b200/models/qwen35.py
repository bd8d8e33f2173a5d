"""Qwen3.5 / 3.6 hybrid decoder (``qwen3_5_text``): gated DeltaNet + gated attention.

Layer kinds come from ``layer_types`` (reference:
backends/graspoflow/models/common/layers.py:31-133):

* ``linear_attention`` -- Gated DeltaNet (Yang, Kautz, Hatamizadeh 2024):
  ``in_proj_qkv`` -> causal depthwise conv1d (kernel K) + SiLU -> split q, k, v;
  q, k L2-normalised per head (q also scaled by 1/sqrt(d_k)); per head a
  decay ``g = -exp(A_log) * softplus(a + dt_bias)`` and a write strength
  ``beta = sigmoid(b)``; the state S [d_k, d_v] evolves as
  ``S <- exp(g) S;  S <- S + k (beta (v - S^T k))^T;  o = S^T q``; the output
  passes a gated RMSNorm with ``z = in_proj_z(x)`` (``w * norm(o) * silu(z)``)
  and ``out_proj`` (reference layers.py:358-633, tensor_utils.py:509-646).
* ``full_attention`` -- ``q_proj`` emits (query, gate) per head; QK-norm,
  partial rotary embedding, GQA attention, output ``o * sigmoid(gate)`` into
  ``o_proj`` (layers.py:145-355).

RMSNorms use the ``(1 + w)`` parametrisation (layers.py:636-651); the MLP is
SwiGLU.  The whole-sequence DeltaNet uses the chunked form (chunk 64): the
in-chunk triangular system is solved with one batched ``solve_triangular``
(not a loop over rows), the chunks are chained by the recurrent state.  The
one-token decode step of the recurrence runs in the ``gated_delta_step``
kernel on GPUs.  LoRA is applied on the reference's targets
(``language.full_attn.*``, ``language.linear_attn.{q,k,v}_proj`` (row blocks of
``in_proj_qkv``), ``in_proj_z``, ``out_proj``, ``language.mlp.*``).  Heads
are split over the tensor-parallel group (``Qwen35Model``).
"""

from __future__ import annotations

import math
from dataclasses import dataclass, field

import torch
import torch.distributed as dist
import torch.nn.functional as F

from graspo_b200.core.lora_targets import lora_target_enabled
from graspo_b200.models.config import DecoderConfig
from graspo_b200.models.loader import SafetensorIndex
from graspo_b200.models.lora import LoRAAdapter, LoRAModule
from graspo_b200.models.qwen3 import EagerLoRA
from graspo_b200.ops.hybrid import conv_silu, sigmoid_gate
from graspo_b200.parallel.state import ParallelState
from graspo_b200.parallel.tp import copy_to_tp, reduce_from_tp

CHUNK = 64


def norm1p(x: torch.Tensor, w: torch.Tensor, eps: float) -> torch.Tensor:
    """RMSNorm with the (1 + w) weight, fp32 statistics."""
    xf = x.float()
    y = xf * torch.rsqrt(xf.pow(2).mean(-1, keepdim=True) + eps)
    return (y * (1.0 + w.float())).to(x.dtype)


def _valid_span_start(mask: torch.Tensor) -> torch.Tensor | None:
    """Per row, the first valid position when each row's valid tokens are one
    contiguous span (None otherwise, or when a row has none)."""
    B, S = mask.shape
    lens = mask.sum(1)
    start = mask.int().argmax(1)
    ar = torch.arange(S, device=mask.device)
    span = (ar[None] >= start[:, None]) & (ar[None] < (start + lens)[:, None])
    if not bool(torch.equal(span, mask.bool()) and (lens > 0).all()):
        return None
    return start


def gated_norm(x: torch.Tensor, z: torch.Tensor, w: torch.Tensor, eps: float) -> torch.Tensor:
    """w * rmsnorm(x) * silu(z); one kernel each way on CUDA (graspo_b200/ops/hybrid.py)."""
    from graspo_b200.ops.hybrid import gated_rmsnorm

    return gated_rmsnorm(x, z, w, eps)


def l2norm(x: torch.Tensor, eps: float = 1e-6) -> torch.Tensor:
    return x / x.norm(dim=-1, keepdim=True).clamp_min(eps)


def chunk_gated_delta(q, k, v, g, beta, state=None):
    """Whole-sequence gated delta rule. q, k [B, S, h, dk]; v [B, S, h, dv];
    g, beta [B, S, h] (g = log decay).  q, k must be L2-normalised and q scaled.
    Returns (o [B, S, h, dv], final state [B, h, dk, dv]); fp32 math."""
    B, S, h, dk = k.shape
    dv = v.shape[-1]
    pad = (-S) % CHUNK
    q, k, v, g, beta = (t.float().transpose(1, 2) for t in (q, k, v, g, beta))   # [B, h, S, .]
    if pad:
        q, k, v = (F.pad(t, (0, 0, 0, pad)) for t in (q, k, v))
        g, beta = F.pad(g, (0, pad)), F.pad(beta, (0, pad))
    n = (S + pad) // CHUNK
    q, k, v = (t.reshape(B, h, n, CHUNK, t.shape[-1]) for t in (q, k, v))
    g = g.reshape(B, h, n, CHUNK).cumsum(-1)                                      # within-chunk cumulative log decay
    beta = beta.reshape(B, h, n, CHUNK)
    idx = torch.arange(CHUNK, device=q.device)
    lower = idx[:, None] > idx[None, :]
    decay = torch.exp((g[..., :, None] - g[..., None, :]).masked_fill(~(idx[:, None] >= idx[None, :]), -math.inf))
    kb = k * beta[..., None]
    # W-representation: (I + strictly-lower(beta K K^T . decay)) u = beta v, w likewise for k exp(g)
    A = (kb @ k.transpose(-1, -2)) * decay
    A = A.masked_fill(~lower, 0.0) + torch.eye(CHUNK, device=q.device)
    rhs = torch.cat([v * beta[..., None], kb * g.exp()[..., None]], -1)
    sol = torch.linalg.solve_triangular(A, rhs, upper=False, unitriangular=True)
    u, w = sol[..., :dv], sol[..., dv:]
    S_t = torch.zeros(B, h, dk, dv, device=q.device, dtype=torch.float32) if state is None else state.float()
    attn = (q @ k.transpose(-1, -2)) * decay                                      # [B, h, n, C, C] (causal)
    # Everything that does not depend on the carried state is computed for all
    # chunks at once; the loop over chunks keeps only the state recurrence, as
    # five batched products per chunk over the (batch, head) pairs.
    BH = B * h
    last = g[..., -1]                                                             # [B, h, n] log decay of a chunk
    qg = (q * g.exp()[..., None]).reshape(BH, n, CHUNK, dk)                       # queries decayed to chunk start
    kd = (k * (last[..., None] - g).exp()[..., None]).transpose(-1, -2).reshape(BH, n, dk, CHUNK)
    el = last.exp().reshape(BH, n, 1, 1)
    u, w, attn = u.reshape(BH, n, CHUNK, dv), w.reshape(BH, n, CHUNK, dk), attn.reshape(BH, n, CHUNK, CHUNK)
    S_t = S_t.reshape(BH, dk, dv)
    # unbind (one stack in the backward) rather than indexing chunk c of each
    # tensor, whose backward would fill and add a full-size gradient per chunk
    u, w, attn, qg, kd, el = (t.unbind(1) for t in (u, w, attn, qg, kd, el))
    outs = []
    for c in range(n):
        u_c = torch.baddbmm(u[c], w[c], S_t, alpha=-1.0)                          # new values after the state
        outs.append(torch.baddbmm(torch.bmm(attn[c], u_c), qg[c], S_t))
        S_t = torch.baddbmm(S_t * el[c], kd[c], u_c)
    o = torch.stack(outs, 1).reshape(B, h, n * CHUNK, dv)[:, :, :S]
    return o.transpose(1, 2), S_t.reshape(B, h, dk, dv)


def recurrent_gated_delta(q, k, v, g, beta, state):
    """One-token step (PyTorch): q, k [B, h, dk]; v [B, h, dv]; g, beta [B, h]; state [B, h, dk, dv] (updated)."""
    state.mul_(g.float().exp()[..., None, None])
    mem = (state * k.float()[..., None]).sum(-2)
    delta = (v.float() - mem) * beta.float()[..., None]
    state.add_(k.float()[..., None] * delta[..., None, :])
    return (state * q.float()[..., None]).sum(-2)


@dataclass
class HybridLayer:
    index: int
    kind: str
    ln1: torch.Tensor
    ln2: torch.Tensor
    w: dict[str, torch.Tensor] = field(default_factory=dict)


_TARGETS = {
    "fq": ("language.full_attn.q_proj", "self_attn.q_proj"),
    "fk": ("language.full_attn.k_proj", "self_attn.k_proj"),
    "fv": ("language.full_attn.v_proj", "self_attn.v_proj"),
    "fo": ("language.full_attn.o_proj", "self_attn.o_proj"),
    "lq": ("language.linear_attn.q_proj", "linear_attn.in_proj_qkv"),
    "lk": ("language.linear_attn.k_proj", "linear_attn.in_proj_qkv"),
    "lv": ("language.linear_attn.v_proj", "linear_attn.in_proj_qkv"),
    "lz": ("language.linear_attn.in_proj_z", "linear_attn.in_proj_z"),
    "lo": ("language.linear_attn.out_proj", "linear_attn.out_proj"),
    "gate": ("language.mlp.gate_proj", "mlp.gate_proj"),
    "up": ("language.mlp.up_proj", "mlp.up_proj"),
    "down": ("language.mlp.down_proj", "mlp.down_proj"),
}


class Qwen35Model:
    """Weights and LoRA state of the hybrid decoder, sharded over the TP group.

    Tensor parallelism splits heads (reference: models/common/layers.py:145-633):
    full attention keeps ``nq/tp`` query heads (their query+gate rows of
    ``q_proj``) and ``nkv/tp`` key/value heads (when TP is a multiple of
    ``nkv`` above it: the one head its query heads read, copied on ``tp/nkv``
    ranks, whose LoRA B gradients ``sync_partial_grads`` sums), DeltaNet keeps ``lk/tp`` key
    heads and ``lv/tp`` value heads (rows of ``in_proj_qkv`` in each of its
    q / k / v blocks, the matching conv channels, rows of ``in_proj_z/b/a``,
    ``dt_bias``, ``A_log``), the MLP keeps ``I/tp`` intermediate rows;
    ``o_proj`` / ``out_proj`` / ``down_proj`` keep the matching input columns
    and their outputs are summed over the group.  Embedding, norms and LM head
    are replicated.  LoRA shard kinds follow the reference checkpoint format:
    ``rows`` for head-row selections (A replicated), ``out`` for
    ``in_proj_z`` / gate / up, ``in`` for the row-parallel projections (B
    replicated).
    """

    supports_kv_cache = True

    def __init__(self, cfg: DecoderConfig, loader: SafetensorIndex, *, ps: ParallelState,
                 local_layers: list[int] | None = None, include_embed: bool = True, include_head: bool = True,
                 lora_targets=frozenset(), lora_r: int = 8, lora_alpha: float = 16, lora_dropout: float = 0.0,
                 dtype: torch.dtype = torch.bfloat16, device: torch.device = torch.device("cpu"), seed: int = 42,
                 gradient_checkpointing: bool = True) -> None:
        t = cfg.extra["text_config"]
        self.cfg, self.ps, self.dtype, self.device = cfg, ps, dtype, device
        self.gradient_checkpointing = gradient_checkpointing
        self.local_layers = list(range(cfg.num_hidden_layers)) if local_layers is None else list(local_layers)
        self.include_embed, self.include_head = include_embed, include_head
        self.lora_targets = frozenset(lora_targets)
        self.nq, self.nkv, self.D = cfg.num_attention_heads, cfg.num_key_value_heads, cfg.head_dim
        rp = dict(t.get("rope_parameters") or {})
        self.rotary_dim = int(self.D * float(rp.get("partial_rotary_factor", t.get("partial_rotary_factor", 1.0))))
        theta = float(rp.get("rope_theta", t.get("rope_theta", 1e6)))
        self.inv_freq = (1.0 / theta ** (torch.arange(0, self.rotary_dim, 2, dtype=torch.float32) / self.rotary_dim)
                         ).to(device)
        # interleaved multimodal RoPE: frequency j follows the height position if j % 3 == 1 and
        # j < 3 * sections[1], the width position if j % 3 == 2 and j < 3 * sections[2], else time
        sec = [int(v) for v in (rp.get("mrope_section") or (11, 11, 10))]
        j = torch.arange(self.rotary_dim // 2)
        comp = torch.zeros_like(j)
        comp[(j % 3 == 1) & (j < 3 * sec[1])] = 1
        comp[(j % 3 == 2) & (j < 3 * sec[2])] = 2
        self.mrope_component = comp.to(device)
        self.lk_heads, self.lv_heads = int(t["linear_num_key_heads"]), int(t["linear_num_value_heads"])
        self.dk, self.dv = int(t["linear_key_head_dim"]), int(t["linear_value_head_dim"])
        self.conv_k = int(t["linear_conv_kernel_dim"])
        self.key_dim, self.value_dim = self.lk_heads * self.dk, self.lv_heads * self.dv
        tp, tr = ps.tp_size, ps.tp_rank
        self.tp_group = ps.tp_group if tp > 1 else None
        # key/value heads: split when TP divides them, else each rank keeps the one head its query
        # heads read and the tp/nkv ranks of a group hold copies (reference: layers.py:182-188)
        self.kv_replicas = tp // self.nkv if (tp > self.nkv and tp % self.nkv == 0) else 1
        for n, what in ((self.nq, "attention heads"), (self.nkv * self.kv_replicas, "key/value heads (or TP multiple)"),
                        (self.lk_heads, "linear-attention key heads"), (self.lv_heads, "linear-attention value heads"),
                        (cfg.intermediate_size, "intermediate size")):
            if n % tp:
                raise ValueError(f"qwen3_5_text: {what} ({n}) must be divisible by tp_size={tp}")
        # local head counts and widths
        self.nq_l, self.nkv_l = self.nq // tp, self.nkv * self.kv_replicas // tp
        self.lk_l, self.lv_l = self.lk_heads // tp, self.lv_heads // tp
        self.kd_l, self.vd_l = self.lk_l * self.dk, self.lv_l * self.dv
        self.inter_l = cfg.intermediate_size // tp
        H, D, kd = cfg.hidden_size, self.D, self.key_dim
        pre = cfg.key_prefix
        dev, dt = device, dtype

        def load(name):
            return loader.get(name).to(device=dev, dtype=dt)

        def rows(name, a, b):
            return loader.get_rows(name, a, b).to(device=dev, dtype=dt)

        def cols(name, a, b):
            return loader.get_cols(name, a, b).to(device=dev, dtype=dt)

        qr = (tr * self.nq_l * 2 * D, (tr + 1) * self.nq_l * 2 * D)          # query+gate rows of q_proj
        kv0 = tr // self.kv_replicas * self.nkv_l
        kvr = (kv0 * D, (kv0 + self.nkv_l) * D)
        oc = (tr * self.nq_l * D, (tr + 1) * self.nq_l * D)
        lqr = (tr * self.kd_l, (tr + 1) * self.kd_l)                          # q block of in_proj_qkv
        lkr = (kd + lqr[0], kd + lqr[1])                                      # k block
        lvr = (2 * kd + tr * self.vd_l, 2 * kd + (tr + 1) * self.vd_l)        # v block
        zr = (tr * self.vd_l, (tr + 1) * self.vd_l)
        hr = (tr * self.lv_l, (tr + 1) * self.lv_l)                           # value heads
        ir = (tr * self.inter_l, (tr + 1) * self.inter_l)
        self.embed = load(f"{pre}.embed_tokens.weight") if include_embed else None
        self.vocab_local, self.vocab_start = cfg.vocab_size, 0
        # frozen vision tower on the stage that embeds the tokens (replicated over
        # TP); every stage keeps its config (image grids give placeholder counts
        # and the multimodal positions)
        self.vision = self.vision_cfg = None
        if cfg.has_vision:
            from graspo_b200.models.vision import VisionConfig, VisionTower

            vc = dict(cfg.extra["vision_config"])
            vc.setdefault("out_hidden_size", cfg.hidden_size)
            self.vision_cfg = VisionConfig.from_dict(vc)
            if include_embed:
                self.vision = VisionTower(self.vision_cfg, loader, "model.visual", dtype=dtype, device=device)
        self.layers: list[HybridLayer] = []
        modules: list[LoRAModule] = []
        for idx in self.local_layers:
            p = f"{pre}.layers.{idx}"
            kind = cfg.layer_kind(idx)
            lay = HybridLayer(idx, kind, load(f"{p}.input_layernorm.weight"), load(f"{p}.post_attention_layernorm.weight"))
            # kind -> (shard kind, full rows, (row range), full cols, (col range), exportable as its own PEFT module)
            if kind == "full_attention":
                a = f"{p}.self_attn"
                lay.w["q_proj"] = rows(f"{a}.q_proj.weight", *qr)
                lay.w["k_proj"] = rows(f"{a}.k_proj.weight", *kvr)
                lay.w["v_proj"] = rows(f"{a}.v_proj.weight", *kvr)
                lay.w["o_proj"] = cols(f"{a}.o_proj.weight", *oc)
                lay.w["q_norm"], lay.w["k_norm"] = load(f"{a}.q_norm.weight"), load(f"{a}.k_norm.weight")
                shards = {"fq": ("rows", 2 * self.nq * D, qr, H, (0, H), True),
                          "fk": ("rows", self.nkv * D, kvr, H, (0, H), True),
                          "fv": ("rows", self.nkv * D, kvr, H, (0, H), True),
                          "fo": ("in", H, (0, H), self.nq * D, oc, True)}
            else:
                a = f"{p}.linear_attn"
                lay.w["in_proj_qkv"] = torch.cat([rows(f"{a}.in_proj_qkv.weight", *r) for r in (lqr, lkr, lvr)])
                lay.w["in_proj_z"] = rows(f"{a}.in_proj_z.weight", *zr)
                lay.w["in_proj_b"] = rows(f"{a}.in_proj_b.weight", *hr)
                lay.w["in_proj_a"] = rows(f"{a}.in_proj_a.weight", *hr)
                lay.w["out_proj"] = cols(f"{a}.out_proj.weight", *zr)
                conv = loader.get(f"{a}.conv1d.weight").reshape(-1, self.conv_k)
                lay.w["conv"] = torch.cat([conv[r0:r1] for r0, r1 in (lqr, lkr, lvr)]).to(device=dev, dtype=dt)
                lay.w["dt_bias"] = loader.get(f"{a}.dt_bias")[hr[0]:hr[1]].float().to(dev)
                lay.w["A_log"] = loader.get(f"{a}.A_log")[hr[0]:hr[1]].float().to(dev)
                lay.w["norm"] = load(f"{a}.norm.weight")
                qkv_rows = 2 * kd + self.value_dim
                shards = {"lq": ("rows", qkv_rows, lqr, H, (0, H), False),
                          "lk": ("rows", qkv_rows, lkr, H, (0, H), False),
                          "lv": ("rows", qkv_rows, lvr, H, (0, H), False),
                          "lz": ("out", self.value_dim, zr, H, (0, H), True),
                          "lo": ("in", H, (0, H), self.value_dim, zr, True)}
            lay.w["gate_proj"] = rows(f"{p}.mlp.gate_proj.weight", *ir)
            lay.w["up_proj"] = rows(f"{p}.mlp.up_proj.weight", *ir)
            lay.w["down_proj"] = cols(f"{p}.mlp.down_proj.weight", *ir)
            I = cfg.intermediate_size
            shards.update({"gate": ("out", I, ir, H, (0, H), True), "up": ("out", I, ir, H, (0, H), True),
                           "down": ("in", H, (0, H), I, ir, True)})
            self.layers.append(lay)
            for k, (sk, out_full, (r0, r1), in_full, (c0, c1), exportable) in shards.items():
                target, sub = _TARGETS[k]
                if not lora_target_enabled(self.lora_targets, target):
                    continue
                modules.append(LoRAModule(
                    module_name=f"layers.{idx}.{k}", target_name=target, hf_module_path=f"{p}.{sub}", layer=idx,
                    kind=k, shard_kind=sk, in_full=in_full, out_full=out_full, in_local=c1 - c0, out_local=r1 - r0,
                    row_start=r0, row_stop=r1, col_start=c0, col_stop=c1, peft_exportable=exportable))
        if include_head:
            self.norm = load(f"{pre}.norm.weight")
            name = "lm_head.weight" if loader.has("lm_head.weight") else f"{pre}.embed_tokens.weight"
            self.lm_head = load(name)
        else:
            self.norm = self.lm_head = None
        if self.vision is not None:
            from graspo_b200.models.vision import vision_lora_modules

            modules += vision_lora_modules(self.vision.cfg, self.lora_targets)
        self.lora = LoRAAdapter(modules, r=lora_r, alpha=lora_alpha, dropout=lora_dropout, device=dev, seed=seed)
        self._mods = {(m.layer, m.kind): m for m in modules}

    # ---------------------------------------------------------------- api parity
    def ensure_transposed(self) -> None:
        return None

    def lora_state_dict(self):
        return self.lora.state_dict()

    def lora_tensor_metadata(self):
        return self.lora.metadata()

    def lora_target_signature(self):
        return self.lora.signature()

    def enabled_lora_target_names(self):
        return self.lora.target_names()

    def estimate_kv_cache_bytes(self, *, batch_size: int, sequence_len: int) -> int:
        """Bytes of this rank's decoding caches (local heads of the local layers)."""
        full = sum(1 for lay in self.layers if lay.kind == "full_attention")
        lin = len(self.layers) - full
        kv = batch_size * full * 2 * self.nkv_l * self.D * sequence_len * self.dtype.itemsize
        state = batch_size * lin * (self.lv_l * self.dk * self.dv * 4
                                    + (2 * self.kd_l + self.vd_l) * self.conv_k * self.dtype.itemsize)
        return kv + state

    def sync_partial_grads(self) -> None:
        """Sum the LoRA B gradients of key/value heads held by several TP ranks over those ranks.

        With replicated key/value heads each copy only sees the gradient of
        its own rank's query heads; the B rows of one head must get the sum.
        The rows are placed in a whole-module buffer, summed over the TP group
        (other groups contribute zeros) and read back."""
        if self.kv_replicas == 1 or self.tp_group is None:
            return
        mods = [m for m in self.lora.modules if m.kind in ("fk", "fv")]
        if not mods:
            return
        full = torch.zeros(len(mods), mods[0].out_full, self.lora.r, device=self.device, dtype=torch.float32)
        for i, m in enumerate(mods):
            full[i, m.row_start : m.row_stop] = m.b_grad
        dist.all_reduce(full, group=self.tp_group)
        for i, m in enumerate(mods):
            m.b_grad.copy_(full[i, m.row_start : m.row_stop])

    def _f(self, x):
        """Identity forward, all-reduce backward (input of the column-parallel projections)."""
        return copy_to_tp(x, self.tp_group) if self.tp_group is not None else x

    def _g(self, x):
        """All-reduce forward, identity backward (output of the row-parallel projections)."""
        return reduce_from_tp(x, self.tp_group) if self.tp_group is not None else x

    # ---------------------------------------------------------------- pieces
    def _lin(self, x, w, lay, kind, lora, training):
        y = F.linear(x, w)
        mod = self._mods.get((lay.index, kind))
        if mod is None or lora is None:
            return y
        a, b = lora.leaves[mod.module_name]
        ad = self.lora
        xin = F.dropout(x, ad.dropout, training) if (training and ad.dropout > 0) else x
        return y + (F.linear(F.linear(xin.to(a.dtype), a), b) * ad.scaling).to(y.dtype)

    def _rope(self, x, pos):
        """Partial rotary embedding (rotate-half on the first rotary_dim dims). x [B, S, h, D]; pos [B, S]
        (text) or [3, B, S] (time / height / width positions of multimodal RoPE)."""
        rd = self.rotary_dim
        f = pos.float()[..., None] * self.inv_freq                     # [B, S, rd/2] or [3, B, S, rd/2]
        if pos.dim() == 3:
            idx = self.mrope_component.view(1, 1, 1, -1).expand(1, *f.shape[1:])
            f = f.gather(0, idx)[0]
        cos, sin = torch.cat([f, f], -1).cos()[:, :, None], torch.cat([f, f], -1).sin()[:, :, None]
        xr, xp = x[..., :rd].float(), x[..., rd:]
        half = rd // 2
        rot = torch.cat([-xr[..., half:], xr[..., :half]], -1)
        return torch.cat([(xr * cos + rot * sin).to(x.dtype), xp], -1)

    def _full_attn(self, lay, h, pos, key_mask, lora, training, cache=None):
        B, S, _ = h.shape
        D = self.D
        nq, nkv = self.nq_l, self.nkv_l
        qg = self._lin(h, lay.w["q_proj"], lay, "fq", lora, training).view(B, S, nq, 2 * D)
        q, gate = qg[..., :D], qg[..., D:].reshape(B, S, nq * D)
        k = self._lin(h, lay.w["k_proj"], lay, "fk", lora, training).view(B, S, nkv, D)
        v = self._lin(h, lay.w["v_proj"], lay, "fv", lora, training).view(B, S, nkv, D)
        q = self._rope(norm1p(q, lay.w["q_norm"], self.cfg.rms_norm_eps), pos)
        k = self._rope(norm1p(k, lay.w["k_norm"], self.cfg.rms_norm_eps), pos)
        if cache is not None:
            if "k" in cache:
                k = torch.cat([cache["k"], k], 1)
                v = torch.cat([cache["v"], v], 1)
            cache["k"], cache["v"] = k, v
        Sk = k.shape[1]
        G = nq // nkv
        qh = q.transpose(1, 2)
        shift = _valid_span_start(key_mask) if cache is None and Sk == S else None
        if shift is not None:
            # Every row's valid tokens form one span (left-padded prompt, right-
            # padded completion): rotate each row so its span starts at 0, run
            # plain causal attention, which SDPA does without a mask (and without
            # copying the key / value heads for the query groups), rotate back.
            # Valid queries see exactly the valid keys before them; the outputs at
            # padding positions differ from the masked form, and nothing reads them
            # (the DeltaNet layers zero padding inputs, attention masks padding keys).
            ar = torch.arange(S, device=h.device)
            fwd = None if not bool(shift.any()) else (ar[None] + shift[:, None]) % S
            qs, ks, vs = ((t if fwd is None else t.gather(1, fwd[:, :, None, None].expand_as(t))).transpose(1, 2)
                          for t in (q, k, v))
            o = F.scaled_dot_product_attention(qs, ks, vs, is_causal=True, scale=1.0 / math.sqrt(D),
                                               enable_gqa=G > 1).transpose(1, 2)
            if fwd is not None:
                back = (ar[None] - shift[:, None]) % S
                o = o.gather(1, back[:, :, None, None].expand_as(o))
            o = o.reshape(B, S, nq * D)
            return self._lin(sigmoid_gate(o, gate), lay.w["o_proj"], lay, "fo", lora, training)
        kh = k.transpose(1, 2).repeat_interleave(G, 1)
        vh = v.transpose(1, 2).repeat_interleave(G, 1)
        qpos = torch.arange(Sk - S, Sk, device=h.device)
        kpos = torch.arange(Sk, device=h.device)
        allowed = (qpos[:, None] >= kpos[None])[None] & key_mask[:, None, :]
        # a padding query attends to itself, so no softmax row is empty
        allowed = allowed | (qpos[:, None] == kpos[None])[None]
        o = F.scaled_dot_product_attention(qh, kh, vh, attn_mask=allowed[:, None], scale=1.0 / math.sqrt(D))
        o = o.transpose(1, 2).reshape(B, S, nq * D)
        return self._lin(sigmoid_gate(o, gate), lay.w["o_proj"], lay, "fo", lora, training)   # partial over TP

    def _linear_attn(self, lay, h, key_mask, lora, training, cache=None):
        B, S, _ = h.shape
        h = h * key_mask[:, -S:, None].to(h.dtype)
        W = lay.w["in_proj_qkv"]
        kd, vd = self.kd_l, self.vd_l
        q = self._lin(h, W[:kd], lay, "lq", lora, training)
        k = self._lin(h, W[kd : 2 * kd], lay, "lk", lora, training)
        v = self._lin(h, W[2 * kd :], lay, "lv", lora, training)
        mixed_in = torch.cat([q, k, v], -1)                                # [B, S, C]
        K = self.conv_k
        prev = cache.get("conv") if cache is not None else None
        if cache is not None:
            # the last K-1 inputs [B, C, K-1] carry the convolution into the next call
            xt = mixed_in.detach().transpose(1, 2)
            ext = torch.cat([prev, xt], -1) if prev is not None else F.pad(xt, (K - 1, 0))
            cache["conv"] = ext[..., -(K - 1):].contiguous().clone()
        mixed = conv_silu(mixed_in, prev, lay.w["conv"])                   # causal conv1d + SiLU, [B, S, C]
        q, k, v = mixed[..., :kd], mixed[..., kd : 2 * kd], mixed[..., 2 * kd :]
        q = q.reshape(B, S, self.lk_l, self.dk)
        k = k.reshape(B, S, self.lk_l, self.dk)
        v = v.reshape(B, S, self.lv_l, self.dv)
        z = self._lin(h, lay.w["in_proj_z"], lay, "lz", lora, training).reshape(B, S, self.lv_l, self.dv)
        beta = torch.sigmoid(F.linear(h, lay.w["in_proj_b"]).float())
        g = -lay.w["A_log"].exp() * F.softplus(F.linear(h, lay.w["in_proj_a"]).float() + lay.w["dt_bias"])
        rep = self.lv_heads // self.lk_heads
        if rep > 1:
            q, k = q.repeat_interleave(rep, 2), k.repeat_interleave(rep, 2)
        q = l2norm(q.float()) / math.sqrt(self.dk)
        k = l2norm(k.float())
        state = cache.get("state") if cache is not None else None
        if cache is not None and state is not None and S == 1:
            o = gated_delta_step(q[:, 0], k[:, 0], v[:, 0], g[:, 0], beta[:, 0], state)[:, None]
        else:
            o, fin = chunk_gated_delta(q, k, v, g, beta, state)
            if cache is not None:
                cache["state"] = fin.detach().clone()
        o = gated_norm(o.to(h.dtype).reshape(-1, self.dv), z.reshape(-1, self.dv), lay.w["norm"],
                       self.cfg.rms_norm_eps).reshape(B, S, vd)
        return self._lin(o, lay.w["out_proj"], lay, "lo", lora, training)   # partial over TP

    def layer(self, lay, x, pos, key_mask, lora=None, training=False, cache=None):
        eps = self.cfg.rms_norm_eps
        h = self._f(norm1p(x, lay.ln1, eps))
        if lay.kind == "full_attention":
            x = x + self._g(self._full_attn(lay, h, pos, key_mask, lora, training, cache))
        else:
            x = x + self._g(self._linear_attn(lay, h, key_mask, lora, training, cache))
        h2 = self._f(norm1p(x, lay.ln2, eps))
        gate = self._lin(h2, lay.w["gate_proj"], lay, "gate", lora, training)
        up = self._lin(h2, lay.w["up_proj"], lay, "up", lora, training)
        return x + self._g(self._lin(F.silu(gate) * up, lay.w["down_proj"], lay, "down", lora, training))

    def mrope_positions(self, ids, mask, images) -> torch.Tensor:
        """[3, B, S] time / height / width positions of a batch with image placeholders.

        Text tokens advance one position (all three equal); the ``t * h * w``
        placeholders of an image (``images.grids``: merged grids in row order)
        take ``start + (0, row, col)`` and the text after it resumes at
        ``start + max(h, w)``.  Padding gets 0 (reference:
        models/qwen35_36/model.py:289-330, 372-461)."""
        B, S = ids.shape
        out = torch.zeros(3, B, S, dtype=torch.long)
        grids = iter(images.grids)
        ids_c, mask_c = ids.cpu(), mask.cpu()
        for b in range(B):
            cols = torch.nonzero(mask_c[b]).flatten().tolist()
            toks = ids_c[b, cols].tolist()
            pos, i, rows = 0, 0, []
            while i < len(toks):
                if toks[i] != images.pad_id:
                    rows.append((pos, pos, pos))
                    pos, i = pos + 1, i + 1
                    continue
                t, h, w = next(grids)
                for ti in range(t):
                    for hi in range(h):
                        for wi in range(w):
                            rows.append((pos + ti, pos + hi, pos + wi))
                i += t * h * w
                pos += max(h, w)
            if len(rows) != len(cols):
                raise ValueError("image placeholder count does not match the image grids")
            out[:, b, cols] = torch.tensor(rows, dtype=torch.long).T
        return out.to(ids.device)

    def forward(self, ids, mask, *, x=None, lora=None, training=False, caches=None, pos=None, key_mask=None,
                embed_hook=None):
        """[B, S] ids -> hidden [B, S, H] after this stage's layers (whole-sequence;
        caches fill for decoding).  On a later pipeline stage ``x`` is the
        previous stage's output and ``ids`` is unused.  ``embed_hook`` places
        image features on the placeholder embeddings; with it the positions
        are the multimodal RoPE ones unless ``pos`` is given."""
        if x is None:
            x = F.embedding(ids, self.embed)
            if embed_hook is not None:
                x = embed_hook(ids, x)
                if pos is None and getattr(embed_hook, "grids", None):
                    pos = self.mrope_positions(ids, mask, embed_hook)
        pos = (mask.long().cumsum(-1) - 1).clamp_min(0) if pos is None else pos
        key_mask = mask if key_mask is None else key_mask
        for i, lay in enumerate(self.layers):
            c = caches[i] if caches is not None else None
            if training and self.gradient_checkpointing and c is None:
                x = torch.utils.checkpoint.checkpoint(self.layer, lay, x, pos, key_mask, lora, training,
                                                      use_reentrant=False)
            else:
                x = self.layer(lay, x, pos, key_mask, lora, training, c)
        return x

    def logits(self, hidden):
        """fp32 logits of the last hidden states (sampling); the head GEMM on the GPU."""
        from graspo_b200.ops.head import kernel_head_ok, vocab_logits

        hn = norm1p(hidden, self.norm, self.cfg.rms_norm_eps)
        flat = hn.reshape(-1, hn.shape[-1])
        if kernel_head_ok(flat, self.lm_head):
            return vocab_logits(flat, self.lm_head).view(*hn.shape[:-1], -1)
        return F.linear(hn.float(), self.lm_head.float())

    def token_logprobs(self, hidden, targets, chunk: int = 8192):
        """log p(targets) from final hidden states.  On the GPU the vocabulary
        GEMM keeps only per-row (max, sum-exp) partials and the target logit
        (``ops/head.py``); on the CPU fp32 logits are formed in token chunks."""
        from graspo_b200.ops.head import kernel_head_ok, selected_token_logprobs

        hn = norm1p(hidden, self.norm, self.cfg.rms_norm_eps)
        flat, tg = hn.reshape(-1, hn.shape[-1]), targets.reshape(-1)
        if kernel_head_ok(flat, self.lm_head):
            return selected_token_logprobs(flat, self.lm_head, tg, chunk_tokens=chunk).view(targets.shape)
        out = []
        for i in range(0, flat.shape[0], chunk):
            lg = F.linear(flat[i : i + chunk].float(), self.lm_head.float())
            out.append(lg.gather(-1, tg[i : i + chunk, None]).squeeze(-1) - torch.logsumexp(lg, -1))
        return torch.cat(out).view(targets.shape)

    def sequence_logprobs(self, seq, mask, *, lora=None, training=False, targets=None, embed_hook=None):
        hidden = self.forward(seq, mask, lora=lora, training=training, embed_hook=embed_hook)
        tgt = seq[:, 1:] if targets is None else targets
        return self.token_logprobs(hidden[:, :-1], tgt)


def gated_delta_step(q, k, v, g, beta, state):
    """One decoding step of the recurrence; the sm_100a kernel on GPUs (state updated in place)."""
    if state.is_cuda:
        from graspo_b200.ops._ext import ext

        out = torch.empty(v.shape, device=v.device, dtype=torch.float32)
        ext().gated_delta_step(q.float().contiguous(), k.float().contiguous(), v.float().contiguous(),
                               g.float().contiguous(), beta.float().contiguous(), state, out)
        return out
    return recurrent_gated_delta(q, k, v, g, beta, state)


class HybridRolloutEngine:
    """Grouped sampling for the hybrid decoder: each prompt is prefilled once,
    its caches (KV for attention layers, conv + recurrent state for DeltaNet
    layers) are copied to its G rows, then tokens are decoded one at a time.

    With pipeline stages (``comm`` over a column of stages, each holding the
    caches of its own layers) the hidden states of the prefill and of every
    decoding step travel stage to stage, the last stage samples, and the token
    is broadcast to the column so every stage embeds / tracks the same rows
    (the reference has no pipelined rollout: qwen35_36/generation.py:645-685).
    """

    def __init__(self, model: Qwen35Model, comm=None) -> None:
        self.m = model
        self.comm = comm if comm is not None and comm.active else None

    def _stage(self, ids, mask, **kw):
        """This stage's layers: input from the previous stage (or the embedding), output to the next."""
        m, comm = self.m, self.comm
        x = None
        if comm is not None and not m.ps.is_first_stage:
            x = comm.recv_prev((ids.shape[0], ids.shape[1], m.cfg.hidden_size), m.dtype)
        y = m.forward(ids, mask, x=x, **kw)
        if comm is not None and not m.ps.is_last_stage:
            comm.send_next(y)
            comm.flush()
        return y

    @torch.no_grad()
    def generate(self, prompts, *, group_size, max_new_tokens, temperature, top_p, eos_id, pad_id,
                 ignore_eos=False, seed=0, embed_hook=None):
        """``embed_hook`` (``ImageInputs``) places image features on the prompts' placeholders;
        decoding then continues from each prompt's largest multimodal position.
        With pipeline stages the first stage's hook carries the features and
        every stage's hook the image grids, from which each stage derives the
        same multimodal positions."""
        import time

        from graspo_b200.engine.rollout import EagerRolloutEngine, RolloutResult, _gen_lengths

        m, dev, comm = self.m, self.m.device, self.comm
        last = comm is None or m.ps.is_last_stage
        n, G = len(prompts), int(group_size)
        lens = [max(1, len(p)) for p in prompts]
        P = max(lens)
        ids = torch.full((n, P), pad_id, dtype=torch.long)
        mask = torch.zeros((n, P), dtype=torch.bool)
        for i, p in enumerate(prompts):
            row = list(p) or [pad_id]
            ids[i, P - len(row):] = torch.tensor(row)
            mask[i, P - len(row):] = True
        t0 = time.perf_counter()
        ids_d, mask_d = ids.to(dev), mask.to(dev)
        caches = [dict() for _ in m.layers]
        lora = EagerLoRA(m.lora, requires_grad=False)      # the current policy's adapter (views of the master)
        if getattr(embed_hook, "grids", None):
            pos3 = m.mrope_positions(ids_d, mask_d, embed_hook)
            hidden = self._stage(ids_d, mask_d, caches=caches, lora=lora, embed_hook=embed_hook, pos=pos3)
            last_pos = pos3.amax(dim=(0, 2))
        else:
            hidden = self._stage(ids_d, mask_d, caches=caches, lora=lora, embed_hook=embed_hook)
            last_pos = mask_d.long().sum(-1) - 1
        for c in caches:
            for key, val in list(c.items()):
                c[key] = val.repeat_interleave(G, 0)
        key_mask = mask_d.repeat_interleave(G, 0)
        pos = last_pos.repeat_interleave(G, 0)
        logits = m.logits(hidden[:, -1]).repeat_interleave(G, 0) if last else None
        gen = torch.Generator(device=dev).manual_seed(int(seed))
        rows = n * G
        out = torch.full((rows, max_new_tokens), pad_id, dtype=torch.long, device=dev)
        finished = torch.zeros(rows, dtype=torch.bool, device=dev)
        t1 = time.perf_counter()
        steps = 0
        for t in range(max_new_tokens):
            if last:
                tok = EagerRolloutEngine._sample(logits, temperature, top_p, gen)
                if m.tp_group is not None:
                    # TP ranks hold the same logits and noise; the leader's draw settles any last-bit difference
                    dist.broadcast(tok, src=m.ps.rank_of(tp=0, pp=m.ps.pp_rank, dp=m.ps.dp_rank), group=m.tp_group)
            else:
                tok = torch.empty(rows, dtype=torch.long, device=dev)
            if comm is not None:
                comm.broadcast_from_last(tok)
            tok = torch.where(finished, torch.full_like(tok, pad_id), tok)
            out[:, t] = tok
            if not ignore_eos:
                finished |= tok == eos_id
            steps += 1
            if t + 1 == max_new_tokens or (not ignore_eos and bool(finished.all())):
                break
            key_mask = torch.cat([key_mask, torch.ones(rows, 1, dtype=torch.bool, device=dev)], 1)
            pos = pos + 1
            x = self._stage(tok[:, None], key_mask[:, -1:], caches=caches, pos=pos[:, None], key_mask=key_mask,
                            lora=lora)
            logits = m.logits(x[:, -1]) if last else None
        tokens = out.cpu()
        return RolloutResult(prompt_ids=ids, prompt_lens=lens, tokens=tokens,
                             gen_lens=_gen_lengths(tokens, eos_id, ignore_eos), group_size=G,
                             prefill_sec=t1 - t0, decode_sec=time.perf_counter() - t1, decode_steps=steps)


__all__ = ["Qwen35Model", "HybridRolloutEngine", "chunk_gated_delta", "recurrent_gated_delta", "gated_delta_step",
           "EagerLoRA"]
