"""LoRA adapter state for a TP/PP-sharded decoder.

Parameters live in one flat fp32 buffer (master weights) with one flat fp32
gradient buffer beside it, so the optimizer, the gradient-norm reduction and
the data-parallel all-reduce each touch a single contiguous tensor.  Every
adapted module owns two views into it:

* ``lora_a [r, in_local]`` -- initialised Kaiming-uniform (bound 1/sqrt(fan_in)),
* ``lora_b [out_local, r]`` -- zeros,

so the adapter starts as an exact no-op (reference: lora.py:76-213).  Shard
kinds follow the reference checkpoint format: ``out`` (column parallel: rows of
W and B are split, A is replicated), ``rows`` (a head-row selection or a row
block of a fused HF matrix, ``row_start:row_stop`` in that matrix's rows; A is
replicated), ``in`` (row parallel: columns of W and A are split, B is
replicated), ``none``.  The initial A of a module is drawn for
the *full* matrix from a generator seeded by (seed, module name) and then
sliced, so a TP=2 run starts from exactly the TP=1 adapter.

The reference keeps LoRA tensors in the model dtype (bf16); here the master
copy is fp32 (an lr of 5e-6 would otherwise be rounded away) and bf16 copies in
the layouts the fused GEMMs consume are rebuilt after every optimizer step.
"""

from __future__ import annotations

import hashlib
import math
from dataclasses import dataclass, field
from typing import Any

import torch


@dataclass
class LoRAModule:
    module_name: str          # e.g. "layers.3.self_attn.q_proj"
    target_name: str          # canonical target, e.g. "language.self_attn.q_proj"
    hf_module_path: str       # e.g. "model.layers.3.self_attn.q_proj"
    layer: int
    kind: str                 # q k v o gate up down
    shard_kind: str           # out | in | none
    in_full: int
    out_full: int
    in_local: int
    out_local: int
    row_start: int | None = None
    row_stop: int | None = None
    col_start: int | None = None
    col_stop: int | None = None
    a: torch.Tensor | None = None
    b: torch.Tensor | None = None
    a_grad: torch.Tensor | None = None
    b_grad: torch.Tensor | None = None
    offset_a: int = 0
    offset_b: int = 0
    # False for a target that is a row block of a larger HF module (DeltaNet
    # q/k/v inside in_proj_qkv): PEFT export combines the blocks into one pair
    peft_exportable: bool = True

    @property
    def replicated_factor(self) -> str:
        """Which factor is replicated across the TP group ('a' or 'b'; 'ab' for a
        module that is not sharded at all, such as a vision-tower linear)."""
        if self.shard_kind == "none":
            return "ab"
        return "b" if self.shard_kind == "in" else "a"


def _module_seed(seed: int, name: str) -> int:
    digest = hashlib.sha256(f"{seed}:{name}".encode()).digest()
    return int.from_bytes(digest[:8], "little") & ((1 << 62) - 1)


class LoRAAdapter:
    def __init__(
        self,
        modules: list[LoRAModule],
        *,
        r: int,
        alpha: float,
        dropout: float,
        device: torch.device,
        seed: int = 42,
        tp_rank: int = 0,
    ) -> None:
        self.modules = modules
        self.r = int(r)
        self.alpha = float(alpha)
        self.scaling = float(alpha) / float(r) if r > 0 else 1.0
        self.dropout = float(dropout)
        self.device = device
        # Replicated factors first, sharded factors after: the TP gradient
        # all-reduce then covers one contiguous prefix of the flat buffer.
        total = 0
        for replicated_pass in (True, False):
            for mod in modules:
                for fac in ("a", "b"):
                    if (fac in mod.replicated_factor) != replicated_pass:
                        continue
                    size = self.r * mod.in_local if fac == "a" else mod.out_local * self.r
                    setattr(mod, f"offset_{fac}", total)
                    total += size
            if replicated_pass:
                self.replicated_numel = total
        self.numel = total
        self.params = torch.zeros(total, dtype=torch.float32, device=device)
        self.grads = torch.zeros(total, dtype=torch.float32, device=device)
        for mod in modules:
            self._bind(mod)
            gen = torch.Generator().manual_seed(_module_seed(seed, mod.module_name))
            bound = 1.0 / math.sqrt(mod.in_full)
            full_a = torch.empty(self.r, mod.in_full).uniform_(-bound, bound, generator=gen)
            if mod.shard_kind == "in":
                full_a = full_a[:, mod.col_start : mod.col_stop]
            mod.a.copy_(full_a.to(device))
        self.by_name = {m.module_name: m for m in modules}
        self.layouts: dict[int, dict[str, torch.Tensor]] = {}

    def layer_ranges(self, layer: int) -> list[tuple[int, int]]:
        """(start, count) ranges of the flat buffer that hold one layer's factors,
        adjacent ranges merged (a layer's factors sit in the replicated and in the
        sharded part of the buffer)."""
        spans = []
        for mod in self.modules:
            if mod.layer != layer:
                continue
            spans.append((mod.offset_a, self.r * mod.in_local))
            spans.append((mod.offset_b, mod.out_local * self.r))
        spans.sort()
        merged: list[list[int]] = []
        for start, count in spans:
            if merged and merged[-1][0] + merged[-1][1] == start:
                merged[-1][1] += count
            else:
                merged.append([start, count])
        return [(a, b) for a, b in merged]

    def _bind(self, mod: LoRAModule) -> None:
        a_n = self.r * mod.in_local
        b_n = mod.out_local * self.r
        mod.a = self.params[mod.offset_a : mod.offset_a + a_n].view(self.r, mod.in_local)
        mod.b = self.params[mod.offset_b : mod.offset_b + b_n].view(mod.out_local, self.r)
        mod.a_grad = self.grads[mod.offset_a : mod.offset_a + a_n].view(self.r, mod.in_local)
        mod.b_grad = self.grads[mod.offset_b : mod.offset_b + b_n].view(mod.out_local, self.r)

    # ------------------------------------------------------------ queries
    def module(self, layer: int, kind: str) -> LoRAModule | None:
        for mod in self.modules:
            if mod.layer == layer and mod.kind == kind:
                return mod
        return None

    def state_dict(self) -> dict[str, torch.Tensor]:
        """CPU copies keyed like the reference (``<module>.lora_a`` / ``.lora_b``)."""
        out: dict[str, torch.Tensor] = {}
        for mod in self.modules:
            out[f"{mod.module_name}.lora_a"] = mod.a.detach().cpu().clone()
            out[f"{mod.module_name}.lora_b"] = mod.b.detach().cpu().clone()
        return out

    def load_state_dict(self, state: dict[str, torch.Tensor], *, strict: bool = True) -> None:
        expected = {f"{m.module_name}.lora_{f}" for m in self.modules for f in ("a", "b")}
        missing = sorted(expected - set(state))
        unexpected = sorted(k for k in state if "lora_" in k and k not in expected)
        if strict and (missing or unexpected):
            raise RuntimeError(f"LoRA state mismatch: missing={missing[:5]} unexpected={unexpected[:5]}")
        for mod in self.modules:
            for fac in ("a", "b"):
                key = f"{mod.module_name}.lora_{fac}"
                if key in state:
                    getattr(mod, fac).copy_(state[key].to(device=self.device, dtype=torch.float32))
        self.layouts.clear()

    def metadata(self) -> list[dict[str, Any]]:
        return [
            {
                "module_name": m.module_name,
                "lora_a_name": f"{m.module_name}.lora_a",
                "lora_b_name": f"{m.module_name}.lora_b",
                "target_name": m.target_name,
                "hf_module_path": m.hf_module_path,
                "base_weight_name": f"{m.hf_module_path}.weight",
                "shard_kind": m.shard_kind,
                "row_start": m.row_start,
                "row_stop": m.row_stop,
                "col_start": m.col_start,
                "col_stop": m.col_stop,
                "row_indices": None,
                "peft_exportable": m.peft_exportable,
                "r": self.r,
                "alpha": int(self.alpha) if float(self.alpha).is_integer() else self.alpha,
            }
            for m in self.modules
        ]

    def target_names(self) -> tuple[str, ...]:
        return tuple(sorted({m.target_name for m in self.modules}))

    def signature(self) -> dict[str, object]:
        return {"resolved": list(self.target_names()), "parameter_count": int(self.numel)}

    def parameter_norm(self) -> float:
        return float(self.params.norm().item())

    def replicated_mask(self) -> torch.Tensor:
        """1.0 for elements that are replicated across the TP group, else 0.0."""
        mask = torch.zeros(self.numel, dtype=torch.float32, device=self.device)
        for m in self.modules:
            if "a" in m.replicated_factor:
                mask[m.offset_a : m.offset_a + self.r * m.in_local] = 1.0
            if "b" in m.replicated_factor:
                mask[m.offset_b : m.offset_b + m.out_local * self.r] = 1.0
        return mask

    def vision_modules(self) -> list[LoRAModule]:
        """LoRA modules of the vision tower (replicated over TP, outside the decoder layers)."""
        return [m for m in self.modules if m.kind == "vision"]

    # ------------------------------------------------------------ fused layouts
    def invalidate(self) -> None:
        self.layouts.clear()

    def layer_layouts(self, layer: int, sizes: dict[str, int]) -> dict[str, torch.Tensor]:
        """bf16 operands for the fused GEMMs of one decoder layer.

        ``a_<group>`` [64*k, in]: the A factors of the group's targets stacked
        (qkv: q,k,v; gu: gate,up), pre-multiplied by the LoRA scale alpha/r and
        zero-padded; ``b_<group>`` [out, 64*k]: the B
        factors placed block-diagonally (gate/up rows interleaved to match the
        interleaved gate/up weight).  Rebuilt lazily after ``invalidate()``.
        """
        cached = self.layouts.get(layer)
        if cached is not None:
            return cached
        r = self.r
        out: dict[str, torch.Tensor] = {}
        dev = self.device
        bf = torch.bfloat16
        s = self.scaling

        def pad64(n: int) -> int:
            return max(64, ((n + 63) // 64) * 64)

        # qkv
        q, k, v = (self.module(layer, x) for x in ("q", "k", "v"))
        parts = [(m, sizes[name]) for m, name in ((q, "q"), (k, "kv"), (v, "kv"))]
        if any(m is not None for m, _ in parts):
            width = pad64(3 * r)
            a = torch.zeros(width, sizes["hidden"], dtype=bf, device=dev)
            b = torch.zeros(sizes["q"] + 2 * sizes["kv"], width, dtype=bf, device=dev)
            row = 0
            for slot, (m, rows) in enumerate(parts):
                if m is not None:
                    a[slot * r : (slot + 1) * r] = (m.a * s).to(bf)
                    b[row : row + rows, slot * r : (slot + 1) * r] = m.b.to(bf)
                row += rows
            out["a_qkv"], out["b_qkv"] = a, b
        o = self.module(layer, "o")
        if o is not None:
            width = pad64(r)
            a = torch.zeros(width, o.in_local, dtype=bf, device=dev)
            a[:r] = (o.a * s).to(bf)
            b = torch.zeros(o.out_local, width, dtype=bf, device=dev)
            b[:, :r] = o.b.to(bf)
            out["a_o"], out["b_o"] = a, b
        g, u = self.module(layer, "gate"), self.module(layer, "up")
        if g is not None or u is not None:
            width = pad64(2 * r)
            inter = sizes["inter"]
            a = torch.zeros(width, sizes["hidden"], dtype=bf, device=dev)
            b = torch.zeros(2 * inter, width, dtype=bf, device=dev)
            if g is not None:
                a[:r] = (g.a * s).to(bf)
                b[0::2, :r] = g.b.to(bf)
            if u is not None:
                a[r : 2 * r] = (u.a * s).to(bf)
                b[1::2, r : 2 * r] = u.b.to(bf)
            out["a_gu"], out["b_gu"] = a, b
        d = self.module(layer, "down")
        if d is not None:
            width = pad64(r)
            a = torch.zeros(width, d.in_local, dtype=bf, device=dev)
            a[:r] = (d.a * s).to(bf)
            b = torch.zeros(d.out_local, width, dtype=bf, device=dev)
            b[:, :r] = d.b.to(bf)
            out["a_down"], out["b_down"] = a, b
        self.layouts[layer] = out
        return out


@dataclass
class LoRAPlan:
    """Which canonical targets are adapted, and the adapter hyper-parameters."""

    targets: frozenset[str]
    r: int = 16
    alpha: float = 32
    dropout: float = 0.1
    extra: dict[str, Any] = field(default_factory=dict)
