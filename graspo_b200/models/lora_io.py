"""PEFT import/export and merged-weights export of native LoRA checkpoints.

Formats (reference: backends/graspoflow/lora_io.py, kept byte-compatible so
adapters move between frameworks and into PEFT / vLLM):

* PEFT adapter directory: ``adapter_model.safetensors`` with keys
  ``base_model.model.<hf_module>.lora_A.weight`` [r, in] / ``lora_B.weight``
  [out, r], and ``adapter_config.json`` (``peft_type: LORA``, ``r``,
  ``lora_alpha``, ``target_modules`` as leaf names, ``rank_pattern`` /
  ``alpha_pattern`` for modules that differ from the first, ``bias``,
  ``task_type``, ``base_model_name_or_path``, ``inference_mode: true``).
* Reconstruction from TP shards: for column-parallel modules (shard ``out``)
  the replicated A must agree across ranks and B rows are placed by
  ``row_start:row_stop``; for row-parallel (``in``) the replicated B must agree
  and A columns are placed by ``col_start:col_stop``.
* Row blocks of one HF module (the DeltaNet ``q/k/v_proj`` targets inside
  ``in_proj_qkv``, records with ``peft_exportable: false``) become ONE PEFT
  pair: the targets' A factors stacked along the rank axis, their B factors
  placed on their rows with the LoRA scale folded in, ``r = lora_alpha`` =
  the summed rank (PEFT scale 1).  ``graspo_adapter_metadata.json`` records
  each target's rank slice and B scale so the import can split the pair again
  (reference: lora_io.py:313-350, 432-499).
* Merged Hugging Face export: every base safetensors file is streamed,
  ``W += (alpha / r) * B @ A`` is added on the rows/columns the shard covered,
  and non-weight sidecar files are copied.
"""

from __future__ import annotations

import json
import shutil
from pathlib import Path
from typing import Any

import torch
from safetensors import safe_open
from safetensors.torch import load_file, save_file

PEFT_PREFIX = "base_model.model."
METADATA_FILE = "graspo_adapter_metadata.json"


def _payloads(checkpoint_dir: str | Path) -> list[dict[str, Any]]:
    files = sorted(Path(checkpoint_dir).glob("rank_*_tp_*_pp_*.pt"))
    if not files:
        raise FileNotFoundError(f"No native GRASPO rank checkpoint files in {checkpoint_dir}")
    payloads = [torch.load(f, map_location="cpu", weights_only=False) for f in files]
    for p in payloads:
        if not p.get("lora_tensor_metadata"):
            raise ValueError("checkpoint shard has no lora_tensor_metadata")
    return payloads


def _grouped(payloads) -> dict[str, list[tuple[dict, dict[str, torch.Tensor]]]]:
    out: dict[str, list] = {}
    for payload in payloads:
        state = payload["lora_state_dict"]
        for rec in payload["lora_tensor_metadata"]:
            pair = {"A": state[rec["lora_a_name"]], "B": state[rec["lora_b_name"]]}
            out.setdefault(rec["hf_module_path"], []).append((dict(rec), pair))
    return out


def _same(module: str, tensors: list[torch.Tensor], label: str) -> torch.Tensor:
    first = tensors[0].float()
    for t in tensors[1:]:
        if t.shape != first.shape or not torch.allclose(t.float(), first, rtol=1e-5, atol=1e-6):
            raise ValueError(
                f"TP shards of {module} disagree on the replicated {label}; a PEFT adapter cannot "
                "represent them (use export_format: merged-hf)"
            )
    return tensors[0]


def reconstruct_pair(module: str, items) -> tuple[torch.Tensor, torch.Tensor]:
    kinds = {r["shard_kind"] for r, _ in items}
    if kinds == {"none"}:
        return items[0][1]["A"], items[0][1]["B"]
    if kinds <= {"out", "rows"}:
        a = _same(module, [p["A"] for _, p in items], "lora_A")
        rows = max(int(r["row_stop"]) for r, _ in items)
        b = torch.zeros(rows, a.shape[0], dtype=items[0][1]["B"].dtype)
        filled = torch.zeros(rows, dtype=torch.bool)
        for r, p in items:
            b[r["row_start"] : r["row_stop"]] = p["B"]
            filled[r["row_start"] : r["row_stop"]] = True
    elif kinds <= {"in", "cols"}:
        b = _same(module, [p["B"] for _, p in items], "lora_B")
        cols = max(int(r["col_stop"]) for r, _ in items)
        a = torch.zeros(b.shape[1], cols, dtype=items[0][1]["A"].dtype)
        filled = torch.zeros(cols, dtype=torch.bool)
        for r, p in items:
            a[:, r["col_start"] : r["col_stop"]] = p["A"]
            filled[r["col_start"] : r["col_stop"]] = True
    else:
        raise ValueError(f"mixed shard kinds for {module}: {kinds}")
    if not bool(filled.all()):
        raise ValueError(f"TP shards of {module} do not cover the full tensor")
    return a, b


def combine_row_blocks(module: str, items) -> tuple[torch.Tensor, torch.Tensor, list[dict[str, Any]]]:
    """One PEFT pair for several row-block targets of one HF module (and the
    rank slices that undo it)."""
    by_target: dict[str, list] = {}
    for rec, pair in items:
        by_target.setdefault(str(rec["target_name"]), []).append((rec, pair))
    rows = max(int(rec["row_stop"]) for rec, _ in items)
    parts = []
    for target, group in sorted(by_target.items()):
        kinds = {rec["shard_kind"] for rec, _ in group}
        if not kinds <= {"rows", "out"}:
            raise ValueError(f"row-block target {target} of {module} has shard kinds {sorted(kinds)}")
        a = _same(module, [p["A"] for _, p in group], f"{target} lora_A")
        b = torch.zeros(rows, a.shape[0], dtype=group[0][1]["B"].dtype)
        for rec, p in group:
            b[rec["row_start"] : rec["row_stop"]] = p["B"]
        rec = group[0][0]
        scale = float(rec["alpha"]) / float(rec["r"])
        parts.append((rec, a, b * scale, scale))
    total = sum(a.shape[0] for _, a, _, _ in parts)
    comb_a = torch.zeros(total, parts[0][1].shape[1], dtype=parts[0][1].dtype)
    comb_b = torch.zeros(rows, total, dtype=parts[0][2].dtype)
    slices, start = [], 0
    for rec, a, b, scale in parts:
        stop = start + a.shape[0]
        comb_a[start:stop], comb_b[:, start:stop] = a, b
        slices.append({"target_name": str(rec["target_name"]), "base_weight_name": str(rec["base_weight_name"]),
                       "rank_start": start, "rank_stop": stop, "native_r": int(rec["r"]),
                       "native_alpha": rec["alpha"], "adapter_b_scale": scale})
        start = stop
    return comb_a, comb_b, slices


def export_peft_adapter(checkpoint_dir, output_dir, *, base_model_path=None) -> Path:
    payloads = _payloads(checkpoint_dir)
    cfg = payloads[0].get("config") or {}
    lora_cfg = dict(cfg.get("lora") or {})
    base = str(base_model_path or (cfg.get("model") or {}).get("model_path") or "")
    tensors: dict[str, torch.Tensor] = {}
    specs: dict[str, tuple[int, int]] = {}
    combined: dict[str, list[dict[str, Any]]] = {}
    for module, items in sorted(_grouped(payloads).items()):
        if any(not rec.get("peft_exportable", True) for rec, _ in items):
            a, b, combined[module] = combine_row_blocks(module, items)
            tensors[f"{PEFT_PREFIX}{module}.lora_A.weight"] = a.contiguous()
            tensors[f"{PEFT_PREFIX}{module}.lora_B.weight"] = b.contiguous()
            specs[module] = (int(a.shape[0]), int(a.shape[0]))
            continue
        a, b = reconstruct_pair(module, items)
        tensors[f"{PEFT_PREFIX}{module}.lora_A.weight"] = a.contiguous()
        tensors[f"{PEFT_PREFIX}{module}.lora_B.weight"] = b.contiguous()
        specs[module] = (int(items[0][0]["r"]), int(items[0][0]["alpha"]))
    if not specs:
        raise ValueError("checkpoint contains no enabled LoRA tensors")
    r0, a0 = next(iter(specs.values()))
    config = {
        "base_model_name_or_path": base,
        "bias": lora_cfg.get("bias", "none"),
        "fan_in_fan_out": False,
        "inference_mode": True,
        "lora_alpha": a0,
        "lora_dropout": float(lora_cfg.get("dropout", 0.0)),
        "peft_type": "LORA",
        "r": r0,
        "target_modules": sorted({m.rsplit(".", 1)[-1] for m in specs}),
        "task_type": lora_cfg.get("task_type", "CAUSAL_LM"),
    }
    rank_pattern = {m: r for m, (r, _) in specs.items() if r != r0}
    alpha_pattern = {m: a for m, (_, a) in specs.items() if a != a0}
    if rank_pattern:
        config["rank_pattern"] = rank_pattern
    if alpha_pattern:
        config["alpha_pattern"] = alpha_pattern
    out = _fresh_dir(output_dir)
    save_file(tensors, str(out / "adapter_model.safetensors"))
    (out / "adapter_config.json").write_text(json.dumps(config, indent=2) + "\n", encoding="utf-8")
    if combined:
        meta = {"format": "graspo-peft-adapter-metadata", "version": 1, "modules": combined}
        (out / METADATA_FILE).write_text(json.dumps(meta, indent=2) + "\n", encoding="utf-8")
    return out


def export_merged_hf(checkpoint_dir, output_dir, *, base_model_path) -> Path:
    base = Path(base_model_path)
    if Path(output_dir).resolve().is_relative_to(base.resolve()):
        raise ValueError("merged-hf output directory must not be inside the base model directory")
    deltas: dict[str, list[tuple[dict, torch.Tensor]]] = {}
    for items in _grouped(_payloads(checkpoint_dir)).values():
        for rec, pair in items:
            delta = (pair["B"].float() @ pair["A"].float()) * (float(rec["alpha"]) / float(rec["r"]))
            deltas.setdefault(rec["base_weight_name"], []).append((rec, delta))
    out = _fresh_dir(output_dir)
    for item in base.iterdir():
        if item.suffix == ".safetensors" or item.name == "model.safetensors.index.json":
            continue
        if item.is_dir():
            if item.name not in (".git", "__pycache__"):
                shutil.copytree(item, out / item.name, dirs_exist_ok=True)
        else:
            shutil.copy2(item, out / item.name)
    total = 0
    for file in sorted(base.glob("*.safetensors")):
        merged: dict[str, torch.Tensor] = {}
        with safe_open(str(file), framework="pt") as handle:
            for name in handle.keys():
                t = handle.get_tensor(name)
                if name in deltas:
                    w = t.float()
                    for rec, delta in deltas.pop(name):
                        kind = rec["shard_kind"]
                        if kind == "none":
                            w += delta
                        elif kind in ("out", "rows"):
                            w[rec["row_start"] : rec["row_stop"]] += delta
                        elif kind in ("in", "cols"):
                            w[:, rec["col_start"] : rec["col_stop"]] += delta
                        else:
                            raise ValueError(f"unsupported shard kind {kind}")
                    t = w.to(t.dtype)
                merged[name] = t.contiguous()
                total += t.numel() * t.element_size()
        save_file(merged, str(out / file.name), metadata={"format": "pt"})
    if deltas:
        raise ValueError(f"base weights not found for LoRA modules: {sorted(deltas)[:5]}")
    index = base / "model.safetensors.index.json"
    if index.exists():
        data = json.loads(index.read_text())
        data.setdefault("metadata", {})["total_size"] = total
        (out / "model.safetensors.index.json").write_text(json.dumps(data, indent=2) + "\n")
    return out


def export_from_checkpoint(checkpoint_dir, output_dir, *, export_format: str, base_model_path=None) -> Path:
    if export_format == "peft-adapter":
        return export_peft_adapter(checkpoint_dir, output_dir, base_model_path=base_model_path)
    if export_format == "merged-hf":
        if not base_model_path:
            cfg = _payloads(checkpoint_dir)[0].get("config") or {}
            base_model_path = (cfg.get("model") or {}).get("model_path")
        if not base_model_path:
            raise ValueError("merged-hf export needs the base model path")
        return export_merged_hf(checkpoint_dir, output_dir, base_model_path=base_model_path)
    raise ValueError(f"Unsupported export format: {export_format}")


def _fresh_dir(path) -> Path:
    out = Path(path)
    if out.exists() and any(out.iterdir()):
        raise FileExistsError(f"Output directory is not empty: {out}")
    out.mkdir(parents=True, exist_ok=True)
    return out


def _parse_key(key: str) -> tuple[str, str]:
    value = key[len(PEFT_PREFIX):] if key.startswith(PEFT_PREFIX) else key
    for marker, which in ((".lora_A.default.weight", "A"), (".lora_B.default.weight", "B"),
                          (".lora_A.weight", "A"), (".lora_B.weight", "B")):
        if value.endswith(marker):
            return value[: -len(marker)], which
    raise ValueError(f"Unsupported PEFT LoRA tensor key: {key}")


def _module_int(config: dict, module: str, pattern: str, default: str) -> int | None:
    pat = config.get(pattern)
    if isinstance(pat, dict):
        for key in (module, f"{PEFT_PREFIX}{module}", module.rsplit(".", 1)[-1]):
            if key in pat:
                return int(pat[key])
    return int(config[default]) if default in config else None


def load_peft_adapter(model, adapter_path, *, base_model_path: str | None = None) -> None:
    """Warm-start the model's LoRA tensors from a PEFT adapter directory."""
    path = Path(adapter_path)
    cfg_file, tensor_file = path / "adapter_config.json", path / "adapter_model.safetensors"
    if not cfg_file.exists():
        raise FileNotFoundError(f"Missing PEFT adapter_config.json: {cfg_file}")
    if not tensor_file.exists():
        raise FileNotFoundError(f"Missing PEFT adapter_model.safetensors: {tensor_file}")
    config = json.loads(cfg_file.read_text(encoding="utf-8"))
    expected = str(config.get("base_model_name_or_path") or "")
    if base_model_path and expected and expected != str(base_model_path):
        raise ValueError(f"PEFT adapter base_model_name_or_path {expected} does not match {base_model_path}")
    grouped: dict[str, dict[str, torch.Tensor]] = {}
    for key, tensor in load_file(str(tensor_file), device="cpu").items():
        module, which = _parse_key(key)
        grouped.setdefault(module, {})[which] = tensor
    incomplete = [m for m, p in grouped.items() if set(p) != {"A", "B"}]
    if incomplete:
        raise ValueError("PEFT adapter has incomplete LoRA A/B pairs: " + ", ".join(incomplete))
    adapter = model.lora
    meta_file = path / METADATA_FILE
    combined = json.loads(meta_file.read_text(encoding="utf-8")).get("modules", {}) if meta_file.exists() else {}
    consumed = set()
    for mod in adapter.modules:
        pair = grouped.get(mod.hf_module_path)
        if pair is None:
            raise ValueError(f"PEFT adapter is missing LoRA tensors for {mod.hf_module_path}")
        if not mod.peft_exportable:
            base_name = f"{mod.hf_module_path}.weight"
            hits = [s for s in combined.get(mod.hf_module_path, [])
                    if s.get("target_name") == mod.target_name and s.get("base_weight_name") == base_name]
            if len(hits) != 1:
                raise ValueError(f"PEFT adapter has no unique {METADATA_FILE} slice for {mod.target_name} "
                                 f"in {mod.hf_module_path}")
            rs, re_ = int(hits[0]["rank_start"]), int(hits[0]["rank_stop"])
            scale = float(hits[0].get("adapter_b_scale") or 1.0)
            a = pair["A"][rs:re_]
            b = pair["B"][mod.row_start : mod.row_stop, rs:re_] / scale
            if tuple(a.shape) != tuple(mod.a.shape) or tuple(b.shape) != tuple(mod.b.shape):
                raise ValueError(f"shape mismatch for {mod.target_name} in {mod.hf_module_path}")
            mod.a.copy_(a.float())
            mod.b.copy_(b.float())
            consumed.add(mod.hf_module_path)
            continue
        r = _module_int(config, mod.hf_module_path, "rank_pattern", "r")
        if r is not None and r != adapter.r:
            raise ValueError(f"PEFT adapter r={r} does not match native LoRA r={adapter.r}")
        alpha = _module_int(config, mod.hf_module_path, "alpha_pattern", "lora_alpha")
        if alpha is not None and float(alpha) != float(adapter.alpha):
            raise ValueError(f"PEFT adapter lora_alpha={alpha} does not match native alpha={adapter.alpha}")
        a, b = pair["A"], pair["B"]
        if mod.shard_kind == "in":
            a = a[:, mod.col_start : mod.col_stop]
        elif mod.shard_kind in ("out", "rows"):
            b = b[mod.row_start : mod.row_stop]
        if tuple(a.shape) != tuple(mod.a.shape) or tuple(b.shape) != tuple(mod.b.shape):
            raise ValueError(f"shape mismatch for {mod.hf_module_path}: adapter A{tuple(a.shape)} B{tuple(b.shape)}, "
                             f"native A{tuple(mod.a.shape)} B{tuple(mod.b.shape)}")
        mod.a.copy_(a.float())
        mod.b.copy_(b.float())
        consumed.add(mod.hf_module_path)
    extra = sorted(set(grouped) - consumed)
    pipeline_stage = len(model.local_layers) < model.cfg.num_hidden_layers
    if extra and not pipeline_stage:
        raise ValueError("PEFT adapter contains unsupported LoRA target(s): " + ", ".join(extra))
    adapter.invalidate()


load_peft_adapter_into_native_model = load_peft_adapter
