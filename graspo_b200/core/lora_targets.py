"""LoRA target selection: presets, exact names and globs over canonical names.

Canonical target names look like ``language.self_attn.q_proj`` or
``visual.blocks.3.attn.qkv``.  Resolution is fail-closed: every requested
pattern must match at least one target the model advertises, and the result
must be non-empty (reference: src/graspo/core/lora.py:10-85).  Presets expand to
several patterns; a preset pattern that names a module kind the model family
does not have (e.g. ``in_proj_z`` on a dense Qwen3) is skipped rather than
failing the whole preset.
"""

from __future__ import annotations

from collections.abc import Iterable
from dataclasses import dataclass
from fnmatch import fnmatchcase

LORA_TARGET_PRESETS: dict[str, tuple[str, ...]] = {
    "language_safe": ("language.*.q_proj", "language.*.v_proj"),
    "language_all_linear": (
        "language.*.q_proj",
        "language.*.k_proj",
        "language.*.v_proj",
        "language.*.o_proj",
        "language.*.in_proj_z",
        "language.*.out_proj",
        "language.*.gate_proj",
        "language.*.up_proj",
        "language.*.down_proj",
    ),
    "vision_merger": ("visual.merger.linear_fc1", "visual.merger.linear_fc2"),
    "vision_common": (
        "visual.merger.linear_fc1",
        "visual.merger.linear_fc2",
        "visual.blocks.*.attn.*",
        "visual.blocks.*.mlp.linear_fc*",
    ),
}


@dataclass(frozen=True, slots=True)
class ResolvedLoRATargets:
    requested: tuple[str, ...]
    resolved: tuple[str, ...]

    @property
    def signature(self) -> dict[str, object]:
        return {"requested": list(self.requested), "resolved": list(self.resolved)}


def _matches(pattern: str, available: tuple[str, ...]) -> list[str]:
    if any(ch in pattern for ch in "*?[]"):
        return [name for name in available if fnmatchcase(name, pattern)]
    return [name for name in available if name == pattern]


def resolve_lora_target_modules(
    requested: Iterable[str] | None,
    *,
    available: Iterable[str],
    default_preset: str = "language_safe",
) -> ResolvedLoRATargets:
    avail = tuple(sorted({str(a) for a in available}))
    asked = tuple(str(r) for r in (requested or (default_preset,)))
    resolved: set[str] = set()
    unsupported: list[str] = []
    for item in asked:
        preset = LORA_TARGET_PRESETS.get(item)
        if preset is None:
            hits = _matches(item, avail)
            if not hits:
                unsupported.append(item)
            resolved.update(hits)
            continue
        preset_hits = [hit for pattern in preset for hit in _matches(pattern, avail)]
        if not preset_hits:
            unsupported.append(item)
        resolved.update(preset_hits)
    if unsupported:
        raise ValueError(
            "Unsupported LoRA target(s): "
            + ", ".join(unsupported)
            + ". Available targets: "
            + ", ".join(avail)
        )
    if not resolved:
        raise ValueError("LoRA target resolution produced no trainable modules")
    return ResolvedLoRATargets(requested=asked, resolved=tuple(sorted(resolved)))


def lora_target_enabled(targets: set[str] | frozenset[str], canonical_name: str) -> bool:
    """A module is adapted if its canonical name or its leaf name was resolved."""
    return canonical_name in targets or canonical_name.rsplit(".", 1)[-1] in targets
