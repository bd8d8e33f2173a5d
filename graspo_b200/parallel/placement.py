"""Layer-to-pipeline-stage placement.

A plan says which decoder layers a stage owns, and whether it owns the
embedding (first stage) and the final norm + LM head (last stage).

Strategies (reference: placement.py:57-223; the stage boundaries must come
out identical so pipeline checkpoints are interchangeable):

* ``manual`` -- ``graspoflow.layer_ranges``: one ``[start, end)`` per stage,
  contiguous and covering every layer exactly once.
* ``qwen36_pp8_static`` -- minimise the most loaded stage, with a layer cost of
  1.18 for full attention and 1.0 for linear attention, plus fixed stage
  overheads 1.5*pp/8 on the first stage (embedding) and 8.0*pp/8 on the last
  (norm + LM head + loss).  Solved exactly by dynamic programming over
  contiguous splits.
* ``qwen36_pp8_lm_head_only_final`` -- the same split over pp-1 stages; the
  last stage holds only the head.
* ``dense_balanced`` -- the minimax split for dense decoders (every layer
  costs 1.0); the default for ``qwen3`` with pp > 1 (the reference has no
  dense-model pipeline placement).
"""

from __future__ import annotations

from dataclasses import dataclass
from typing import Any


@dataclass(frozen=True, slots=True)
class NativePlacementPlan:
    strategy: str
    model_family: str
    tp_size: int
    pp_size: int
    pp_rank: int
    tp_rank: int
    local_layer_indices: tuple[int, ...]
    include_embeddings: bool
    include_lm_head: bool

    @property
    def is_pipeline(self) -> bool:
        return self.pp_size > 1


def validate_manual_ranges(ranges: list[list[int]], num_hidden_layers: int) -> None:
    covered: list[int] = []
    for i, (start, end) in enumerate(ranges):
        if start >= end:
            raise ValueError(f"layer_ranges[{i}]=[{start},{end}) is invalid: start must be < end")
        covered.extend(range(start, end))
    if set(covered) != set(range(num_hidden_layers)) or len(covered) != num_hidden_layers:
        raise ValueError(f"layer_ranges covers {len(set(covered))} layers, but model has {num_hidden_layers} layers")
    for i in range(len(ranges) - 1):
        if ranges[i][1] != ranges[i + 1][0]:
            raise ValueError(
                f"layer_ranges[{i}] ends at {ranges[i][1]} but layer_ranges[{i + 1}] starts at "
                f"{ranges[i + 1][0]}: ranges must be contiguous without gaps or overlaps"
            )


def minimax_contiguous_ranges(costs: list[float], overheads: list[float]) -> list[tuple[int, int]]:
    """Split ``costs`` into ``len(overheads)`` contiguous non-empty stages
    minimising the maximum (stage cost + stage overhead).

    Bottom-up DP over (first layer of the suffix, stage index); ties keep the
    earliest boundary.
    """
    n, stages = len(costs), len(overheads)
    if stages > n:
        raise ValueError("pp_size cannot exceed num_hidden_layers")
    prefix = [0.0]
    for c in costs:
        prefix.append(prefix[-1] + float(c))
    inf = float("inf")
    # value[s][i]: best max-load for layers i.. on stages s..; cut[s][i]: end of stage s
    value = [[inf] * (n + 1) for _ in range(stages)]
    cut = [[-1] * (n + 1) for _ in range(stages)]
    last = stages - 1
    for i in range(n):
        value[last][i] = prefix[n] - prefix[i] + overheads[last]
        cut[last][i] = n
    for s in range(stages - 2, -1, -1):
        remaining = stages - s - 1
        for i in range(n - remaining):
            best, where = inf, -1
            for stop in range(i + 1, n - remaining + 1):
                load = max(prefix[stop] - prefix[i] + overheads[s], value[s + 1][stop])
                if load < best:
                    best, where = load, stop
            value[s][i], cut[s][i] = best, where
    ranges, start = [], 0
    for s in range(stages):
        stop = cut[s][start]
        ranges.append((start, stop))
        start = stop
    return ranges


def _layer_costs(num_layers: int, layer_types, dense: bool) -> list[float]:
    if dense:
        return [1.0] * num_layers
    types = list(layer_types or [])
    if len(types) != num_layers:
        types = ["linear_attention"] * num_layers
    return [1.18 if t == "full_attention" else 1.0 for t in types]


def build_placement_plan(
    *,
    strategy: str,
    model_family: str,
    num_hidden_layers: int,
    tp_size: int,
    pp_size: int,
    tp_rank: int,
    pp_rank: int,
    layer_types=None,
    manual_ranges: list[list[int]] | None = None,
) -> NativePlacementPlan:
    name = (strategy or "auto").strip()
    if name == "auto":
        if pp_size > 1:
            name = "qwen36_pp8_static" if model_family == "qwen3_5_text" else "dense_balanced"
        else:
            name = "qwen3_tp"

    def plan(local: tuple[int, ...], strat: str) -> NativePlacementPlan:
        return NativePlacementPlan(
            strategy=strat, model_family=model_family, tp_size=int(tp_size), pp_size=int(pp_size),
            pp_rank=int(pp_rank), tp_rank=int(tp_rank), local_layer_indices=local,
            include_embeddings=int(pp_rank) == 0, include_lm_head=int(pp_rank) == int(pp_size) - 1,
        )

    if pp_size == 1:
        return plan(tuple(range(int(num_hidden_layers))), name)
    if manual_ranges is not None and len(manual_ranges) == int(pp_size):
        validate_manual_ranges(manual_ranges, int(num_hidden_layers))
        start, end = manual_ranges[int(pp_rank)]
        return plan(tuple(range(start, end)), "manual")
    scale = float(pp_size) / 8.0
    if name == "dense_balanced":
        over = [0.0] * pp_size
        over[0], over[-1] = 1.5 * scale, 8.0 * scale
        ranges = minimax_contiguous_ranges(_layer_costs(num_hidden_layers, layer_types, True), over)
    elif name in ("qwen36_pp8_static", "qwen36_pp8_lm_head_only_final"):
        if model_family != "qwen3_5_text":
            raise ValueError(f"{name} placement requires qwen3_5_text model family")
        costs = _layer_costs(num_hidden_layers, layer_types, False)
        if name == "qwen36_pp8_static":
            over = [0.0] * pp_size
            over[0], over[-1] = 1.5 * scale, 8.0 * scale
            ranges = minimax_contiguous_ranges(costs, over)
        else:
            if pp_size < 2:
                raise ValueError("lm-head-only final placement requires at least two pipeline stages")
            over = [0.0] * (pp_size - 1)
            over[0] = 1.5
            ranges = [*minimax_contiguous_ranges(costs, over), (num_hidden_layers, num_hidden_layers)]
    else:
        raise ValueError(f"Unsupported pipeline placement strategy: {name}")
    return plan(tuple(range(*ranges[int(pp_rank)])), name)


def placement_summary(plan: NativePlacementPlan | None) -> dict[str, Any] | None:
    if plan is None:
        return None
    return {
        "placement_strategy": plan.strategy,
        "model_family": plan.model_family,
        "tp_size": plan.tp_size,
        "pp_size": plan.pp_size,
        "tp_rank": plan.tp_rank,
        "pp_rank": plan.pp_rank,
        "local_layer_indices": list(plan.local_layer_indices),
        "include_embeddings": plan.include_embeddings,
        "include_lm_head": plan.include_lm_head,
    }
