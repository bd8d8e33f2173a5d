"""Pipeline placement: layer ranges per stage, manual ranges, minimax balancing,
summary payload, immutability (reference behaviour: parallel/placement.py)."""

import dataclasses

import pytest

from graspo_b200.parallel.placement import (
    NativePlacementPlan,
    build_placement_plan,
    minimax_contiguous_ranges,
    placement_summary,
    validate_manual_ranges,
)


def _plan(pp_rank, pp_size=4, layers=16, **kw):
    return build_placement_plan(strategy=kw.pop("strategy", "auto"), model_family=kw.pop("family", "qwen3"),
                                num_hidden_layers=layers, tp_size=kw.pop("tp", 1), pp_size=pp_size,
                                tp_rank=kw.pop("tp_rank", 0), pp_rank=pp_rank, **kw)


def test_single_stage_holds_everything():
    for tp_rank in (0, 1):
        p = _plan(0, pp_size=1, layers=36, tp=2, tp_rank=tp_rank)
        assert p.local_layer_indices == tuple(range(36)) and p.include_embeddings and p.include_lm_head
        assert p.strategy == "qwen3_tp" and p.tp_rank == tp_rank and not p.is_pipeline


def test_stages_partition_the_layers_contiguously():
    plans = [_plan(r) for r in range(4)]
    layers = [i for p in plans for i in p.local_layer_indices]
    assert layers == list(range(16))
    assert [p.include_embeddings for p in plans] == [True, False, False, False]
    assert [p.include_lm_head for p in plans] == [False, False, False, True]
    assert all(p.local_layer_indices for p in plans) and all(p.is_pipeline for p in plans)
    # the last stage also carries the LM head, so it gets no more layers than a middle stage
    assert len(plans[-1].local_layer_indices) <= len(plans[1].local_layer_indices)


def test_manual_ranges():
    ranges = [[0, 3], [3, 9], [9, 12], [12, 16]]
    plans = [_plan(r, manual_ranges=ranges) for r in range(4)]
    assert [p.local_layer_indices for p in plans] == [tuple(range(a, b)) for a, b in ranges]
    assert all(p.strategy == "manual" for p in plans)
    validate_manual_ranges(ranges, 16)
    for bad, msg in (([[0, 8], [9, 16]], "layers"), ([[0, 9], [8, 16]], "layers"), ([[0, 8], [8, 15]], "layers"),
                     ([[4, 4], [4, 16]], "start must be < end")):
        with pytest.raises(ValueError, match=msg):
            validate_manual_ranges(bad, 16)


def test_minimax_ranges():
    assert minimax_contiguous_ranges([1.0] * 6, [0.0, 0.0, 0.0]) == [(0, 2), (2, 4), (4, 6)]
    assert minimax_contiguous_ranges([5.0], [0.0]) == [(0, 1)]
    heavy_tail = minimax_contiguous_ranges([1.0] * 10, [0.0, 4.0])
    assert heavy_tail[0][1] - heavy_tail[0][0] > heavy_tail[1][1] - heavy_tail[1][0]
    with pytest.raises(ValueError):
        minimax_contiguous_ranges([1.0, 1.0], [0.0, 0.0, 0.0])


def test_hybrid_strategies():
    types = ["linear_attention", "linear_attention", "linear_attention", "full_attention"] * 4
    plans = [_plan(r, family="qwen3_5_text", layer_types=types) for r in range(4)]
    assert plans[0].strategy == "qwen36_pp8_static"
    assert [i for p in plans for i in p.local_layer_indices] == list(range(16))
    final = [_plan(r, family="qwen3_5_text", strategy="qwen36_pp8_lm_head_only_final", layer_types=types)
             for r in range(4)]
    assert final[-1].local_layer_indices == () and final[-1].include_lm_head
    with pytest.raises(ValueError, match="qwen3_5_text"):
        _plan(0, strategy="qwen36_pp8_static")
    with pytest.raises(ValueError, match="Unsupported"):
        _plan(0, strategy="round_robin")


def test_summary_and_immutability():
    p = _plan(2)
    s = placement_summary(p)
    assert set(s) == {"placement_strategy", "model_family", "tp_size", "pp_size", "tp_rank", "pp_rank",
                      "local_layer_indices", "include_embeddings", "include_lm_head"}
    assert s["local_layer_indices"] == list(p.local_layer_indices)
    assert placement_summary(None) is None
    with pytest.raises(dataclasses.FrozenInstanceError):
        p.pp_rank = 0
    assert isinstance(p, NativePlacementPlan)
