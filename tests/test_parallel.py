"""Schedules, placement, dataflow operators and multi-rank (gloo) equivalence."""

import os
import zlib

import pytest
import torch

from graspo_b200.parallel.operator import ComputeOperator, Microbatch, OpBuffer, PipelineGraph
from graspo_b200.parallel.placement import build_placement_plan, minimax_contiguous_ranges, validate_manual_ranges
from graspo_b200.parallel.schedule import PipelineAction, get_scheduler, peak_inflight

from tests.dist_util import run_world


def test_gpipe_and_1f1b_plans():
    g = get_scheduler("simple", pp_size=4, pp_rank=0).plan(3)
    assert [repr(s) for s in g] == ["forward(0)", "forward(1)", "forward(2)", "backward(2)", "backward(1)", "backward(0)"]
    s = get_scheduler("one_f_one_b", pp_size=4, pp_rank=1)
    plan = s.plan(6)
    assert [st.microbatch_idx for st in plan if st.action == PipelineAction.FORWARD] == list(range(6))
    assert [st.microbatch_idx for st in plan if st.action == PipelineAction.BACKWARD] == list(range(6))
    assert peak_inflight(plan) == 3  # warmup (pp-rank-1 = 2) + 1
    assert peak_inflight(get_scheduler("1f1b", pp_size=4, pp_rank=3).plan(6)) == 1
    assert peak_inflight(get_scheduler("1f1b", pp_size=4, pp_rank=0).plan(6, max_inflight=1)) == 2
    phases = s.plan_phases(6)
    assert len(phases["fill"]) == 2 and len(phases["drain"]) == 2
    with pytest.raises(ValueError):
        get_scheduler("nope", pp_size=2, pp_rank=0)


def test_schedule_phases_keep_the_plan_order():
    from graspo_b200.utils.timing import schedule_phases

    for name in ("simple", "one_f_one_b"):
        for rank in range(4):
            sch = get_scheduler(name, pp_size=4, pp_rank=rank)
            pairs = schedule_phases(sch, 6)
            assert [step for _, step in pairs] == sch.plan(6)
            assert {p for p, _ in pairs} <= {"fill", "steady", "drain"}


def test_minimax_placement():
    ranges = minimax_contiguous_ranges([1.0] * 8, [0.0, 0.0])
    assert ranges == [(0, 4), (4, 8)]
    # heavy last stage gets fewer layers
    ranges = minimax_contiguous_ranges([1.0] * 64, [1.5 * 0.5, 0, 0, 8.0 * 0.5])
    sizes = [b - a for a, b in ranges]
    assert sum(sizes) == 64 and sizes[-1] < sizes[1]
    plan = build_placement_plan(strategy="auto", model_family="qwen3", num_hidden_layers=64, tp_size=2, pp_size=4,
                                tp_rank=1, pp_rank=3)
    assert plan.include_lm_head and not plan.include_embeddings and plan.strategy == "dense_balanced"
    manual = build_placement_plan(strategy="auto", model_family="qwen3", num_hidden_layers=4, tp_size=1, pp_size=2,
                                  tp_rank=0, pp_rank=1, manual_ranges=[[0, 1], [1, 4]])
    assert manual.local_layer_indices == (1, 2, 3) and manual.strategy == "manual"
    with pytest.raises(ValueError):
        validate_manual_ranges([[0, 2], [3, 4]], 4)
    hybrid = build_placement_plan(strategy="qwen36_pp8_lm_head_only_final", model_family="qwen3_5_text",
                                  num_hidden_layers=16, tp_size=1, pp_size=4, tp_rank=0, pp_rank=3)
    assert hybrid.local_layer_indices == ()


class _Double(ComputeOperator):
    def forward(self, mb):
        mb.tensors["x"] = mb.tensors["x"] * 2
        return mb

    def backward(self, mb):
        mb.meta.setdefault("bwd", []).append(self.name)
        return mb


def test_opbuffer_backpressure_and_graph():
    buf = OpBuffer(2)
    assert buf.push(Microbatch(0)) and buf.push(Microbatch(1)) and not buf.push(Microbatch(2))
    assert buf.is_full and buf.waterlevel == 1.0 and buf.pop().idx == 0
    graph = PipelineGraph([_Double(name="a"), _Double(name="b")])
    inputs = {i: Microbatch(i, {"x": torch.ones(2)}) for i in range(3)}
    out = graph.execute_plan(get_scheduler("1f1b", pp_size=2, pp_rank=0).plan(3), inputs)
    assert all(torch.equal(out[i].tensors["x"], torch.full((2,), 4.0)) for i in range(3))
    assert inputs[0].meta["bwd"] == ["b", "a"]


# ---------------------------------------------------------------- gloo worlds
TINY_TARGETS = {"language.self_attn.q_proj", "language.self_attn.k_proj", "language.self_attn.v_proj",
                "language.self_attn.o_proj", "language.mlp.gate_proj", "language.mlp.up_proj", "language.mlp.down_proj"}


def _tiny_ckpt(tmp):
    from graspo_b200.utils.synth import TINY, write_qwen3_checkpoint

    return write_qwen3_checkpoint(tmp, TINY, seed=7, std=0.05, device="cpu", with_tokenizer=False)


def _grads_for(tp, rank_unused, path, batch):
    from graspo_b200.models.config import load_decoder_config
    from graspo_b200.models.loader import SafetensorIndex
    from graspo_b200.models.qwen3 import EagerLoRA, Qwen3Model, eager_stage_forward, eager_token_logprobs
    from graspo_b200.parallel import state as pstate

    ps = pstate.initialize(tp, 1, 0, timeout_sec=60, device="cpu")
    m = Qwen3Model(load_decoder_config(path), SafetensorIndex(path), ps=ps, lora_targets=TINY_TARGETS, lora_r=4,
                   lora_alpha=8, lora_dropout=0.0, dtype=torch.float32, device=ps.device, seed=3)
    with torch.no_grad():  # make B non-zero (same on every rank: seeded by module name)
        for mod in m.lora.modules:
            g = torch.Generator().manual_seed(zlib.crc32(mod.module_name.encode()))
            full = torch.randn(mod.out_full, m.lora.r, generator=g) * 0.1
            mod.b.copy_(full[mod.row_start : mod.row_stop] if mod.shard_kind == "out" else full)
    seq, mask = batch
    lora = EagerLoRA(m.lora, requires_grad=True)
    hidden = eager_stage_forward(m, seq, mask, lora=lora, training=True)
    lp = eager_token_logprobs(m, hidden[:, :-1], seq[:, 1:])
    (lp * mask[:, 1:]).sum().backward()
    lora.accumulate_grads()
    if ps.tp_size > 1:
        rep = m.lora.replicated_numel
        torch.distributed.all_reduce(m.lora.grads[:rep], group=ps.tp_group)
    out = {}
    for mod in m.lora.modules:
        out[mod.module_name] = (mod.a_grad.clone(), mod.b_grad.clone(), mod.shard_kind, mod.row_start, mod.row_stop,
                                mod.col_start, mod.col_stop)
    return out, lp.detach()


def _tp2_worker(rank, world, path, batch, ref_file):
    grads, lp = _grads_for(2, rank, path, batch)
    ref = torch.load(ref_file)
    assert torch.allclose(lp, ref["lp"], atol=1e-5), (lp - ref["lp"]).abs().max()
    for name, (ga, gb, kind, r0, r1, c0, c1) in grads.items():
        ra, rb = ref["grads"][name]
        if kind == "out":
            assert torch.allclose(ga, ra, atol=1e-5, rtol=1e-4), name
            assert torch.allclose(gb, rb[r0:r1], atol=1e-5, rtol=1e-4), name
        else:
            assert torch.allclose(ga, ra[:, c0:c1], atol=1e-5, rtol=1e-4), name
            assert torch.allclose(gb, rb, atol=1e-5, rtol=1e-4), name
    torch.distributed.destroy_process_group()


@pytest.mark.slow
def test_tp2_lora_grads_equal_tp1(tmp_path):
    path = _tiny_ckpt(tmp_path / "ckpt")
    g = torch.Generator().manual_seed(0)
    seq = torch.randint(0, 2040, (2, 24), generator=g)
    mask = torch.ones(2, 24, dtype=torch.bool)
    mask[0, :5] = False
    os.environ.pop("WORLD_SIZE", None)
    grads, lp = _grads_for(1, 0, path, (seq, mask))
    from graspo_b200.parallel import state as pstate

    pstate.destroy()
    ref_file = tmp_path / "ref.pt"
    torch.save({"grads": {k: (v[0], v[1]) for k, v in grads.items()}, "lp": lp}, ref_file)
    run_world(2, _tp2_worker, path, (seq, mask), ref_file)


def _dp2_worker(rank, world, path, batch, ref_file):
    """DP = 2: each replica takes half the rows; the mean-loss gradients averaged
    over the replicas (the adapter's DP step) equal the single-replica gradients
    of the whole batch, and the replica check passes."""
    from types import SimpleNamespace

    from graspo_b200.engine.adapter import Qwen3Adapter
    from graspo_b200.models.config import load_decoder_config
    from graspo_b200.models.loader import SafetensorIndex
    from graspo_b200.models.qwen3 import EagerLoRA, Qwen3Model, eager_stage_forward, eager_token_logprobs
    from graspo_b200.parallel import state as pstate

    ps = pstate.initialize(1, 1, 2, timeout_sec=60, device="cpu")
    assert ps.dp_size == 2 and ps.tp_size == 1
    m = Qwen3Model(load_decoder_config(path), SafetensorIndex(path), ps=ps, lora_targets=TINY_TARGETS, lora_r=4,
                   lora_alpha=8, lora_dropout=0.0, dtype=torch.float32, device=ps.device, seed=3)
    with torch.no_grad():
        m.lora.params.copy_(torch.load(ref_file)["params"])
    seq, mask = batch
    half = seq.shape[0] // 2
    rows = slice(rank * half, (rank + 1) * half)
    lora = EagerLoRA(m.lora, requires_grad=True)
    hidden = eager_stage_forward(m, seq[rows], mask[rows], lora=lora, training=True)
    lp = eager_token_logprobs(m, hidden[:, :-1], seq[rows, 1:])
    w = mask[rows, 1:].float()
    ((lp * w).sum() / w.sum()).backward()
    lora.accumulate_grads()
    fake = SimpleNamespace(ps=ps, model=m, _dp_reducer=lambda: None)  # CPU ranks: the library all-reduce
    Qwen3Adapter._dp_average_grads(fake)
    ref = torch.load(ref_file)["grads"]
    assert torch.allclose(m.lora.grads, ref, atol=1e-6, rtol=1e-4), (m.lora.grads - ref).abs().max()
    Qwen3Adapter.check_replicas(fake)   # identical parameters on both replicas
    if rank == 1:
        with torch.no_grad():
            m.lora.params[0] += 1.0
    try:
        Qwen3Adapter.check_replicas(fake)
    except RuntimeError as exc:
        assert "lora (dp)" in str(exc)
    else:
        raise AssertionError("a diverged replica was not reported")
    torch.distributed.destroy_process_group()


@pytest.mark.slow
def test_dp2_grads_equal_dp1_and_replica_check(tmp_path):
    from graspo_b200.models.config import load_decoder_config
    from graspo_b200.models.loader import SafetensorIndex
    from graspo_b200.models.qwen3 import EagerLoRA, Qwen3Model, eager_stage_forward, eager_token_logprobs
    from graspo_b200.parallel import state as pstate

    path = _tiny_ckpt(tmp_path / "ckpt")
    g = torch.Generator().manual_seed(1)
    seq = torch.randint(0, 2040, (4, 20), generator=g)
    mask = torch.ones(4, 20, dtype=torch.bool)
    mask[0, :4] = False
    mask[3, -3:] = False
    os.environ.pop("WORLD_SIZE", None)
    ps = pstate.initialize(1, 1, timeout_sec=60, device="cpu")
    m = Qwen3Model(load_decoder_config(path), SafetensorIndex(path), ps=ps, lora_targets=TINY_TARGETS, lora_r=4,
                   lora_alpha=8, lora_dropout=0.0, dtype=torch.float32, device=ps.device, seed=3)
    with torch.no_grad():
        m.lora.params.normal_(0, 0.05)
    # the reference: mean over each half, averaged (equal-size halves, per-replica normalisation)
    grads = torch.zeros_like(m.lora.grads)
    for rows in (slice(0, 2), slice(2, 4)):
        m.lora.grads.zero_()
        lora = EagerLoRA(m.lora, requires_grad=True)
        hidden = eager_stage_forward(m, seq[rows], mask[rows], lora=lora, training=True)
        lp = eager_token_logprobs(m, hidden[:, :-1], seq[rows, 1:])
        w = mask[rows, 1:].float()
        ((lp * w).sum() / w.sum()).backward()
        lora.accumulate_grads()
        grads += m.lora.grads / 2
    ref_file = tmp_path / "ref.pt"
    torch.save({"grads": grads, "params": m.lora.params.clone()}, ref_file)
    pstate.destroy()
    run_world(2, _dp2_worker, path, (seq, mask), ref_file)
