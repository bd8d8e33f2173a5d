"""Pipeline stages of the Qwen3.5 hybrid decoder on CPU ranks (gloo).

PP = 2 and TP = 2 x PP = 2: pipelined log-probs, the 1F1B / GPipe gradients
of a weighted log-prob loss and pipelined sampling equal the single-process
model's; then a TP = 2 x PP = 2 ``graspo launch`` runs one GRPO step.
Reference behaviour: models/qwen35_36/training.py:567-1043 (simple and 1F1B
PPO over pipeline stages), logprobs.py:65-121 (stage-sequential log-probs).
"""

import os
import zlib

import pytest
import torch

from tests.dist_util import run_world

TARGETS = {"language.full_attn.q_proj", "language.full_attn.v_proj", "language.full_attn.o_proj",
           "language.linear_attn.q_proj", "language.linear_attn.v_proj", "language.linear_attn.in_proj_z",
           "language.linear_attn.out_proj", "language.mlp.gate_proj", "language.mlp.down_proj"}


def _model(path, ps, layers=None, embed=True, head=True):
    from graspo_b200.models.config import load_decoder_config
    from graspo_b200.models.loader import SafetensorIndex
    from graspo_b200.models.qwen35 import Qwen35Model

    m = Qwen35Model(load_decoder_config(path), SafetensorIndex(path), ps=ps, local_layers=layers,
                    include_embed=embed, include_head=head, lora_targets=TARGETS, lora_r=4, lora_alpha=8,
                    dtype=torch.float32, seed=2)
    with torch.no_grad():
        for mod in m.lora.modules:
            g = torch.Generator().manual_seed(zlib.crc32(mod.module_name.encode()))
            full = torch.randn(mod.out_full, m.lora.r, generator=g) * 0.1
            mod.b.copy_(full if mod.shard_kind == "in" else full[mod.row_start : mod.row_stop])
    return m


def _batch():
    g = torch.Generator().manual_seed(0)
    ids = torch.randint(0, 500, (3, 40), generator=g)
    mask = torch.ones(3, 40, dtype=torch.bool)
    mask[1, :7] = False
    w = torch.randn(3, 39, generator=g) * (mask[:, :-1] & mask[:, 1:])
    return ids, mask, w


KW = dict(group_size=2, max_new_tokens=6, temperature=1.0, top_p=1.0, eos_id=508, pad_id=508, ignore_eos=True,
          seed=5)
PROMPTS = [[5, 6, 7], list(range(20, 45))]


def _reference(path, out):
    from graspo_b200.models.qwen3 import EagerLoRA
    from graspo_b200.models.qwen35 import HybridRolloutEngine
    from graspo_b200.parallel.state import ParallelState

    m = _model(path, ParallelState())
    ids, mask, w = _batch()
    lora = EagerLoRA(m.lora, requires_grad=True)
    lp = m.sequence_logprobs(ids, mask, lora=lora, training=True)
    (lp * w).sum().backward()
    lora.accumulate_grads()
    full = {}
    for mod in m.lora.modules:
        b = mod.b_grad.clone()
        if mod.shard_kind != "in":
            b = torch.zeros(mod.out_full, b.shape[1])
            b[mod.row_start : mod.row_stop] = mod.b_grad
        full[mod.module_name] = (mod.a_grad.clone(), b)
    tokens = HybridRolloutEngine(m).generate(PROMPTS, **KW).tokens
    torch.save({"lp": lp.detach(), "grads": full, "tokens": tokens}, out)


def _worker(rank, world, path, ref_file, tp):
    from graspo_b200.engine.pipeline import pp_logprobs_autograd, pp_train_autograd
    from graspo_b200.models.qwen35 import HybridRolloutEngine
    from graspo_b200.parallel import state as pstate
    from graspo_b200.parallel.p2p import StageComm

    ps = pstate.initialize(tp, 2, 0, timeout_sec=120, device="cpu")
    comm = StageComm(ps)
    first = ps.is_first_stage
    m = _model(path, ps, [0, 1] if first else [2, 3], first, not first)
    ref = torch.load(ref_file)
    ids, mask, w = _batch()
    valid = mask[:, :-1] & mask[:, 1:]
    lp = pp_logprobs_autograd(m, comm, ids, mask, ids[:, 1:], chunk_rows=2)
    assert (lp - ref["lp"]).abs()[valid].max().item() < 1e-4
    from graspo_b200.utils.timing import PhaseClock

    for schedule in ("one_f_one_b", "simple"):
        m.lora.grads.zero_()
        clock = PhaseClock()
        loss = pp_train_autograd(m, comm, ids, mask, ids[:, 1:], lambda lp_c, sl: (lp_c * w[sl]).sum(),
                                 chunk_rows=1, schedule=schedule, clock=clock)
        # stage timers in the reference's key names
        want = {"pipeline_stage_compute_sec", "pipeline_backward_autograd_sec",
                "pipeline_send_sec" if first else "pipeline_recv_sec"}
        assert want <= set(clock.sec), (schedule, sorted(clock.sec))
        # 1F1B: the first stage warms up (fill), the last runs steady only; GPipe: fill then drain
        phases = {"fill_sec", "drain_sec"} if schedule == "simple" else ({"fill_sec", "steady_sec", "drain_sec"}
                                                                         if first else {"steady_sec"})
        assert {k for k in clock.sec if k in ("fill_sec", "steady_sec", "drain_sec")} == phases, sorted(clock.sec)
        assert clock.calls["pipeline_forward_calls"] == 3
        assert abs(loss.item() - (ref["lp"] * w).sum().item()) < 1e-3
        if tp > 1:
            torch.distributed.all_reduce(m.lora.grads[: m.lora.replicated_numel], group=ps.tp_group)
        for mod in m.lora.modules:
            ra, rb = ref["grads"][mod.module_name]
            want_a = ra[:, mod.col_start : mod.col_stop] if mod.shard_kind == "in" else ra
            want_b = rb if mod.shard_kind == "in" else rb[mod.row_start : mod.row_stop]
            for got, want in ((mod.a_grad, want_a), (mod.b_grad, want_b)):
                err = (got - want).abs().max().item()
                assert err <= 1e-4 * (want.abs().max().item() + 1e-3), (schedule, mod.module_name, err)
    got = HybridRolloutEngine(m, comm=comm).generate(PROMPTS, **KW)
    assert torch.equal(got.tokens, ref["tokens"]), (got.tokens, ref["tokens"])
    pstate.destroy()


@pytest.mark.parametrize("tp", [1, 2])
def test_qwen35_pipeline_matches_single_process(tmp_path, tp):
    from graspo_b200.utils.synth import QWEN35_TINY, write_qwen35_checkpoint

    os.environ.setdefault("GLOO_SOCKET_IFNAME", "lo")
    path = write_qwen35_checkpoint(tmp_path / "q35", QWEN35_TINY, seed=1, std=0.05, with_tokenizer=False)
    ref_file = tmp_path / "ref.pt"
    _reference(path, ref_file)
    run_world(2 * tp, _worker, path, ref_file, tp, timeout=600)


@pytest.mark.slow
@pytest.mark.parametrize("method", ["graspo", "sft"])
def test_qwen35_tp2_pp2_launch(tmp_path, method):
    """`graspo launch` at TP = 2 x PP = 2 (4 CPU ranks, 1F1B): one GRPO step (or one
    supervised step) and a final checkpoint."""
    import subprocess
    import sys
    from pathlib import Path

    import yaml

    from graspo_b200.utils.synth import QWEN35_TINY, synthetic_json_records, write_jsonl_records, \
        write_qwen35_checkpoint

    root = Path(__file__).resolve().parents[1]
    model = write_qwen35_checkpoint(tmp_path / "q35", QWEN35_TINY, seed=1, std=0.05, dtype=torch.float32)
    data = write_jsonl_records(synthetic_json_records(4, seed=0), tmp_path / "train.jsonl")
    cfg = yaml.safe_load((root / "configs" / "config0_cpu_tp2.yaml").read_text())
    cfg["model"]["model_path"] = str(model)
    cfg["data"]["train_path"] = str(data)
    cfg["lora"]["target_modules"] = sorted(TARGETS)
    cfg["training"].update(output_dir=str(tmp_path / "run"), max_steps=1, max_new_tokens=12, rollout_group_size=2,
                           learning_rate=1e-3)
    cfg["graspoflow"].update(tp_size=2, pp_size=2, pg_timeout_sec=60.0, pp_schedule="one_f_one_b",
                             pp_micro_batch_size=1)
    cfg["launch"].update(nproc_per_node=4, master_port=29000 + (os.getpid() * 3) % 2000)
    cfg["train_method"] = method
    if method == "sft":
        cfg.pop("reward", None)
    path = tmp_path / "q35_tp2_pp2.yaml"
    path.write_text(yaml.safe_dump(cfg))
    env = {k: v for k, v in os.environ.items() if not k.startswith("GRASPO_FAULT")}
    env.update(PYTHONPATH=str(root), CUDA_VISIBLE_DEVICES="")
    proc = subprocess.run([sys.executable, "-m", "graspo_b200", "launch", "--config", str(path)], env=env,
                          capture_output=True, text=True, timeout=900, cwd=root)
    assert proc.returncode == 0, proc.stdout[-3000:] + proc.stderr[-3000:]
    final = tmp_path / "run" / "final"
    assert (final / "manifest.json").exists()
    assert len(list(final.glob("rank_*_tp_*_pp_*.pt"))) == 4
