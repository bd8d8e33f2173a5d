"""Tensor parallelism of the Qwen3.5 hybrid decoder on CPU ranks (gloo, TP=2).

Each rank keeps half of the heads of both layer kinds and half of the MLP;
the log-probs, the LoRA gradients (after the TP sum of the replicated
factors) and the sampled rollouts must equal the TP = 1 model's.  The PEFT
export of the TP shards (``in_proj_qkv`` blocks combined into one pair)
loads back into a TP = 1 model bit-exactly.
Reference behaviour: models/common/layers.py:145-633 (head-row sharding),
lora.py:216-241 (replicated-factor gradient sum), lora_io.py (combined PEFT
pairs for the DeltaNet q/k/v row blocks).
"""

import os
import zlib

import pytest
import torch

from tests.dist_util import run_world

TARGETS = {"language.full_attn.q_proj", "language.full_attn.k_proj", "language.full_attn.v_proj",
           "language.full_attn.o_proj", "language.linear_attn.q_proj", "language.linear_attn.k_proj",
           "language.linear_attn.v_proj", "language.linear_attn.in_proj_z", "language.linear_attn.out_proj",
           "language.mlp.gate_proj", "language.mlp.up_proj", "language.mlp.down_proj"}


def _model(path, ps):
    from graspo_b200.models.config import load_decoder_config
    from graspo_b200.models.loader import SafetensorIndex
    from graspo_b200.models.qwen35 import Qwen35Model

    m = Qwen35Model(load_decoder_config(path), SafetensorIndex(path), ps=ps, lora_targets=TARGETS, lora_r=4,
                    lora_alpha=8, dtype=torch.float32, seed=2, gradient_checkpointing=True)
    with torch.no_grad():  # non-zero B, seeded by module name so every TP layout slices the same full matrix
        for mod in m.lora.modules:
            g = torch.Generator().manual_seed(zlib.crc32(mod.module_name.encode()))
            full = torch.randn(mod.out_full, m.lora.r, generator=g) * 0.1
            mod.b.copy_(full if mod.shard_kind == "in" else full[mod.row_start : mod.row_stop])
    return m


def _batch():
    g = torch.Generator().manual_seed(0)
    ids = torch.randint(0, 500, (2, 70), generator=g)
    mask = torch.ones(2, 70, dtype=torch.bool)
    mask[0, :9] = False
    return ids, mask


def _grads(m, ids, mask):
    from graspo_b200.models.qwen3 import EagerLoRA

    m.lora.grads.zero_()
    lora = EagerLoRA(m.lora, requires_grad=True)
    lp = m.sequence_logprobs(ids, mask, lora=lora, training=True)
    (lp * mask[:, 1:]).sum().backward()
    lora.accumulate_grads()
    return lp.detach()


def _to_full(mod, fac, t):
    """A TP = 1 factor (or gradient) in the coordinates of its whole HF module."""
    if fac == "a" or mod.shard_kind == "in":
        return t.clone()
    full = torch.zeros(mod.out_full, t.shape[1])
    full[mod.row_start : mod.row_stop] = t
    return full


def _local(mod, fac, full):
    """The part of a whole-module factor (or gradient) that this rank's shard holds."""
    if fac == "a":
        return full[:, mod.col_start : mod.col_stop] if mod.shard_kind == "in" else full
    return full if mod.shard_kind == "in" else full[mod.row_start : mod.row_stop]


def _worker(rank, world, path, ref_file, out_dir):
    tp = world
    from graspo_b200.models.lora_io import export_peft_adapter
    from graspo_b200.models.qwen35 import HybridRolloutEngine
    from graspo_b200.parallel import state as pstate
    from graspo_b200.train.checkpoint import rank_file_name

    ps = pstate.initialize(tp, 1, 0, timeout_sec=120, device="cpu")
    m = _model(path, ps)
    ref = torch.load(ref_file)
    ids, mask = _batch()
    lp = _grads(m, ids, mask)
    valid = mask[:, :-1] & mask[:, 1:]
    assert (lp - ref["lp"]).abs()[valid].max().item() < 1e-4
    rep = m.lora.replicated_numel
    torch.distributed.all_reduce(m.lora.grads[:rep], group=ps.tp_group)
    m.sync_partial_grads()        # key/value heads held by several ranks (TP above the KV head count)
    for mod in m.lora.modules:
        for fac, g in (("a", mod.a_grad), ("b", mod.b_grad)):
            want = _local(mod, fac, ref["grads"][mod.module_name][fac])
            err = (g - want).abs().max().item()
            assert err <= 1e-4 * (want.abs().max().item() + 1e-3), (mod.module_name, fac, err)
    kw = dict(group_size=2, max_new_tokens=6, temperature=1.0, top_p=1.0, eos_id=508, pad_id=508,
              ignore_eos=True, seed=5)
    got = HybridRolloutEngine(m).generate([[5, 6, 7], list(range(20, 45))], **kw)
    assert torch.equal(got.tokens, ref["tokens"]), (got.tokens, ref["tokens"])
    # checkpoint shards of both ranks -> one PEFT adapter
    torch.save({"lora_state_dict": m.lora_state_dict(), "lora_tensor_metadata": m.lora_tensor_metadata(),
                "config": {"lora": {"r": 4, "alpha": 8}}}, os.path.join(out_dir, rank_file_name(rank, ps.tp_rank, 0)))
    torch.distributed.barrier()
    if rank == 0:
        export_peft_adapter(out_dir, os.path.join(out_dir, "peft"))
    torch.distributed.barrier()
    pstate.destroy()


@pytest.mark.parametrize("tp", [2, 4])
def test_qwen35_tp_matches_tp1(tmp_path, tp):
    """TP = 2 splits every head kind; TP = 4 exceeds the 2 key/value heads, so
    pairs of ranks hold copies of one head and sum their B gradients."""
    from graspo_b200.models.lora_io import load_peft_adapter
    from graspo_b200.models.qwen35 import HybridRolloutEngine
    from graspo_b200.parallel import state as pstate
    from graspo_b200.parallel.state import ParallelState
    from graspo_b200.utils.synth import QWEN35_TINY, write_qwen35_checkpoint

    os.environ.setdefault("GLOO_SOCKET_IFNAME", "lo")
    dims = dict(QWEN35_TINY, linear_num_key_heads=4, linear_num_value_heads=4)   # DeltaNet heads divide by 4
    path = write_qwen35_checkpoint(tmp_path / "q35", dims, seed=1, std=0.05, with_tokenizer=False)
    m = _model(path, ParallelState())
    assert m.nkv < 4
    ids, mask = _batch()
    lp = _grads(m, ids, mask)
    grads = {mod.module_name: {"a": _to_full(mod, "a", mod.a_grad), "b": _to_full(mod, "b", mod.b_grad)}
             for mod in m.lora.modules}
    kw = dict(group_size=2, max_new_tokens=6, temperature=1.0, top_p=1.0, eos_id=508, pad_id=508,
              ignore_eos=True, seed=5)
    tokens = HybridRolloutEngine(m).generate([[5, 6, 7], list(range(20, 45))], **kw).tokens
    ref_file = tmp_path / "ref.pt"
    torch.save({"lp": lp, "grads": grads, "tokens": tokens}, ref_file)
    pstate.destroy()
    ckpt = tmp_path / "ckpt"
    ckpt.mkdir()
    run_world(tp, _worker, path, ref_file, str(ckpt), timeout=600)
    # the TP = 2 shards exported as one PEFT adapter give back the TP = 1 LoRA state
    fresh = _model(path, ParallelState())
    with torch.no_grad():
        fresh.lora.params.zero_()
    load_peft_adapter(fresh, ckpt / "peft")
    for name, t in m.lora_state_dict().items():
        assert torch.allclose(fresh.lora_state_dict()[name], t, atol=1e-6), name


def test_qwen35_tp2_grpo_run_and_export(tmp_path):
    """`graspo launch` of a Qwen3.5 run at TP = 2 (CPU ranks): one GRPO step,
    a final checkpoint, and its PEFT export with the combined in_proj_qkv pairs."""
    import json
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
    cfg["training"].update(output_dir=str(tmp_path / "run"), max_steps=1, max_new_tokens=16, rollout_group_size=2,
                           learning_rate=1e-3)
    cfg["graspoflow"]["pg_timeout_sec"] = 60.0
    cfg["launch"]["master_port"] = 29000 + os.getpid() % 2000
    path = tmp_path / "q35_tp2.yaml"
    path.write_text(yaml.safe_dump(cfg))
    env = {k: v for k, v in os.environ.items() if not k.startswith("GRASPO_FAULT")}
    env.update(PYTHONPATH=str(root), CUDA_VISIBLE_DEVICES="")
    proc = subprocess.run([sys.executable, "-m", "graspo_b200", "launch", "--config", str(path)], env=env,
                          capture_output=True, text=True, timeout=600, cwd=root)
    assert proc.returncode == 0, proc.stdout[-3000:] + proc.stderr[-3000:]
    final = tmp_path / "run" / "final"
    assert (final / "manifest.json").exists()
    from graspo_b200.models.lora_io import export_from_checkpoint

    export_from_checkpoint(final, tmp_path / "peft", export_format="peft-adapter")
    export_from_checkpoint(final, tmp_path / "merged", export_format="merged-hf", base_model_path=model)
    meta = json.loads((tmp_path / "peft" / "graspo_adapter_metadata.json").read_text())
    qkv = [m for m in meta["modules"] if m.endswith("linear_attn.in_proj_qkv")]
    assert qkv and all(len(meta["modules"][m]) == 3 for m in qkv)
