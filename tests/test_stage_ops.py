"""Stage operators chained in a ``PipelineGraph`` (CPU, one process).

Embedding -> decoder layers -> head operators run a 1F1B plan over three
micro-batches of one row; the log-probs and the LoRA gradients of the loss
sum(w * logp) equal one autograd pass over the whole batch, on both model
families.  Reference behaviour: models/qwen3/ops.py:12-256,
models/qwen35_36/ops.py:12-281, graph.py:29-168.
"""

import zlib

import pytest
import torch


def _model(tmp_path, family):
    from graspo_b200.models.config import load_decoder_config
    from graspo_b200.models.loader import SafetensorIndex
    from graspo_b200.parallel.state import ParallelState
    from graspo_b200.utils.synth import QWEN35_TINY, TINY, write_qwen3_checkpoint, write_qwen35_checkpoint

    if family == "qwen3":
        from graspo_b200.models.qwen3 import Qwen3Model as cls

        path = write_qwen3_checkpoint(tmp_path / "m", TINY, seed=1, device="cpu", dtype=torch.float32,
                                      with_tokenizer=False)
        targets = {"language.self_attn.q_proj", "language.self_attn.o_proj", "language.mlp.up_proj"}
    else:
        from graspo_b200.models.qwen35 import Qwen35Model as cls

        path = write_qwen35_checkpoint(tmp_path / "m", QWEN35_TINY, seed=1, std=0.05, dtype=torch.float32,
                                       with_tokenizer=False)
        targets = {"language.full_attn.q_proj", "language.linear_attn.v_proj", "language.mlp.up_proj"}
    m = cls(load_decoder_config(path), SafetensorIndex(path), ps=ParallelState(), lora_targets=targets, lora_r=4,
            lora_alpha=8, dtype=torch.float32, device=torch.device("cpu"), seed=2)
    with torch.no_grad():
        for mod in m.lora.modules:
            g = torch.Generator().manual_seed(zlib.crc32(mod.module_name.encode()))
            mod.b.copy_(torch.randn(mod.b.shape, generator=g) * 0.1)
    m.lora.invalidate()
    return m


@pytest.mark.parametrize("family", ["qwen3", "qwen3_5"])
def test_stage_ops_graph_matches_autograd(tmp_path, family):
    from graspo_b200.models.qwen3 import EagerLoRA, eager_sequence_logprobs
    from graspo_b200.parallel.operator import Microbatch, PipelineGraph
    from graspo_b200.parallel.schedule import get_scheduler
    from graspo_b200.parallel.stage_ops import build_stage_ops

    m = _model(tmp_path, family)
    g = torch.Generator().manual_seed(0)
    ids = torch.randint(0, 500, (3, 30), generator=g)
    mask = torch.ones(3, 30, dtype=torch.bool)
    mask[1, :6] = False
    w = torch.randn(3, 29, generator=g) * (mask[:, :-1] & mask[:, 1:])
    # reference: one autograd pass
    m.lora.grads.zero_()
    lora = EagerLoRA(m.lora, requires_grad=True)
    if family == "qwen3":
        lp_ref = eager_sequence_logprobs(m, ids, mask, lora=lora, training=True)
    else:
        lp_ref = m.sequence_logprobs(ids, mask, lora=lora, training=True)
    (lp_ref * w).sum().backward()
    lora.accumulate_grads()
    ref = m.lora.grads.clone()
    m.lora.grads.zero_()
    # graph of operators, one row per micro-batch
    ops = build_stage_ops(m)
    assert [type(op).__name__ for op in ops] == ["EmbedStageOp", "DecoderStageOp", "HeadStageOp"]
    graph = PipelineGraph(ops)
    inputs = {i: Microbatch(i, tensors={"input_ids": ids[i : i + 1], "attention_mask": mask[i : i + 1],
                                        "targets": ids[i : i + 1, 1:], "grad_logprobs": w[i : i + 1]})
              for i in range(3)}
    out = graph.execute_plan(get_scheduler("one_f_one_b", pp_size=1, pp_rank=0).plan(3), inputs)
    ops[1].finish()
    graph.shutdown()
    lp = torch.cat([out[i].tensors["logprobs"] for i in range(3)])
    valid = mask[:, :-1] & mask[:, 1:]
    assert (lp - lp_ref.detach()).abs()[valid].max().item() < 1e-4
    assert torch.allclose(m.lora.grads, ref, atol=1e-5, rtol=1e-4), (m.lora.grads - ref).abs().max()
    assert all(op.forward_count == 3 and op.backward_count == 3 for op in ops)
