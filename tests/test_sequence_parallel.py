"""Sequence parallelism on CPU (gloo, TP=2, emulated kernels): log-probs and
LoRA gradients of the SP path equal those of the unsharded model."""

import zlib

import torch
import torch.distributed as dist

from tests.dist_util import run_world

SMALL = dict(vocab_size=512, hidden_size=128, intermediate_size=256, num_hidden_layers=2,
             num_attention_heads=4, num_key_value_heads=2, head_dim=128)
TARGETS = {"language.self_attn.q_proj", "language.self_attn.k_proj", "language.self_attn.v_proj",
           "language.self_attn.o_proj", "language.mlp.gate_proj", "language.mlp.up_proj", "language.mlp.down_proj"}


def _model(path, ps, **stage):
    from graspo_b200.models.config import load_decoder_config
    from graspo_b200.models.loader import SafetensorIndex
    from graspo_b200.models.qwen3 import Qwen3Model

    m = Qwen3Model(load_decoder_config(path), SafetensorIndex(path), ps=ps, lora_targets=TARGETS, lora_r=8,
                   lora_alpha=16, lora_dropout=0.0, dtype=torch.float32, device=torch.device("cpu"), seed=3,
                   **stage)
    with torch.no_grad():
        for mod in m.lora.modules:
            g = torch.Generator().manual_seed(zlib.crc32(mod.module_name.encode()))
            full = torch.randn(mod.out_full, m.lora.r, generator=g) * 0.05
            mod.b.copy_(full[mod.row_start : mod.row_stop] if mod.shard_kind == "out" else full)
    m.lora.invalidate()
    return m


def _run(f, seq, mask, w):
    """log-probs and LoRA grads of sum(w * logp) through FusedQwen3 ``f`` (SP-aware)."""
    from graspo_b200.models.fused import AttnMeta
    from graspo_b200.ops._ext import ext

    m = f.m
    m.lora.grads.zero_()
    meta = AttnMeta.from_mask(mask)
    xL, inputs = f.stage_forward(f.sp_shard(f.embed(seq)), meta, train=True, keep_inputs=True)
    hn, rstd = f.final_norm(xL)
    hn_all = f.sp_gather(hn)
    tgt = torch.zeros_like(seq)
    tgt[:, :-1] = seq[:, 1:]
    lp, lse = f.token_logprobs(hn_all, tgt.reshape(-1))
    g = torch.zeros(seq.shape)
    g[:, :-1] = w
    dhn = f.token_logprobs_backward(hn_all, tgt.reshape(-1), lse, g.view(-1))
    dx = torch.empty_like(xL)
    ext().rmsnorm_bwd(dhn, xL, m.norm, rstd, None, dx, m.cfg.rms_norm_eps)
    f.stage_backward(inputs, dx, meta, train=True)
    return lp.view(seq.shape)[:, :-1]


def _worker(rank, world, path):
    from graspo_b200.models.fused import FusedQwen3
    from graspo_b200.ops.emulate import use_emulation
    from graspo_b200.parallel import state as pstate
    from graspo_b200.parallel.state import ParallelState

    ps = pstate.initialize(2, 1, 0, timeout_sec=60, device="cpu")
    g = torch.Generator().manual_seed(0)
    seq = torch.randint(0, 500, (3, 22), generator=g)   # 66 tokens: 33 per rank
    mask = torch.ones(3, 22, dtype=torch.bool)
    mask[1, :5] = False
    mask[2, -4:] = False
    w = torch.randn(3, 21, generator=g) * (mask[:, :-1] & mask[:, 1:])
    with use_emulation():
        m2 = _model(path, ps)
        lp_tp = _run(FusedQwen3(m2, sequence_parallel=False), seq, mask, w)
        dist.all_reduce(m2.lora.grads[: m2.lora.replicated_numel], group=ps.tp_group)
        g_tp = m2.lora.grads.clone()
        lp_sp = _run(FusedQwen3(m2, sequence_parallel=True), seq, mask, w)
        dist.all_reduce(m2.lora.grads[: m2.lora.replicated_numel], group=ps.tp_group)
        g_sp = m2.lora.grads.clone()
        m1 = _model(path, ParallelState())
        lp1 = _run(FusedQwen3(m1), seq, mask, w)
    valid = mask[:, :-1] & mask[:, 1:]
    # SP only moves where the sums happen: same values as the all-reduce TP path
    assert (lp_sp - lp_tp).abs()[valid].max().item() < 1e-5
    assert (g_sp - g_tp).abs().max().item() <= 1e-3 * g_tp.abs().max().item()
    # and both agree with the unsharded model up to bf16 rounding of partial sums
    assert (lp1 - lp_sp).abs()[valid].max().item() < 3e-2
    for mod2 in m2.lora.modules:
        mod1 = m1.lora.by_name[mod2.module_name]
        if mod2.shard_kind == "out":
            a1, b1 = mod1.a_grad, mod1.b_grad[mod2.row_start : mod2.row_stop]
        else:
            a1, b1 = mod1.a_grad[:, mod2.col_start : mod2.col_stop], mod1.b_grad
        for x1, x2 in ((a1, mod2.a_grad), (b1, mod2.b_grad)):
            cos = torch.nn.functional.cosine_similarity(x1.flatten(), x2.flatten(), dim=0).item()
            assert cos > 0.99, (mod2.module_name, cos)
    pstate.destroy()


def test_sequence_parallel_tp2_matches_tp1(tmp_path):
    from graspo_b200.utils.synth import write_qwen3_checkpoint

    path = write_qwen3_checkpoint(tmp_path / "sp", SMALL, seed=2, std=0.05, with_tokenizer=False)
    run_world(2, _worker, path, timeout=600)


def _pp_worker(rank, world, path):
    """TP=2 with SP x PP=2: pipelined log-probs and 1F1B gradients equal the
    unsharded model's; each stage sends its TP rank's token shard."""
    from graspo_b200.engine.pipeline import pp_logprobs, pp_train
    from graspo_b200.models.fused import FusedQwen3
    from graspo_b200.ops.emulate import use_emulation
    from graspo_b200.parallel import state as pstate
    from graspo_b200.parallel.p2p import StageComm
    from graspo_b200.parallel.state import ParallelState

    ps = pstate.initialize(2, 2, 0, timeout_sec=60, device="cpu")
    comm = StageComm(ps)
    g = torch.Generator().manual_seed(1)
    seq = torch.randint(0, 500, (3, 23), generator=g)   # odd length: padded to 24 under SP
    mask = torch.ones(3, 23, dtype=torch.bool)
    mask[0, :4] = False
    mask[2, -3:] = False
    w = torch.randn(3, 22, generator=g) * (mask[:, :-1] & mask[:, 1:])
    first, last = ps.pp_rank == 0, ps.pp_rank == 1
    with use_emulation():
        stage = _model(path, ps, local_layers=[0] if first else [1], include_embed=first, include_head=last)
        f = FusedQwen3(stage, sequence_parallel=True)
        lp = pp_logprobs(f, comm, seq, mask, seq[:, 1:], chunk_rows=1)
        stage.lora.grads.zero_()

        def loss_fn(lp_c, sl):
            return (lp_c * w[sl]).sum().reshape(1), w[sl].clone()

        loss = pp_train(f, comm, seq, mask, seq[:, 1:], loss_fn, seed=0, chunk_rows=1, schedule="one_f_one_b")
        dist.all_reduce(stage.lora.grads[: stage.lora.replicated_numel], group=ps.tp_group)
        m1 = _model(path, ParallelState())
        lp1 = _run(FusedQwen3(m1), seq, mask, w)
    valid = mask[:, :-1] & mask[:, 1:]
    assert lp.shape == lp1.shape
    assert (lp - lp1).abs()[valid].max().item() < 3e-2
    assert abs(loss.item() - (lp1 * w).sum().item()) < 5e-2 * (1 + abs(loss.item()))
    for mod2 in stage.lora.modules:
        mod1 = m1.lora.by_name[mod2.module_name]
        if mod2.shard_kind == "out":
            a1, b1 = mod1.a_grad, mod1.b_grad[mod2.row_start : mod2.row_stop]
        else:
            a1, b1 = mod1.a_grad[:, mod2.col_start : mod2.col_stop], mod1.b_grad
        for x1, x2 in ((a1, mod2.a_grad), (b1, mod2.b_grad)):
            cos = torch.nn.functional.cosine_similarity(x1.flatten(), x2.flatten(), dim=0).item()
            assert cos > 0.99, (mod2.module_name, cos)
    pstate.destroy()


def test_sequence_parallel_with_pipeline_stages(tmp_path):
    from graspo_b200.utils.synth import write_qwen3_checkpoint

    path = write_qwen3_checkpoint(tmp_path / "sp_pp", SMALL, seed=2, std=0.05, with_tokenizer=False)
    run_world(4, _pp_worker, path, timeout=600)
