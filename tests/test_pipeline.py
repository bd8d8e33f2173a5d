"""Pipeline parallelism on CPU (gloo, 2 stages, emulated kernels): log-probs,
1F1B training gradients and pipelined decoding match the single-stage model."""

import os
import zlib

import torch

from tests.dist_util import run_world

SMALL = dict(vocab_size=512, hidden_size=128, intermediate_size=256, num_hidden_layers=4,
             num_attention_heads=4, num_key_value_heads=2, head_dim=128)
TARGETS = {"language.self_attn.q_proj", "language.self_attn.k_proj", "language.self_attn.v_proj",
           "language.self_attn.o_proj", "language.mlp.gate_proj", "language.mlp.up_proj", "language.mlp.down_proj"}


def _model(path, ps, layers, embed, head):
    from graspo_b200.models.config import load_decoder_config
    from graspo_b200.models.loader import SafetensorIndex
    from graspo_b200.models.qwen3 import Qwen3Model

    m = Qwen3Model(load_decoder_config(path), SafetensorIndex(path), ps=ps, local_layers=layers,
                   include_embed=embed, include_head=head, lora_targets=TARGETS, lora_r=8, lora_alpha=16,
                   lora_dropout=0.0, dtype=torch.float32, device=torch.device("cpu"), seed=3)
    with torch.no_grad():
        for mod in m.lora.modules:
            g = torch.Generator().manual_seed(zlib.crc32(mod.module_name.encode()))
            mod.b.copy_(torch.randn(mod.b.shape, generator=g) * 0.05)
    m.lora.invalidate()
    return m


def _batch():
    g = torch.Generator().manual_seed(0)
    seq = torch.randint(0, 500, (3, 40), generator=g)
    mask = torch.ones(3, 40, dtype=torch.bool)
    mask[1, :9] = False
    mask[2, -7:] = False
    w = torch.randn(3, 39, generator=g) * (mask[:, :-1] & mask[:, 1:])
    return seq, mask, w


def _worker(rank, world, path):
    from graspo_b200.engine.pipeline import pp_logprobs, pp_train
    from graspo_b200.engine.rollout import FusedRolloutEngine
    from graspo_b200.models.fused import AttnMeta, FusedQwen3
    from graspo_b200.ops.emulate import use_emulation
    from graspo_b200.parallel import state as pstate
    from graspo_b200.parallel.p2p import StageComm
    from graspo_b200.parallel.state import ParallelState

    ps = pstate.initialize(1, 2, 0, timeout_sec=60, device="cpu")
    comm = StageComm(ps)
    seq, mask, w = _batch()
    with use_emulation():
        stage = _model(path, ps, [0, 1] if rank == 0 else [2, 3], rank == 0, rank == 1)
        ref = _model(path, ParallelState(), [0, 1, 2, 3], True, True)
        fs, fr = FusedQwen3(stage), FusedQwen3(ref)
        # ---- forward log-probs
        lp = pp_logprobs(fs, comm, seq, mask, seq[:, 1:], chunk_rows=1)
        meta = AttnMeta.from_mask(mask)
        x, inputs = fr.stage_forward(fr.embed(seq), meta, train=True, keep_inputs=True)
        hn, rstd = fr.final_norm(x)
        tgt = torch.zeros_like(seq)
        tgt[:, :-1] = seq[:, 1:]
        lp_ref, lse = fr.token_logprobs(hn, tgt.reshape(-1))
        lp_ref = lp_ref.view(seq.shape)[:, :-1]
        valid = mask[:, :-1] & mask[:, 1:]
        err = (lp - lp_ref).abs()[valid].max().item()
        assert err < 1e-4, (err, lp[:, :5], lp_ref[:, :5])
        # ---- 1F1B training: loss = sum(w * logp), chunks of one row
        def loss_fn(lp_c, sl):
            return (lp_c * w[sl]).sum().reshape(1), w[sl].clone()

        stage.lora.grads.zero_()
        loss = pp_train(fs, comm, seq, mask, seq[:, 1:], loss_fn, seed=0, chunk_rows=1, schedule="one_f_one_b")
        assert abs(loss.item() - (lp_ref * w).sum().item()) < 1e-3
        ref.lora.grads.zero_()
        g = torch.zeros(seq.shape)
        g[:, :-1] = w
        dhn = fr.token_logprobs_backward(hn, tgt.reshape(-1), lse, g.view(-1))
        from graspo_b200.ops._ext import ext

        dx = torch.empty_like(x)
        ext().rmsnorm_bwd(dhn, x, ref.norm, rstd, None, dx, ref.cfg.rms_norm_eps)
        fr.stage_backward(inputs, dx, meta, train=True)
        for mod in stage.lora.modules:
            rm = ref.lora.by_name[mod.module_name]
            for a, b in ((mod.a_grad, rm.a_grad), (mod.b_grad, rm.b_grad)):
                err = (a - b).abs().max().item()
                assert err <= 1e-4 * (b.abs().max().item() + 1e-3), (mod.module_name, err)
        # ---- pipelined decoding reproduces the single-stage engine
        kw = dict(group_size=2, max_new_tokens=6, temperature=1.0, top_p=1.0, eos_id=511, pad_id=511,
                  ignore_eos=True, seed=5)
        prompts = [[5, 6, 7], list(range(20, 45))]
        got = FusedRolloutEngine(stage, fs, page_size=16, use_graph=False, comm=comm).generate(prompts, **kw)
        want = FusedRolloutEngine(ref, fr, page_size=16, use_graph=False).generate(prompts, **kw)
        assert torch.equal(got.tokens, want.tokens), (got.tokens, want.tokens)
    pstate.destroy()


def test_pipeline_two_stages_match_single_stage(tmp_path):
    from graspo_b200.utils.synth import write_qwen3_checkpoint

    os.environ.setdefault("GLOO_SOCKET_IFNAME", "lo")
    path = write_qwen3_checkpoint(tmp_path / "pp", SMALL, seed=2, std=0.05, with_tokenizer=False)
    run_world(2, _worker, path, timeout=600)
