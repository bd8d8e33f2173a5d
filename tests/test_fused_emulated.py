"""Fused execution path on CPU, with every kernel replaced by its PyTorch
emulation: checks the orchestration (LoRA layouts and K-extension, split-K
workspaces, recompute backward, paged KV bookkeeping) against the eager oracle."""

import pytest
import torch

from graspo_b200.ops.emulate import use_emulation

SMALL = dict(vocab_size=4096, hidden_size=512, intermediate_size=1024, num_hidden_layers=2,
             num_attention_heads=4, num_key_value_heads=2, head_dim=128)
TARGETS = {"language.self_attn.q_proj", "language.self_attn.k_proj", "language.self_attn.v_proj",
           "language.self_attn.o_proj", "language.mlp.gate_proj", "language.mlp.up_proj", "language.mlp.down_proj"}


@pytest.fixture(scope="module")
def model(tmp_path_factory):
    from graspo_b200.models.config import load_decoder_config
    from graspo_b200.models.loader import SafetensorIndex
    from graspo_b200.models.qwen3 import Qwen3Model
    from graspo_b200.parallel.state import ParallelState
    from graspo_b200.utils.synth import write_qwen3_checkpoint

    path = write_qwen3_checkpoint(tmp_path_factory.mktemp("small"), SMALL, seed=3, std=0.05, device="cpu")
    ps = ParallelState(device=torch.device("cpu"))
    m = Qwen3Model(load_decoder_config(path), SafetensorIndex(path), ps=ps, lora_targets=TARGETS, lora_r=8,
                   lora_alpha=16, lora_dropout=0.0, dtype=torch.float32, device=ps.device, seed=1)
    g = torch.Generator().manual_seed(5)
    with torch.no_grad():
        m.lora.params.copy_(torch.randn(m.lora.params.shape, generator=g) * 0.02)
    m.lora.invalidate()
    m.ensure_transposed()
    return m


def _batch():
    g = torch.Generator().manual_seed(0)
    seq = torch.randint(0, 4088, (3, 64), generator=g)
    mask = torch.ones(3, 64, dtype=torch.bool)
    mask[1, :11] = False
    mask[2, -7:] = False
    return seq, mask


def _fused_logprobs(m, seq, mask, train=False):
    from graspo_b200.models.fused import AttnMeta, FusedQwen3

    f = FusedQwen3(m)
    meta = AttnMeta.from_mask(mask)
    x, inputs = f.stage_forward(f.embed(seq), meta, train=train, keep_inputs=train)
    hn, rstd = f.final_norm(x)
    tgt = torch.zeros_like(seq)
    tgt[:, :-1] = seq[:, 1:]
    lp, lse = f.token_logprobs(hn, tgt.reshape(-1))
    return lp.view(seq.shape)[:, :-1], (f, meta, inputs, x, hn, rstd, tgt, lse)


def test_emulated_fused_logprobs_match_eager(model):
    from graspo_b200.models.qwen3 import eager_sequence_logprobs

    seq, mask = _batch()
    ref = eager_sequence_logprobs(model, seq, mask)
    with use_emulation():
        lp, _ = _fused_logprobs(model, seq, mask)
    valid = mask[:, :-1] & mask[:, 1:]
    assert (lp - ref).abs()[valid].max().item() < 0.05


def test_emulated_fused_lora_grads_match_eager(model):
    from graspo_b200.models.qwen3 import EagerLoRA, eager_stage_forward, eager_token_logprobs
    from graspo_b200.ops._ext import ext

    seq, mask = _batch()
    B, S = seq.shape
    w = torch.randn(B, S - 1, generator=torch.Generator().manual_seed(1)) * (mask[:, :-1] & mask[:, 1:])
    model.lora.grads.zero_()
    lora = EagerLoRA(model.lora, requires_grad=True)
    hidden = eager_stage_forward(model, seq, mask, lora=lora, training=True)
    (eager_token_logprobs(model, hidden[:, :-1], seq[:, 1:]) * w).sum().backward()
    lora.accumulate_grads()
    ref = model.lora.grads.clone()
    model.lora.grads.zero_()
    with use_emulation():
        _, (f, meta, inputs, x, hn, rstd, tgt, lse) = _fused_logprobs(model, seq, mask, train=True)
        g = torch.zeros(B, S)
        g[:, :-1] = w
        dhn = f.token_logprobs_backward(hn, tgt.reshape(-1), lse, g.view(-1))
        dx = torch.empty_like(x)
        ext().rmsnorm_bwd(dhn, x, model.norm, rstd, None, dx, model.cfg.rms_norm_eps)
        f.stage_backward(inputs, dx, meta, train=True)
    got = model.lora.grads.clone()
    cos = torch.nn.functional.cosine_similarity(got, ref, dim=0).item()
    assert cos > 0.995, cos
    assert ((got - ref).norm() / ref.norm()).item() < 0.05


def test_emulated_paged_rollout_matches_eager(model):
    from graspo_b200.engine.rollout import EagerRolloutEngine, FusedRolloutEngine
    from graspo_b200.models.fused import FusedQwen3

    prompts = [[5, 6, 7, 8, 9], list(range(20, 50)), [300]]
    kw = dict(group_size=2, max_new_tokens=6, temperature=0.0, top_p=1.0, eos_id=4095, pad_id=4095,
              ignore_eos=True, seed=0)
    eager = EagerRolloutEngine(model).generate(prompts, **kw)
    with use_emulation():
        fused = FusedRolloutEngine(model, FusedQwen3(model), page_size=16, use_graph=False).generate(prompts, **kw)
    assert torch.equal(fused.tokens, eager.tokens)


def _fused_grads(model, monkeypatch, mode):
    from graspo_b200.ops._ext import ext

    monkeypatch.setenv("GRASPO_CACHE_ATTN", mode)
    seq, mask = _batch()
    B, S = seq.shape
    w = torch.randn(B, S - 1, generator=torch.Generator().manual_seed(1)) * (mask[:, :-1] & mask[:, 1:])
    model.lora.grads.zero_()
    with use_emulation():
        _, (f, meta, inputs, x, hn, rstd, tgt, lse) = _fused_logprobs(model, seq, mask, train=True)
        cached = [c is not None for _, c in inputs]
        g = torch.zeros(B, S)
        g[:, :-1] = w
        dhn = f.token_logprobs_backward(hn, tgt.reshape(-1), lse, g.view(-1))
        dx = torch.empty_like(x)
        ext().rmsnorm_bwd(dhn, x, model.norm, rstd, None, dx, model.cfg.rms_norm_eps)
        dx0 = f.stage_backward(inputs, dx, meta, train=True)
    assert inputs == []  # consumed layer by layer
    return model.lora.grads.clone(), dx0, cached


def test_attention_cache_gives_the_recompute_values(model, monkeypatch):
    """Keeping q/k/v, attention output and LSE from the forward (instead of
    recomputing them in the backward) changes no gradient."""
    ref, dref, cached_ref = _fused_grads(model, monkeypatch, "0")
    assert not any(cached_ref)
    for mode in ("1", "2"):   # attention values; attention and MLP values
        got, dgot, cached = _fused_grads(model, monkeypatch, mode)
        assert all(cached), mode
        assert torch.equal(got, ref) and torch.equal(dgot, dref), mode


def test_split_rollout_merges_to_the_unsplit_result(model):
    """Decoding the prompts in several engine calls (graspoflow.rollout_engine_batch)
    and merging gives the rows, prompt padding and lengths of one call (greedy)."""
    from graspo_b200.engine.rollout import EagerRolloutEngine, merge_results

    prompts = [[5, 6, 7, 8, 9], list(range(20, 50)), [300]]
    kw = dict(group_size=2, max_new_tokens=5, temperature=0.0, top_p=1.0, eos_id=4095, pad_id=4095,
              ignore_eos=True, seed=0)
    eng = EagerRolloutEngine(model)
    whole = eng.generate(prompts, **kw)
    parts = [eng.generate(prompts[:1], **kw), eng.generate(prompts[1:], **kw)]
    merged = merge_results(parts, pad_id=4095)
    assert merged.splits == 2 and merged.group_size == 2
    assert torch.equal(merged.tokens, whole.tokens)
    assert merged.prompt_lens == whole.prompt_lens and merged.gen_lens == whole.gen_lens
    assert torch.equal(merged.prompt_ids, whole.prompt_ids)
    assert merge_results(parts[:1], pad_id=4095) is parts[0]


def test_layer_gradient_ranges_cover_the_buffer_once(model):
    """The data-parallel push sends each layer's LoRA factors as merged ranges of the flat
    buffer; over all layers they cover every entry exactly once."""
    lora = model.lora
    seen = torch.zeros(lora.numel, dtype=torch.int32)
    for lw in model.layers:
        ranges = lora.layer_ranges(lw.index)
        assert ranges == sorted(ranges)
        for start, count in ranges:
            seen[start : start + count] += 1
    assert bool((seen == 1).all())


def test_stage_backward_reports_each_finished_layer(model):
    from graspo_b200.models.fused import AttnMeta, FusedQwen3

    with use_emulation():
        f = FusedQwen3(model)
        seq, mask = _batch()
        meta = AttnMeta.from_mask(mask)
        x, inputs = f.stage_forward(f.embed(seq), meta, train=True, keep_inputs=True)
        done = []
        f.stage_backward(inputs, torch.randn_like(x) * 1e-3, meta, train=True, on_layer_done=done.append)
    assert done == [lw.index for lw in reversed(model.layers)]
