"""Qwen3.5 hybrid decoder (CPU): the chunked gated delta rule equals the
token-by-token recurrence, cached decoding equals whole-sequence forward, and
LoRA gradients flow through both layer kinds."""

import torch

from graspo_b200.models.qwen35 import chunk_gated_delta, l2norm, recurrent_gated_delta


def test_chunked_delta_rule_matches_recurrence():
    g = torch.Generator().manual_seed(0)
    B, S, h, dk, dv = 2, 150, 3, 16, 24
    q = l2norm(torch.randn(B, S, h, dk, generator=g)) / dk ** 0.5
    k = l2norm(torch.randn(B, S, h, dk, generator=g))
    v = torch.randn(B, S, h, dv, generator=g)
    gl = -torch.rand(B, S, h, generator=g) * 0.5
    beta = torch.rand(B, S, h, generator=g)
    s0 = torch.randn(B, h, dk, dv, generator=g) * 0.1
    o, fin = chunk_gated_delta(q, k, v, gl, beta, s0.clone())
    state = s0.clone()
    ref = torch.stack([recurrent_gated_delta(q[:, t], k[:, t], v[:, t], gl[:, t], beta[:, t], state)
                       for t in range(S)], 1)
    assert (o - ref).abs().max().item() < 1e-4
    assert (fin - state).abs().max().item() < 1e-4


def _model(tmp_path):
    from graspo_b200.models.config import load_decoder_config
    from graspo_b200.models.loader import SafetensorIndex
    from graspo_b200.models.qwen35 import Qwen35Model
    from graspo_b200.parallel.state import ParallelState
    from graspo_b200.utils.synth import QWEN35_TINY, write_qwen35_checkpoint

    path = write_qwen35_checkpoint(tmp_path / "q35", QWEN35_TINY, seed=1, std=0.05, with_tokenizer=False)
    targets = {"language.full_attn.q_proj", "language.full_attn.o_proj", "language.linear_attn.q_proj",
               "language.linear_attn.v_proj", "language.linear_attn.in_proj_z", "language.linear_attn.out_proj",
               "language.mlp.down_proj"}
    m = Qwen35Model(load_decoder_config(path), SafetensorIndex(path), ps=ParallelState(), lora_targets=targets,
                    lora_r=4, lora_alpha=8, dtype=torch.float32, seed=2)
    with torch.no_grad():
        m.lora.params.copy_(torch.randn(m.lora.params.shape, generator=torch.Generator().manual_seed(3)) * 0.05)
    return m


def test_hybrid_cached_decoding_matches_full_forward(tmp_path):
    m = _model(tmp_path)
    g = torch.Generator().manual_seed(4)
    ids = torch.randint(0, 500, (2, 21), generator=g)
    mask = torch.ones(2, 21, dtype=torch.bool)
    mask[1, :6] = False
    full = m.forward(ids, mask)
    caches = [dict() for _ in m.layers]
    out = [m.forward(ids[:, :15], mask[:, :15], caches=caches)]
    pos = mask[:, :15].long().sum(-1) - 1
    for t in range(15, 21):
        pos = pos + 1
        out.append(m.forward(ids[:, t : t + 1], mask[:, t : t + 1], caches=caches, pos=pos[:, None],
                             key_mask=mask[:, : t + 1]))
    inc = torch.cat(out, 1)
    valid = mask
    assert (inc - full).abs()[valid].max().item() < 1e-3


def test_hybrid_lora_gradients_flow(tmp_path):
    from graspo_b200.models.qwen3 import EagerLoRA

    m = _model(tmp_path)
    ids = torch.randint(0, 500, (2, 70), generator=torch.Generator().manual_seed(5))
    mask = torch.ones(2, 70, dtype=torch.bool)
    lora = EagerLoRA(m.lora, requires_grad=True)
    lp = m.sequence_logprobs(ids, mask, lora=lora, training=True)
    lp.sum().backward()
    lora.accumulate_grads()
    for mod in m.lora.modules:
        assert mod.b_grad.abs().sum() > 0 and mod.a_grad.abs().sum() > 0, mod.module_name


def test_hybrid_adapter_grpo_round_trip(tmp_path):
    """Default adapter string + a qwen3_5 checkpoint -> hybrid adapter: rollout,
    old log-probs and one GRPO optimizer step through the public runtime API."""
    from graspo_b200.core.buffer import Experience
    from graspo_b200.core.data import sample_from_record
    from graspo_b200.core.schema import GraspoConfig
    from graspo_b200.engine.adapter import Qwen35Adapter
    from graspo_b200.engine.runtime import GraspoFlowRuntime
    from graspo_b200.utils.synth import QWEN35_TINY, synthetic_json_records, write_qwen35_checkpoint

    path = write_qwen35_checkpoint(tmp_path / "q35", QWEN35_TINY, seed=1, std=0.05)
    cfg = GraspoConfig.from_dict({
        "train_method": "graspo",
        "model": {"model_path": str(path), "torch_dtype": "float32"},
        "data": {"train_path": "", "max_prompt_length": 64},
        "lora": {"r": 4, "alpha": 8, "dropout": 0.0, "target_modules": [
            "language.full_attn.q_proj", "language.linear_attn.q_proj", "language.linear_attn.out_proj",
            "language.mlp.down_proj"]},
        "training": {"output_dir": str(tmp_path / "run"), "run_name": "t", "rollout_group_size": 2,
                     "optimize_prompt_batch_size": 2, "learning_rate": 1e-3, "max_new_tokens": 6},
        "graspoflow": {"tp_size": 1, "pp_size": 1, "raw_log_enabled": False, "readable_log_enabled": False},
    })
    (tmp_path / "run" / "logs").mkdir(parents=True)
    api = GraspoFlowRuntime.from_config(cfg)
    api.setup()
    assert isinstance(api.adapter, Qwen35Adapter)
    samples = [sample_from_record(r) for r in synthetic_json_records(2, seed=3)]
    gens = api.generate_sample_groups(samples=samples, rollout_group_size=2, max_new_tokens=6, temperature=1.0,
                                      top_p=1.0)
    assert len(gens) == 2 and gens[0].sequences.shape[0] == 2
    exps = []
    for gen in gens:
        old = api.sequence_log_probs(gen.sequences, gen.attention_mask)
        adv = torch.tensor([1.0, -1.0])[:, None].expand_as(old).contiguous()
        for i in range(2):
            exps.append(Experience(sequences=gen.sequences[i], old_log_probs=old[i].cpu(), advantages=adv[i].cpu(),
                                   attention_mask=gen.attention_mask[i], action_mask=gen.action_mask[i],
                                   rewards=torch.zeros(()), metadata={}))
    before = api.adapter.model.lora.params.clone()
    metrics = api.train_batch(exps, policy_ratio_clip_eps=0.2, optimize_iterations_per_step=1, max_grad_norm=1.0)
    assert metrics["optimizer_steps"] == 2 and metrics["loss_mean"] is not None
    for key in ("micro_batch_forward_sec", "backward_sec", "optimizer_step_sec"):
        assert metrics[key] > 0, key
    assert len(metrics["optimize_round_sec"]) == 1
    assert not torch.equal(before, api.adapter.model.lora.params)


def test_chunked_delta_rule_gradients_match_recurrence():
    """Gradients of the chunked form (the training path) equal those of a
    functional token-by-token recurrence, initial state included."""
    g = torch.Generator().manual_seed(1)
    B, S, h, dk, dv = 1, 140, 2, 8, 12
    qi = torch.randn(B, S, h, dk, generator=g)
    ki = torch.randn(B, S, h, dk, generator=g)
    v = torch.randn(B, S, h, dv, generator=g)
    gl = -torch.rand(B, S, h, generator=g) * 0.5
    beta = torch.rand(B, S, h, generator=g)
    s0 = torch.randn(B, h, dk, dv, generator=g) * 0.1
    wo = torch.randn(B, S, h, dv, generator=g)
    wf = torch.randn(B, h, dk, dv, generator=g)
    leaves = [t.clone().requires_grad_(True) for t in (qi, ki, v, gl, beta, s0)]

    def loss_chunked(qi, ki, v, gl, beta, s0):
        o, fin = chunk_gated_delta(l2norm(qi) / dk ** 0.5, l2norm(ki), v, gl, beta, s0)
        return (o * wo).sum() + (fin * wf).sum()

    def loss_recurrent(qi, ki, v, gl, beta, s0):
        q, k = l2norm(qi) / dk ** 0.5, l2norm(ki)
        st, outs = s0, []
        for t in range(S):
            st = st * gl[:, t].exp()[..., None, None]
            mem = (st * k[:, t, :, :, None]).sum(-2)
            delta = (v[:, t] - mem) * beta[:, t, :, None]
            st = st + k[:, t, :, :, None] * delta[:, :, None, :]
            outs.append((st * q[:, t, :, :, None]).sum(-2))
        return (torch.stack(outs, 1) * wo).sum() + (st * wf).sum()

    ga = torch.autograd.grad(loss_chunked(*leaves), leaves)
    gb = torch.autograd.grad(loss_recurrent(*leaves), leaves)
    for name, a, b in zip(("q", "k", "v", "g", "beta", "state"), ga, gb):
        assert (a - b).abs().max().item() <= 1e-4 * (1 + b.abs().max().item()), name


def test_full_attention_span_rotation_matches_masked(tmp_path):
    """Rows whose valid tokens form one span (left and right padding) take the
    rotated causal-attention path; their valid positions equal the explicitly
    masked attention's, in values and LoRA gradients."""
    from graspo_b200.models import qwen35 as q35
    from graspo_b200.models.qwen3 import EagerLoRA

    m = _model(tmp_path)
    g = torch.Generator().manual_seed(5)
    ids = torch.randint(0, 500, (3, 30), generator=g)
    mask = torch.ones(3, 30, dtype=torch.bool)
    mask[0, :6] = False
    mask[1, -5:] = False
    mask[2, :3] = False
    mask[2, -4:] = False
    assert q35._valid_span_start(mask).tolist() == [6, 0, 3]
    w = torch.randn(3, 29, generator=g)
    valid = mask[:, :-1] & mask[:, 1:]

    def run():
        m.lora.grads.zero_()
        lora = EagerLoRA(m.lora, requires_grad=True)
        lp = m.sequence_logprobs(ids, mask, lora=lora, training=True)
        (lp * w * valid).sum().backward()
        lora.accumulate_grads()
        return lp.detach(), m.lora.grads.clone()

    lp_rot, g_rot = run()
    orig = q35._valid_span_start
    q35._valid_span_start = lambda mask: None        # force the masked form
    try:
        lp_mask, g_mask = run()
    finally:
        q35._valid_span_start = orig
    assert (lp_rot - lp_mask).abs()[valid].max().item() < 1e-4
    assert (g_rot - g_mask).abs().max().item() <= 1e-4 * (1 + g_mask.abs().max().item())
    holes = mask.clone()
    holes[1, 10] = False
    assert q35._valid_span_start(holes) is None
