"""Images with pipeline stages (CPU ranks over gloo, PP=2), Qwen3.5 hybrid with
a vision tower and LoRA on the tower, through the public runtime API.

The first stage runs the tower and places the image features; the second
stage derives the multimodal RoPE positions from the image grids alone (its
full-attention layer is the one that uses them).  The rollout, the old
log-probs and one GRPO step equal the single-stage run
(reference: backends/graspoflow/models/qwen35_36/training.py:509-565, where
every stage receives the multimodal inputs)."""

import os

import torch

from tests.dist_util import run_world

TARGETS = ["language.full_attn.q_proj", "language.linear_attn.out_proj", "language.mlp.down_proj", "vision_merger"]


def _config(path, out_dir, pp):
    from graspo_b200.core.schema import GraspoConfig

    flow = {"tp_size": 1, "pp_size": pp, "raw_log_enabled": False, "readable_log_enabled": False}
    if pp > 1:
        flow.update(pp_schedule="one_f_one_b", pp_micro_batch_size=1)
    return GraspoConfig.from_dict({
        "train_method": "graspo",
        "model": {"model_path": str(path), "torch_dtype": "float32"},
        "data": {"train_path": "", "max_prompt_length": 600},
        "lora": {"r": 4, "alpha": 8, "dropout": 0.0, "target_modules": TARGETS},
        "training": {"output_dir": str(out_dir), "run_name": "t", "rollout_group_size": 2, "seed": 11,
                     "optimize_prompt_batch_size": 2, "learning_rate": 1e-2, "max_new_tokens": 4},
        "graspoflow": flow,
    })


def _round(api, samples):
    from graspo_b200.core.buffer import Experience

    gens = api.generate_sample_groups(samples=samples, rollout_group_size=2, max_new_tokens=4, temperature=1.0,
                                      top_p=1.0)
    seqs, olds, exps = [], [], []
    for gen in gens:
        old = api.sequence_log_probs(gen.sequences, gen.attention_mask, metadata=gen.metadata)
        seqs.append(gen.sequences.clone())
        olds.append(old.detach().cpu().clone())
        for i in range(2):
            exps.append(Experience(sequences=gen.sequences[i], old_log_probs=old[i].cpu(),
                                   advantages=torch.full_like(old[i].cpu(), 1.0 - 2 * i),
                                   attention_mask=gen.attention_mask[i], action_mask=gen.action_mask[i],
                                   rewards=torch.zeros(()), metadata={"_media": gen.metadata["_media_rows"][i]}))
    api.train_batch(exps, policy_ratio_clip_eps=0.2, optimize_iterations_per_step=1, max_grad_norm=1.0)
    params = {m.module_name: (m.a.detach().clone(), m.b.detach().clone()) for m in api.adapter.model.lora.modules}
    return seqs, olds, params


def _samples(img_dir):
    from graspo_b200.core.data import sample_from_record
    from graspo_b200.utils.synth import synthetic_image_records

    return [sample_from_record(r) for r in synthetic_image_records(2, img_dir, seed=3, size=64, text_words=4)]


def _worker(rank, world, path, img_dir, out_dir, ref_file):
    from graspo_b200.engine.runtime import GraspoFlowRuntime

    os.makedirs(os.path.join(out_dir, "logs"), exist_ok=True)
    api = GraspoFlowRuntime.from_config(_config(path, out_dir, 2))
    api.setup()
    seqs, olds, params = _round(api, _samples(img_dir))
    ref = torch.load(ref_file)
    for a, b in zip(seqs, ref["seqs"], strict=True):
        assert torch.equal(a, b), "pipelined image rollout differs from the single-stage one"
    for a, b in zip(olds, ref["olds"], strict=True):
        assert (a - b).abs().max().item() < 1e-4
    lora = api.adapter.model.lora
    if rank == 0:
        assert lora.vision_modules(), "the first stage owns the tower's LoRA modules"
    else:
        assert not lora.vision_modules()
    # one AdamW step of lr 1e-2 moves every factor entry by up to ~lr; summation
    # order differences only show in entries whose gradient is near zero
    for name, (a, b) in params.items():
        ra, rb = ref["params"][name]
        assert (a - ra).abs().max().item() < 5e-4, (name, "A")
        assert (b - rb).abs().max().item() < 5e-4, (name, "B")
    if rank == 0:
        assert any(ref["params"][n][1].abs().max() > 1e-3 for n in params if n.startswith("visual.")), \
            "the step moved the tower's LoRA factors"
    from graspo_b200.parallel import state as pstate

    pstate.destroy()


def test_images_through_pipeline_stages_match_single_stage(tmp_path):
    from graspo_b200.engine.runtime import GraspoFlowRuntime
    from graspo_b200.utils.synth import QWEN35_TINY, VIT_TINY, add_vision_tower, write_qwen35_checkpoint

    os.environ.setdefault("GLOO_SOCKET_IFNAME", "lo")
    base = write_qwen35_checkpoint(tmp_path / "vl35", dict(QWEN35_TINY, vocab_size=2048, head_dim=64), seed=1,
                                   std=0.05)
    path = add_vision_tower(base, VIT_TINY, seed=2)
    img_dir = tmp_path / "img"
    samples = _samples(img_dir)
    (tmp_path / "run1" / "logs").mkdir(parents=True)
    api = GraspoFlowRuntime.from_config(_config(path, tmp_path / "run1", 1))
    api.setup()
    seqs, olds, params = _round(api, samples)
    moved = [n for n in params if n.startswith("visual.")]
    assert moved, "vision LoRA modules exist"
    ref_file = tmp_path / "ref.pt"
    torch.save({"seqs": seqs, "olds": olds, "params": params}, ref_file)
    run_world(2, _worker, str(path), str(img_dir), str(tmp_path / "run2"), str(ref_file), timeout=600)


# ---------------------------------------------------------------------------
# Dense Qwen3 on the fused kernel path (emulated kernels on CPU): the first
# stage places the image features per micro-batch; with LoRA on the tower the
# embedding gradients of the image rows go back through the tower once.

PAD = 2000
QWEN3_TARGETS = {"language.self_attn.q_proj", "language.self_attn.o_proj", "language.mlp.down_proj",
                 "visual.merger.linear_fc1", "visual.merger.linear_fc2", "visual.blocks.1.attn.qkv"}


def _qwen3(path, ps, layers, embed, head):
    import zlib

    from graspo_b200.models.config import load_decoder_config
    from graspo_b200.models.loader import SafetensorIndex
    from graspo_b200.models.qwen3 import Qwen3Model

    m = Qwen3Model(load_decoder_config(path), SafetensorIndex(path), ps=ps, local_layers=layers,
                   include_embed=embed, include_head=head, lora_targets=QWEN3_TARGETS, lora_r=4, lora_alpha=8,
                   lora_dropout=0.0, dtype=torch.float32, device=torch.device("cpu"), seed=3)
    with torch.no_grad():
        for mod in m.lora.modules:
            g = torch.Generator().manual_seed(zlib.crc32(mod.module_name.encode()))
            mod.b.copy_(torch.randn(mod.b.shape, generator=g) * 0.05)
    m.lora.invalidate()
    return m


def _image_batch():
    from graspo_b200.models.vision import VisionConfig, preprocess
    from graspo_b200.utils.synth import VIT_TINY

    g = torch.Generator().manual_seed(4)
    cfg = VisionConfig.from_dict(VIT_TINY)
    images = [torch.randint(0, 256, (64, 64, 3), generator=g, dtype=torch.uint8) for _ in range(3)]
    pre = [preprocess(im, cfg) for im in images]
    m = cfg.spatial_merge_size
    grids = [(t, gh // m, gw // m) for _, (t, gh, gw) in pre]
    # three rows: one image, none, two images (4 merged tokens each)
    rows = [[5, 6] + [PAD] * 4 + list(range(30, 48)),
            list(range(60, 84)),
            [7] + [PAD] * 4 + [8, 9] + [PAD] * 4 + list(range(90, 103))]
    seq = torch.tensor(rows)
    mask = torch.ones_like(seq, dtype=torch.bool)
    mask[1, :3] = False
    w = torch.randn(3, seq.shape[1] - 1, generator=g) * (mask[:, :-1] & mask[:, 1:])
    return seq, mask, w, [p for p, _ in pre], [grid for _, grid in pre], grids


def _fused_reference(f, seq, mask, w, patches, grids, merged):
    """Single-stage log-probs and LoRA gradients (tower included) of sum(w * logp)."""
    from graspo_b200.models.fused import AttnMeta
    from graspo_b200.models.vision import ImageInputs, VisionLoRA
    from graspo_b200.ops._ext import ext

    m = f.m
    m.lora.grads.zero_()
    vl = VisionLoRA(m.lora, training=True)
    hook = ImageInputs(m.vision.encode(patches, grids, lora=vl), PAD, merged)
    meta = AttnMeta.from_mask(mask)
    x0g = hook(seq, f.embed(seq))
    xL, inputs = f.stage_forward(x0g.detach(), meta, train=True, keep_inputs=True)
    hn, rstd = f.final_norm(xL)
    tgt = torch.zeros_like(seq)
    tgt[:, :-1] = seq[:, 1:]
    lp, lse = f.token_logprobs(hn, tgt.reshape(-1))
    g = torch.zeros(seq.shape)
    g[:, :-1] = w
    dhn = f.token_logprobs_backward(hn, tgt.reshape(-1), lse, g.view(-1))
    dx = torch.empty_like(xL)
    ext().rmsnorm_bwd(dhn, xL, m.norm, rstd, None, dx, m.cfg.rms_norm_eps)
    dx0 = f.stage_backward(inputs, dx, meta, train=True)
    torch.autograd.backward(x0g, dx0.view_as(x0g).to(x0g.dtype))
    vl.accumulate()
    return lp.view(seq.shape)[:, :-1].detach()


def _fused_worker(rank, world, path):
    from graspo_b200.engine.pipeline import pp_logprobs, pp_train
    from graspo_b200.models.fused import FusedQwen3
    from graspo_b200.models.vision import ImageInputs, VisionLoRA
    from graspo_b200.ops.emulate import use_emulation
    from graspo_b200.parallel import state as pstate
    from graspo_b200.parallel.p2p import StageComm
    from graspo_b200.parallel.state import ParallelState

    ps = pstate.initialize(1, 2, 0, timeout_sec=60, device="cpu")
    comm = StageComm(ps)
    seq, mask, w, patches, grids, merged = _image_batch()
    first = rank == 0
    with use_emulation():
        stage = _qwen3(path, ps, [0] if first else [1], first, not first)
        ref = _qwen3(path, ParallelState(), [0, 1], True, True)
        lp_ref = _fused_reference(FusedQwen3(ref), seq, mask, w, patches, grids, merged)
        fs = FusedQwen3(stage)
        hook = None
        if first:
            with torch.no_grad():
                hook = ImageInputs(stage.vision.encode(patches, grids, lora=VisionLoRA(stage.lora, training=False)),
                                   PAD, merged)
        lp = pp_logprobs(fs, comm, seq, mask, seq[:, 1:], chunk_rows=1, embed_hook=hook)
        valid = mask[:, :-1] & mask[:, 1:]
        err = (lp - lp_ref).abs()[valid]
        assert err.max().item() < 1e-4, (err.max().item(), (lp - lp_ref).abs().max(1))
        stage.lora.grads.zero_()
        vl = None
        if first:
            vl = VisionLoRA(stage.lora, training=True)
            hook = ImageInputs(stage.vision.encode(patches, grids, lora=vl), PAD, merged)

        def loss_fn(lp_c, sl):
            return (lp_c * w[sl]).sum().reshape(1), w[sl].clone()

        pp_train(fs, comm, seq, mask, seq[:, 1:], loss_fn, seed=0, chunk_rows=1, schedule="one_f_one_b",
                 embed_hook=hook)
        if vl is not None:
            vl.accumulate()
    names = [mod.module_name for mod in stage.lora.modules]
    assert any(n.startswith("visual.") for n in names) == first
    for mod in stage.lora.modules:
        rm = ref.lora.by_name[mod.module_name]
        for a, b in ((mod.a_grad, rm.a_grad), (mod.b_grad, rm.b_grad)):
            assert b.abs().max().item() > 0, mod.module_name
            err = (a - b).abs().max().item()
            assert err <= 1e-4 * (b.abs().max().item() + 1e-3), (mod.module_name, err)
    pstate.destroy()


def test_images_through_fused_pipeline_stages(tmp_path):
    from graspo_b200.utils.synth import TINY, VIT_TINY, add_vision_tower, write_qwen3_checkpoint

    os.environ.setdefault("GLOO_SOCKET_IFNAME", "lo")
    base = write_qwen3_checkpoint(tmp_path / "vl", dict(TINY, head_dim=128), seed=1, device="cpu")
    path = add_vision_tower(base, VIT_TINY, seed=2)
    run_world(2, _fused_worker, str(path), timeout=600)
