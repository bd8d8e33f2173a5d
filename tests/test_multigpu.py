"""Tensor parallelism on real GPUs (NCCL): the fused TP=2 model matches the
fused TP=1 model (log-probs, LoRA gradients, greedy rollout).  Needs 2 GPUs."""

import os

import pytest
import torch

from tests.dist_util import run_world

pytestmark = pytest.mark.gpu

SMALL = dict(vocab_size=4096, hidden_size=512, intermediate_size=1024, num_hidden_layers=2,
             num_attention_heads=4, num_key_value_heads=2, head_dim=128)
TARGETS = {"language.self_attn.q_proj", "language.self_attn.k_proj", "language.self_attn.v_proj",
           "language.self_attn.o_proj", "language.mlp.gate_proj", "language.mlp.up_proj", "language.mlp.down_proj"}


def _build(path, ps):
    import zlib

    from graspo_b200.models.config import load_decoder_config
    from graspo_b200.models.loader import SafetensorIndex
    from graspo_b200.models.qwen3 import Qwen3Model

    m = Qwen3Model(load_decoder_config(path), SafetensorIndex(path), ps=ps, lora_targets=TARGETS, lora_r=8,
                   lora_alpha=16, lora_dropout=0.0, dtype=torch.bfloat16, device=ps.device, seed=3)
    with torch.no_grad():
        for mod in m.lora.modules:
            g = torch.Generator().manual_seed(zlib.crc32(mod.module_name.encode()))
            full = torch.randn(mod.out_full, m.lora.r, generator=g) * 0.05
            mod.b.copy_(full[mod.row_start : mod.row_stop] if mod.shard_kind == "out" else full)
    m.lora.invalidate()
    m.ensure_transposed()
    return m


def _run(m, seq, mask, w):
    from graspo_b200.models.fused import AttnMeta, FusedQwen3
    from graspo_b200.ops._ext import ext

    f = FusedQwen3(m)
    meta = AttnMeta.from_mask(mask)
    m.lora.grads.zero_()
    x, inputs = f.stage_forward(f.embed(seq), meta, train=True, keep_inputs=True)
    hn, rstd = f.final_norm(x)
    tgt = torch.zeros_like(seq)
    tgt[:, :-1] = seq[:, 1:]
    lp, lse = f.token_logprobs(hn, tgt.reshape(-1))
    g = torch.zeros(seq.shape, device=seq.device)
    g[:, :-1] = w
    dhn = f.token_logprobs_backward(hn, tgt.reshape(-1), lse, g.view(-1))
    dx = torch.empty_like(x)
    ext().rmsnorm_bwd(dhn, x, m.norm, rstd, None, dx, m.cfg.rms_norm_eps)
    f.stage_backward(inputs, dx, meta, train=True)
    return lp.view(seq.shape)[:, :-1]


def _worker(rank, world, path):
    from graspo_b200.engine.rollout import FusedRolloutEngine
    from graspo_b200.models.fused import FusedQwen3
    from graspo_b200.parallel import state as pstate
    from graspo_b200.parallel.state import ParallelState

    os.environ["NCCL_NVLS_ENABLE"] = "0"
    ps = pstate.initialize(2, 1, 0, timeout_sec=120)
    g = torch.Generator().manual_seed(0)
    seq = torch.randint(0, 4088, (3, 96), generator=g).cuda()
    mask = torch.ones(3, 96, dtype=torch.bool, device="cuda")
    mask[1, :17] = False
    w = torch.randn(3, 95, generator=g).cuda() * (mask[:, :-1] & mask[:, 1:])
    m2 = _build(path, ps)
    lp2 = _run(m2, seq, mask, w)
    torch.distributed.all_reduce(m2.lora.grads[: m2.lora.replicated_numel], group=ps.tp_group)
    m1 = _build(path, ParallelState(device=ps.device))
    lp1 = _run(m1, seq, mask, w)
    valid = mask[:, :-1] & mask[:, 1:]
    assert (lp1 - lp2).abs()[valid].max().item() < 0.08
    cos = []
    for mod2 in m2.lora.modules:
        mod1 = m1.lora.by_name[mod2.module_name]
        if mod2.shard_kind == "out":
            a1, b1 = mod1.a_grad, mod1.b_grad[mod2.row_start : mod2.row_stop]
        else:
            a1, b1 = mod1.a_grad[:, mod2.col_start : mod2.col_stop], mod1.b_grad
        for x1, x2 in ((a1, mod2.a_grad), (b1, mod2.b_grad)):
            cos.append(torch.nn.functional.cosine_similarity(x1.flatten(), x2.flatten(), dim=0).item())
    assert min(cos) > 0.98, cos
    # decode through NCCL collectives captured in a CUDA graph: both ranks agree
    res = FusedRolloutEngine(m2, FusedQwen3(m2), page_size=64).generate(
        [[5, 6, 7], list(range(20, 90))], group_size=2, max_new_tokens=20, temperature=1.0, top_p=1.0,
        eos_id=4095, pad_id=4095, ignore_eos=True, seed=11)
    toks = res.tokens.cuda()
    other = toks.clone()
    torch.distributed.broadcast(other, src=0)
    assert torch.equal(toks, other), "TP ranks sampled different tokens"
    pstate.destroy()


def _peer_reduce_worker(rank, world):
    from graspo_b200.ops._ext import check_errors, ext
    from graspo_b200.ops.gemm import gemm
    from graspo_b200.parallel import state as pstate
    from graspo_b200.parallel.symm import PeerReduce

    os.environ["NCCL_NVLS_ENABLE"] = "0"
    ps = pstate.initialize(2, 1, 0, timeout_sec=120)
    C = ext()
    rows, H, tail, K = 96, 1024, 64, 768
    site = PeerReduce(rows, H + tail, ps.tp_group, ps.device)
    g = torch.Generator(device="cuda").manual_seed(100 + rank)
    shared = torch.Generator(device="cuda").manual_seed(7)
    h = torch.randn(rows, H, device="cuda", generator=shared).bfloat16()
    w = (torch.rand(H, device="cuda", generator=shared) + 0.5).bfloat16()
    lb = (torch.randn(H, 64, device="cuda", generator=shared) * 0.1).bfloat16()
    ws = torch.zeros(rows, H + tail, device="cuda")
    for it in range(3):  # counters must come back to their start state every step
        W = (torch.randn(H + tail, K, device="cuda", generator=g) * 0.05).bfloat16()
        x = torch.randn(rows, K, device="cuda", generator=g).bfloat16()
        gemm(W, x, ws, swap=True, epilogue="atomic", splits=3, push=site)
        h_out = torch.empty_like(h)
        y = torch.empty_like(h)
        # the norm kernel takes the LoRA B factor transposed: B^T [r, H]
        lbt = lb[:, :16].T.contiguous()
        C.add_rmsnorm(h, ws, h_out, w, y, None, None, None, 1.0, 1e-6, lbt, 16, **site.norm_kwargs())
        torch.cuda.synchronize()
        check_errors()
        part = x.float() @ W.float().T
        parts = [torch.empty_like(part) for _ in range(2)]
        torch.distributed.all_gather(parts, part, group=ps.tp_group)
        tot = parts[0] + parts[1]
        d = tot[:, :H] + tot[:, H : H + 16] @ lb[:, :16].float().T
        xr = (h.float() + d).bfloat16().float()
        ref = (xr * torch.rsqrt(xr.pow(2).mean(-1, keepdim=True) + 1e-6) * w.float()).bfloat16()
        err = (y.float() - ref.float()).abs().max().item()
        assert err < 0.05 * ref.float().abs().max().item(), f"step {it}: max err {err}"
        assert torch.count_nonzero(ws).item() == 0, "workspace must be zeroed by the consumer"
        other = y.clone()
        torch.distributed.broadcast(other, src=0, group=ps.tp_group)
        assert torch.equal(y, other), "ranks must hold bit-identical sums"
    site.close()
    pstate.destroy()


@pytest.mark.skipif(torch.cuda.device_count() < 2, reason="needs 2 GPUs")
def test_fused_tp_allreduce_matches_nccl():
    run_world(2, _peer_reduce_worker, timeout=300)


def _tp_reduce_worker(rank, world):
    """GEMM slot push + tp_reduce over real peers == the NCCL sum of the same partials."""
    import torch.distributed as dist

    from graspo_b200.ops._ext import check_errors
    from graspo_b200.ops.gemm import gemm
    from graspo_b200.parallel import state as pstate
    from graspo_b200.parallel.symm import TPAllReduce

    os.environ["NCCL_NVLS_ENABLE"] = "0"
    ps = pstate.initialize(world, 1, 0, timeout_sec=120)
    H = 1024
    red = TPAllReduce(ps.tp_group, ps.device, H)
    g = torch.Generator(device="cuda").manual_seed(100 + rank)
    shared = torch.Generator(device="cuda").manual_seed(7)
    # the 4096-token site outgrows the slots: the buffers are re-made mid-sequence
    for T, scatter in [(512, False), (256, True), (4096, False), (640, True), (300, False), (1024, True),
                       (8192, False), (8192, True)]:
        rows = T // world if scatter else T
        a = (torch.randn(T, 384, device="cuda", generator=g) * 0.5).bfloat16()
        w = (torch.randn(H, 384, device="cuda", generator=g) * 0.5).bfloat16()
        res = torch.randn(rows, H, device="cuda", generator=shared).bfloat16()
        if T == 640:
            # the GEMM epilogue's own slot push (kept as a tested library path)
            push = red.begin(T, scatter=scatter)
            gemm(a, w, push.pop("out"), push=push)
            y = red.finish(residual=res)
        else:
            y = red.gemm_reduce(lambda rows, dst: gemm(a[rows], w, dst), T, scatter=scatter, residual=res)
        part = (a.float() @ w.float().T).bfloat16().float()
        parts = [torch.empty_like(part) for _ in range(world)]
        dist.all_gather(parts, part)
        total = parts[0]
        for q in range(1, world):
            total = total + parts[q]
        if scatter:
            total = total[rank * rows : (rank + 1) * rows]
        want = total + res.float()
        err = (y.float() - want).abs().max().item() / want.abs().max().item()
        assert err < 1e-2, (T, scatter, err)
        if not scatter:
            other = [torch.empty_like(y) for _ in range(world)]
            dist.all_gather(other, y)
            assert all(torch.equal(o, y) for o in other), "ranks must hold bit-identical sums"
    # vocab-parallel log-prob: each rank holds a vocabulary shard of the head
    T, Hd, V = 300, 256, 4096
    h = (torch.randn(T, Hd, device="cuda", generator=shared)).bfloat16()
    head = (torch.randn(V, Hd, device="cuda", generator=shared) * 0.2).bfloat16()
    tgt = torch.randint(0, V, (T,), device="cuda", generator=shared)
    vs = V // world
    local = head[rank * vs : (rank + 1) * vs].contiguous()
    nblk = -(-vs // 256)
    part = torch.empty(T, nblk, 2, device="cuda")
    tl = torch.zeros(T, device="cuda")
    gemm(h, local, torch.empty(0, device="cuda"), epilogue="lse", aux=part.view(T, nblk * 2),
         targets=(tgt - rank * vs).contiguous(), tgt_logit=tl, bn=256)
    lse, logp = red.lse_exchange(part, tl)
    logits = h.float() @ head.float().T
    want_lse = torch.logsumexp(logits, -1)
    want = logits.gather(1, tgt[:, None]).squeeze(1) - want_lse
    assert (lse - want_lse).abs().max().item() < 2e-3
    assert (logp - want).abs().max().item() < 2e-3
    # vocab-parallel sampling: the shards' winners through peer memory == one full-vocabulary pass
    from graspo_b200.ops._ext import ext, err_word
    from graspo_b200.parallel.symm import SampleExchange

    rows, V = 6, 151936
    logits = torch.randn(rows, V, device="cuda", generator=shared) * 2
    vs = V // world
    sx = SampleExchange(rows, ps.tp_group, ps.device)

    def state():
        return [torch.zeros(rows, dtype=torch.long, device="cuda"),
                torch.arange(rows, device="cuda", dtype=torch.long) + 7,
                torch.zeros(rows, dtype=torch.long, device="cuda"), torch.zeros(rows, dtype=torch.int32, device="cuda"),
                torch.zeros(rows, dtype=torch.uint8, device="cuda"), torch.zeros(rows, 16, dtype=torch.long, device="cuda")]

    full, part = state(), state()
    chunk = 4096
    scratch = torch.zeros(rows * (1 + 2 * (-(-vs // chunk))) + 2, device="cuda")
    local = logits[:, rank * vs : (rank + 1) * vs].contiguous()
    tick = torch.zeros(1, device="cuda")
    for _ in range(4):
        ext().sample_append(logits, 1.0, 1.0, 5, *full, 3, -1, 0, True, None)
        ext().sample_append_split(local, 1.0, 5, *part, 3, -1, 0, True, rank * vs, scratch, chunk, err_word(),
                                  **sx.kwargs())
        dist.all_reduce(tick)  # consecutive exchanges are separated by a collective (a decode step has several)
    torch.cuda.synchronize()
    check_errors()
    for x, y in zip(full, part):
        assert torch.equal(x, y)
    sx.close()
    torch.cuda.synchronize()
    check_errors()
    red.close()
    pstate.destroy()


def _dp_worker(rank, world, path):
    """DP=2: LoRA gradients sent layer by layer during the backward and summed by dp_reduce
    equal (1/2 x) the DP=1 gradients of the whole batch, bit-identical on both replicas."""
    import torch.distributed as dist

    from graspo_b200.models.fused import AttnMeta, FusedQwen3
    from graspo_b200.ops._ext import check_errors, ext
    from graspo_b200.parallel import state as pstate
    from graspo_b200.parallel.state import ParallelState
    from graspo_b200.parallel.symm import DPGradReduce

    os.environ["NCCL_NVLS_ENABLE"] = "0"
    ps = pstate.initialize(1, 1, world, timeout_sec=120)
    g = torch.Generator().manual_seed(0)
    B, S = 4, 80
    seq = torch.randint(0, 4088, (B, S), generator=g).cuda()
    mask = torch.ones(B, S, dtype=torch.bool, device="cuda")
    mask[1, :9] = False
    w = torch.randn(B, S - 1, generator=g).cuda() * (mask[:, :-1] & mask[:, 1:])

    def grads_of(m, rows, hook=None):
        f = FusedQwen3(m)
        sq, mk = seq[rows], mask[rows]
        meta = AttnMeta.from_mask(mk)
        m.lora.grads.zero_()
        x, inputs = f.stage_forward(f.embed(sq), meta, train=True, keep_inputs=True)
        hn, rstd = f.final_norm(x)
        tgt = torch.zeros_like(sq)
        tgt[:, :-1] = sq[:, 1:]
        lp, lse = f.token_logprobs(hn, tgt.reshape(-1))
        gg = torch.zeros(sq.shape, device="cuda")
        gg[:, :-1] = w[rows]
        dhn = f.token_logprobs_backward(hn, tgt.reshape(-1), lse, gg.view(-1))
        dx = torch.empty_like(x)
        ext().rmsnorm_bwd(dhn, x, m.norm, rstd, None, dx, m.cfg.rms_norm_eps)
        f.stage_backward(inputs, dx, meta, train=True, on_layer_done=hook)
        return m.lora.grads

    m2 = _build(path, ps)
    red = DPGradReduce(m2.lora.numel, ps.dp_group, ps.device)
    half = slice(rank * B // world, (rank + 1) * B // world)
    for step in range(3):  # both slot sets, twice
        gr = grads_of(m2, half, hook=lambda layer: red.push(m2.lora.grads, m2.lora.layer_ranges(layer)))
        red.finish(gr)
        torch.cuda.synchronize()
        check_errors()
        other = [torch.empty_like(gr) for _ in range(world)]
        dist.all_gather(other, gr)
        assert all(torch.equal(o, gr) for o in other), "replicas must hold bit-identical gradients"
    m1 = _build(path, ParallelState(device=ps.device))
    full = grads_of(m1, slice(0, B)) / world
    err = (gr - full).abs().max().item() / full.abs().max().item()
    assert err < 2e-2, err
    red.close()
    pstate.destroy()


@pytest.mark.skipif(torch.cuda.device_count() < 2, reason="needs 2 GPUs")
def test_dp2_overlapped_grad_reduce_matches_dp1(tmp_path):
    from graspo_b200.utils.synth import write_qwen3_checkpoint

    path = write_qwen3_checkpoint(tmp_path / "small", SMALL, seed=4, std=0.05, with_tokenizer=False)
    run_world(2, _dp_worker, path, timeout=600)


@pytest.mark.skipif(torch.cuda.device_count() < 2, reason="needs 2 GPUs")
def test_fused_gemm_tp_reduce_matches_nccl():
    run_world(2, _tp_reduce_worker, timeout=300)


@pytest.mark.skipif(torch.cuda.device_count() < 2, reason="needs 2 GPUs")
def test_tp2_fused_matches_tp1(tmp_path):
    from graspo_b200.utils.synth import write_qwen3_checkpoint

    path = write_qwen3_checkpoint(tmp_path / "small", SMALL, seed=4, std=0.05, with_tokenizer=False)
    run_world(2, _worker, path, timeout=600)


def _pp_worker(rank, world, path):
    from graspo_b200.engine.pipeline import pp_logprobs
    from graspo_b200.engine.rollout import FusedRolloutEngine
    from graspo_b200.models.config import load_decoder_config
    from graspo_b200.models.fused import FusedQwen3
    from graspo_b200.models.loader import SafetensorIndex
    from graspo_b200.models.qwen3 import Qwen3Model
    from graspo_b200.parallel import state as pstate
    from graspo_b200.parallel.p2p import StageComm
    from graspo_b200.parallel.state import ParallelState

    os.environ["NCCL_NVLS_ENABLE"] = "0"
    ps = pstate.initialize(1, 2, 0, timeout_sec=120)
    comm = StageComm(ps)

    def build(ps_, layers, embed, head):
        return Qwen3Model(load_decoder_config(path), SafetensorIndex(path), ps=ps_, local_layers=layers,
                          include_embed=embed, include_head=head, lora_targets=TARGETS, lora_r=8, lora_alpha=16,
                          lora_dropout=0.0, dtype=torch.bfloat16, device=ps.device, seed=3)

    stage = build(ps, [0] if rank == 0 else [1], rank == 0, rank == 1)
    ref = build(ParallelState(device=ps.device), [0, 1], True, True)
    g = torch.Generator().manual_seed(0)
    seq = torch.randint(0, 4088, (3, 96), generator=g).cuda()
    mask = torch.ones(3, 96, dtype=torch.bool, device="cuda")
    mask[1, :17] = False
    lp = pp_logprobs(FusedQwen3(stage), comm, seq, mask, seq[:, 1:], chunk_rows=1)
    f = FusedQwen3(ref)
    from graspo_b200.models.fused import AttnMeta

    x, _ = f.stage_forward(f.embed(seq), AttnMeta.from_mask(mask))
    hn, _ = f.final_norm(x)
    tgt = torch.zeros_like(seq)
    tgt[:, :-1] = seq[:, 1:]
    lp_ref = f.token_logprobs(hn, tgt.reshape(-1))[0].view(seq.shape)[:, :-1]
    valid = mask[:, :-1] & mask[:, 1:]
    assert (lp - lp_ref).abs()[valid].max().item() < 0.08
    kw = dict(group_size=2, max_new_tokens=12, temperature=1.0, top_p=1.0, eos_id=4095, pad_id=4095,
              ignore_eos=True, seed=7)
    prompts = [[5, 6, 7], list(range(20, 90))]
    got = FusedRolloutEngine(stage, FusedQwen3(stage), page_size=64, comm=comm).generate(prompts, **kw)
    toks = got.tokens.cuda()
    other = toks.clone()
    torch.distributed.broadcast(other, src=1)
    assert torch.equal(toks, other), "pipeline stages disagree on the sampled tokens"
    pstate.destroy()


@pytest.mark.skipif(torch.cuda.device_count() < 2, reason="needs 2 GPUs")
def test_pipeline_two_stages_on_gpus(tmp_path):
    from graspo_b200.utils.synth import write_qwen3_checkpoint

    path = write_qwen3_checkpoint(tmp_path / "pp", SMALL, seed=4, std=0.05, with_tokenizer=False)
    run_world(2, _pp_worker, path, timeout=600)
