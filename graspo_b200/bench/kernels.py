"""Kernel micro-benchmarks: CUDA-event timing, warm-up, L2 flush between runs.

``python -m graspo_b200.bench.kernels gemm`` times the tcgen05 GEMM on the
Qwen3-8B projection shapes next to ``torch.matmul`` (cuBLAS) on the same
inputs and prints one JSON line per case with achieved TFLOP/s and the
fraction of the measured bf16 peak.  ``decode`` times the swap-AB decode GEMMs
and the paged decode attention as bytes/s against the measured copy bandwidth.
``step`` runs the rollout engine on a Qwen3-8B-shaped model with fewer layers
(every layer has the 8B shapes, so per-layer figures carry over) and reports
the decode-step time per layer with and without the CUDA graph; its eager
decode steps sit in NVTX ranges named ``decode_step`` so that a profiler can
select exactly those launches.
"""

from __future__ import annotations

import argparse
import json
import math
from pathlib import Path

import torch

L2_FLUSH_BYTES = 256 << 20


def measured_peaks() -> dict:
    path = Path(__file__).resolve().parents[2] / "MEASURED_PEAKS.json"
    if path.exists():
        return json.loads(path.read_text())
    return {"hbm_gbs": 6650.0, "bf16_tflops": 1590.0, "fallback": True}


class Timer:
    def __init__(self, warmup: int = 3, iters: int = 10, flush: bool = True) -> None:
        self.warmup, self.iters, self.flush = warmup, iters, flush
        self._buf = torch.empty(L2_FLUSH_BYTES, dtype=torch.uint8, device="cuda") if flush else None

    def __call__(self, fn) -> float:
        """Median milliseconds of ``fn()`` over ``iters`` runs."""
        for _ in range(self.warmup):
            fn()
        torch.cuda.synchronize()
        times = []
        for _ in range(self.iters):
            if self._buf is not None:
                self._buf.zero_()
            start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            start.record()
            fn()
            end.record()
            torch.cuda.synchronize()
            times.append(start.elapsed_time(end))
        times.sort()
        return times[len(times) // 2]


def bench_gemm(args) -> None:
    from graspo_b200.ops._ext import check_errors
    from graspo_b200.ops.gemm import gemm

    peaks = measured_peaks()
    timer = Timer(iters=args.iters)
    shapes = [
        ("qkv", 8192, 6144, 4096),
        ("o", 8192, 4096, 4096),
        ("gate_up", 8192, 24576, 4096),
        ("down", 8192, 4096, 12288),
        ("train_qkv", 24576, 6144, 4096),
        ("train_gate_up", 24576, 24576, 4096),
        ("lm_head", 8192, 151936, 4096),
    ]
    for name, m, n, k in shapes:
        a = torch.randn(m, k, device="cuda").bfloat16()
        b = torch.randn(n, k, device="cuda").bfloat16()
        c = torch.empty(m, n, device="cuda", dtype=torch.bfloat16)
        flops = 2.0 * m * n * k
        ours = timer(lambda: gemm(a, b, c))
        ours128 = timer(lambda: gemm(a, b, c, bn=128))
        ref = timer(lambda: torch.matmul(a, b.T, out=c))
        check_errors()
        print(json.dumps({
            "kernel": "gemm_tc", "case": name, "m": m, "n": n, "k": k,
            "ms": round(ours, 4), "tflops": round(flops / ours / 1e9, 1),
            "frac_of_measured_bf16": round(flops / ours / 1e9 / peaks["bf16_tflops"], 3),
            "cublas_ms": round(ref, 4), "cublas_tflops": round(flops / ref / 1e9, 1),
            "speedup_vs_cublas": round(ref / ours, 3), "ms_bn128": round(ours128, 4),
        }), flush=True)
        del a, b, c


def bench_decode(args) -> None:
    from graspo_b200.ops._ext import check_errors, ext
    from graspo_b200.ops.gemm import gemm

    peaks = measured_peaks()
    timer = Timer(iters=args.iters)
    T = args.tokens
    for name, n, k, splits in [("qkv", 6144, 4096, 3), ("o", 4096, 4096, 4), ("gate_up", 24576, 4096, 1),
                               ("down", 4096, 12288, 4), ("lm_head", 151936, 4096, 1)]:
        w = torch.randn(n, k, device="cuda").bfloat16()
        x = torch.randn(T, k, device="cuda").bfloat16()
        if splits > 1:
            out = torch.zeros(T, n, device="cuda")
            fn = lambda: gemm(w, x, out, swap=True, epilogue="atomic", splits=splits)  # noqa: E731
        else:
            out = torch.empty(T, n, device="cuda", dtype=torch.float32 if name == "lm_head" else torch.bfloat16)
            epi = "store_f32" if name == "lm_head" else "store"
            fn = lambda: gemm(w, x, out, swap=True, epilogue=epi)  # noqa: E731
        ms = timer(fn)
        if name == "gate_up":
            # the decode step runs gate/up as split-K 3 with a last-split SwiGLU
            act = torch.empty(T, n // 2, device="cuda", dtype=torch.bfloat16)
            ws = torch.empty(4 * T * n, device="cuda")
            ctr = torch.zeros(-(-n // 128) * -(-T // 64), device="cuda", dtype=torch.int32)
            for sp in (1, 2, 3, 4):
                kw = dict(aux=ws, tile_ctr=ctr) if sp > 1 else {}
                ms_s = timer(lambda: gemm(w, x, act, swap=True, epilogue="swiglu", splits=sp, **kw))  # noqa: B023
                print(json.dumps({"kernel": "gemm_tc_swap_swiglu", "tokens": T, "n": n, "k": k, "splits": sp,
                                  "ms": round(ms_s, 4),
                                  "frac_of_measured_hbm": round(n * k * 2 / ms_s / 1e6 / peaks["hbm_gbs"], 3)}),
                      flush=True)
        ref = timer(lambda: torch.matmul(x, w.T))
        check_errors()
        nbytes = n * k * 2 + T * k * 2
        print(json.dumps({
            "kernel": "gemm_tc_swap", "case": name, "tokens": T, "n": n, "k": k, "splits": splits,
            "ms": round(ms, 4), "GBps": round(nbytes / ms / 1e6, 1),
            "frac_of_measured_hbm": round(nbytes / ms / 1e6 / peaks["hbm_gbs"], 3),
            "cublas_ms": round(ref, 4),
        }), flush=True)
    # paged decode attention: rows x context
    nq, nkv, D, page = 32, 8, 128, 64
    for ctx in (1024, 2048, 3072):
        rows = T
        pages_per_row = math.ceil(ctx / page)
        num_pages = rows * pages_per_row
        kp = torch.randn(num_pages, nkv, page, D, device="cuda").bfloat16()
        vp = torch.randn_like(kp)
        bt = torch.arange(num_pages, device="cuda", dtype=torch.int32).view(rows, pages_per_row)
        q = torch.randn(rows, nq, D, device="cuda").bfloat16()
        start = torch.zeros(rows, device="cuda", dtype=torch.int32)
        ln = torch.full((rows,), ctx, device="cuda", dtype=torch.int32)
        out = torch.empty(rows, nq * D, device="cuda", dtype=torch.bfloat16)
        from graspo_b200.engine.rollout import decode_attention_splits

        splits = decode_attention_splits(rows, nkv, ctx)
        scratch = torch.zeros(rows * nq * splits * (D + 2) + rows * nkv, device="cuda")
        ms = timer(lambda: ext().paged_decode_attention(q, kp, vp, bt, start, ln, out, 1 / math.sqrt(D), splits,
                                                        scratch))
        nbytes = 2 * rows * ctx * nkv * D * 2
        print(json.dumps({
            "kernel": "paged_decode_attention", "rows": rows, "ctx": ctx, "splits": splits, "ms": round(ms, 4),
            "GBps": round(nbytes / ms / 1e6, 1),
            "frac_of_measured_hbm": round(nbytes / ms / 1e6 / peaks["hbm_gbs"], 3),
        }), flush=True)


def bench_attn(args) -> None:
    """Decode attention on the GRASPO shape: ``--prompts`` groups of ``--group`` rows sharing a
    ``--prompt-len`` prompt, each row with ``--new`` generated keys (32 / 8 heads, page 64).

    Times the mma.sync split kernel (prompt keys re-read per row) and the tcgen05 / TMA kernel
    (prompt keys once per group), with the bytes each must read and the fraction of the measured
    HBM copy rate."""
    from graspo_b200.engine.rollout import decode_attention_splits, decode_tc_splits
    from graspo_b200.ops._ext import check_errors, err_word, ext

    peaks = measured_peaks()
    timer = Timer(iters=args.iters)
    nq, nkv, D, page = 32, 8, 128, 64
    n, G, P, gen = args.prompts, args.group, args.prompt_len, args.new
    rows = n * G
    pp, gp = P // page, -(-gen // page)
    num_pages = n * pp + rows * gp
    kp = torch.randn(num_pages, nkv, page, D, device="cuda").bfloat16()
    vp = torch.randn_like(kp)
    bt = torch.empty(rows, pp + gp, dtype=torch.int32)
    for r in range(rows):
        bt[r, :pp] = torch.arange((r // G) * pp, (r // G + 1) * pp)
        bt[r, pp:] = torch.arange(n * pp + r * gp, n * pp + (r + 1) * gp)
    bt = bt.cuda()
    q = torch.randn(rows, nq, D, device="cuda").bfloat16()
    start = torch.zeros(rows, device="cuda", dtype=torch.int32)
    ln = torch.full((rows,), P + gen, device="cuda", dtype=torch.int32)
    out = torch.empty(rows, nq * D, device="cuda", dtype=torch.bfloat16)
    scale = 1 / math.sqrt(D)
    kv_row = nkv * D * 2 * 2  # K and V bytes per key position
    bytes_per_row = rows * (P + gen) * kv_row
    bytes_shared = (n * P + rows * gen) * kv_row
    splits = decode_attention_splits(rows, nkv, P + gp * page)
    scr = torch.zeros(rows * nq * 8 * (D + 2) + rows * nkv, device="cuda")
    old = timer(lambda: ext().paged_decode_attention(q, kp, vp, bt, start, ln, out, scale, splits, scr))
    ref = out.clone()
    for sp in (1, 2, 3, 4, 6, 8):
        ms = timer(lambda: ext().paged_decode_attention(q, kp, vp, bt, start, ln, out, scale, sp, scr))  # noqa: B023
        print(json.dumps({"kernel": "split_mma_sync", "splits": sp, "chosen": sp == splits, "ms": round(ms, 4)}),
              flush=True)
    sp, psp = decode_tc_splits(rows, nkv, gp * page, n, P)
    scr2 = torch.zeros(rows * nq * (sp + psp) * (D + 2) + rows * nkv, device="cuda")
    ew = err_word(q.device)
    new = timer(lambda: ext().paged_decode_attention_tc(q, kp, vp, bt, start, ln, out, scale, sp, scr2, P, G, psp,
                                                        ew))
    check_errors()
    err = (out.float() - ref.float()).abs().max().item()
    for name, ms, nbytes in (("split_mma_sync", old, bytes_per_row), ("tcgen05_shared_prompt", new, bytes_shared)):
        print(json.dumps({
            "kernel": name, "rows": rows, "prompt": P, "generated": gen, "ms": round(ms, 4),
            "bytes": nbytes, "GBps": round(nbytes / ms / 1e6, 1),
            "frac_of_measured_hbm": round(nbytes / ms / 1e6 / peaks["hbm_gbs"], 3),
            "floor_ms_shared": round(bytes_shared / peaks["hbm_gbs"] / 1e6, 4), "max_abs_diff": err,
        }), flush=True)


def bench_push(args) -> None:
    """One process, two GPUs: the TP=2 training o_proj GEMM (24576 x 4096 x 2048) plain, with its
    tiles pushed to a second local slot, and pushed to GPU 1 over NVLink; plus a copy-engine copy
    of the same 201 MB to GPU 1 and the rank-order sum (tp_reduce)."""
    from graspo_b200.ops._ext import check_errors, err_word, ext
    from graspo_b200.ops.gemm import gemm

    if not ext().enable_peer_access(0, 1):
        raise SystemExit("GPU 0 cannot reach GPU 1")
    timer = Timer(iters=args.iters)
    T, H, K = 24576, 4096, 2048
    a = torch.randn(T, K, device="cuda:0").bfloat16()
    w = (torch.randn(H, K, device="cuda:0") * 0.02).bfloat16()
    own = torch.empty(T, H, device="cuda:0", dtype=torch.bfloat16)
    local2 = torch.empty_like(own)
    peer = torch.empty(T, H, device="cuda:1", dtype=torch.bfloat16)
    ctr0 = torch.zeros(2, device="cuda:0", dtype=torch.int64)
    ctr1 = torch.zeros(2, device="cuda:1", dtype=torch.int64)

    def push(dst, ctr):
        return {"push_out": torch.tensor([own.data_ptr(), dst.data_ptr()], dtype=torch.int64),
                "push_sig": torch.tensor([0, ctr.data_ptr()], dtype=torch.int64), "push_self": 0, "push_rows": 0}

    nbytes = T * H * 2
    flops = 2.0 * T * H * K
    res = {}
    res["gemm"] = timer(lambda: gemm(a, w, own))
    res["gemm_push_local"] = timer(lambda: gemm(a, w, own, push=push(local2, ctr0)))
    res["gemm_push_peer"] = timer(lambda: gemm(a, w, own, push=push(peer, ctr1)))
    res["gemm_push_peer_fence_once"] = timer(lambda: gemm(a, w, own, push={**push(peer, ctr1), "push_fence_once": 1}))
    res["gemm_push_local_fence_once"] = timer(lambda: gemm(a, w, own, push={**push(local2, ctr0),
                                                                             "push_fence_once": 1}))
    res["copy_engine_to_peer"] = timer(lambda: ext().peer_copy(peer.data_ptr(), own, 0, nbytes))
    side = torch.cuda.Stream(device="cuda:0")

    def chunked(nch):
        # the GEMM in row chunks; the copy engines send each finished chunk to GPU 1 on a side
        # stream while the next chunk computes
        rows = T // nch
        for c in range(nch):
            sl = slice(c * rows, (c + 1) * rows)
            gemm(a[sl], w, own[sl])
            ev = torch.cuda.Event()
            ev.record()
            side.wait_event(ev)
            with torch.cuda.stream(side):
                ext().peer_copy(peer[sl].data_ptr(), own, c * rows * H * 2, rows * H * 2)
        torch.cuda.current_stream().wait_stream(side)

    res["gemm_chunked_copy2"] = timer(lambda: chunked(2))
    res["gemm_chunked_copy4"] = timer(lambda: chunked(4))
    res["gemm_chunked_copy8"] = timer(lambda: chunked(8))
    done = torch.ones(1, device="cuda:0", dtype=torch.int64)
    out = torch.empty_like(own)
    srcs = torch.tensor([own.data_ptr(), local2.data_ptr()], dtype=torch.int64)
    res["tp_reduce"] = timer(lambda: ext().tp_reduce(srcs, done.data_ptr(), 1, own, out, H, err_word(out.device), 0))
    check_errors(0)
    for name, ms in res.items():
        extra = {"tflops": round(flops / ms / 1e9, 1)} if name.startswith("gemm") else {}
        print(json.dumps({"case": name, "ms": round(ms, 4), "GBps_201MB": round(nbytes / ms / 1e6, 1), **extra}),
              flush=True)


def bench_dsweep(args) -> None:
    """Decode GEMM shapes (``--tokens`` rows, swap layout): tile width x split-K sweep with the
    fraction of the measured HBM copy rate reached on the weight bytes."""
    from graspo_b200.ops._ext import check_errors
    from graspo_b200.ops.gemm import gemm

    peaks = measured_peaks()
    timer = Timer(iters=args.iters)
    T = args.tokens
    x = torch.randn(T, 4096, device="cuda").bfloat16()
    for name, n, k in [("qkv", 6144 + 64, 4096), ("o", 4096 + 64, 4096), ("down", 4096 + 64, 12288),
                       ("gate_up", 24576, 4096)]:
        w = torch.randn(n, k, device="cuda").bfloat16()
        xx = x if k == 4096 else torch.randn(T, k, device="cuda").bfloat16()
        for bn in (32, 64):
            for sp in ((1,) if name == "gate_up" else (1, 2, 3, 4, 6, 8)):
                if name == "gate_up":
                    act = torch.empty(T, n // 2, device="cuda", dtype=torch.bfloat16)
                    ms = timer(lambda: gemm(w, xx, act, swap=True, epilogue="swiglu", bn=bn))  # noqa: B023
                else:
                    ws = torch.zeros(T, n, device="cuda")
                    ms = timer(lambda: gemm(w, xx, ws, swap=True, epilogue="atomic", splits=sp, bn=bn))  # noqa: B023
                print(json.dumps({"case": name, "bn": bn, "splits": sp, "us": round(ms * 1e3, 1),
                                  "frac_of_measured_hbm": round(n * k * 2 / ms / 1e6 / peaks["hbm_gbs"], 3)}),
                      flush=True)
        del w
    check_errors()


def bench_step(args) -> None:
    from graspo_b200.engine.rollout import FusedRolloutEngine
    from graspo_b200.models.fused import FusedQwen3

    model = _step_model(args)
    g = torch.Generator().manual_seed(0)
    prompts = [torch.randint(0, 150000, (args.prompt_len,), generator=g).tolist() for _ in range(args.prompts)]
    configs = {"gn": (True, False), "gp": (True, True), "en": (False, False), "ep": (False, True)}
    for name in args.configs.split(","):
        graph, prefix = configs[name]
        eng = FusedRolloutEngine(model, FusedQwen3(model), page_size=64, use_graph=graph)
        eng.nvtx = not graph
        eng.prefix_attention = prefix
        kw = dict(group_size=args.group, max_new_tokens=args.new, temperature=1.0, top_p=1.0, eos_id=0, pad_id=0,
                  ignore_eos=True, seed=1)
        eng.generate(prompts, **kw)  # warm-up (pools, kernel attributes)
        res = eng.generate(prompts, **kw)
        ms = res.decode_sec * 1e3 / max(1, res.decode_steps - 1)
        print(json.dumps({
            "kernel": "decode_step", "graph": graph, "prefix_attention": prefix, "layers": args.layers,
            "rows": args.prompts * args.group,
            "prompt_len": args.prompt_len, "new_tokens": args.new, "ms_per_step": round(ms, 3),
            "ms_per_layer": round(ms / args.layers, 4), "prefill_s": round(res.prefill_sec, 3),
        }), flush=True)


def _step_model(args):
    from graspo_b200.models.config import load_decoder_config
    from graspo_b200.models.loader import SafetensorIndex
    from graspo_b200.models.qwen3 import Qwen3Model
    from graspo_b200.parallel.state import ParallelState
    from graspo_b200.utils.synth import QWEN3_8B, write_qwen3_checkpoint

    dims = dict(QWEN3_8B, num_hidden_layers=args.layers)
    path = write_qwen3_checkpoint(Path(args.ckpt) / f"qwen3-8b-{args.layers}l", dims, seed=7, device="cuda",
                                  with_tokenizer=False)
    ps = ParallelState(device=torch.device("cuda", 0))
    targets = {f"language.{m}" for m in ("self_attn.q_proj", "self_attn.k_proj", "self_attn.v_proj",
                                          "self_attn.o_proj", "mlp.gate_proj", "mlp.up_proj", "mlp.down_proj")}
    model = Qwen3Model(load_decoder_config(path), SafetensorIndex(path), ps=ps, lora_targets=targets, lora_r=16,
                       lora_alpha=32, lora_dropout=args.dropout, dtype=torch.bfloat16, device=ps.device, seed=1)
    model.ensure_transposed()
    return model


def bench_train(args) -> None:
    """One GRASPO micro-batch (forward with saved inputs, log-probs, backward
    with recompute) on ``--rows`` x ``--seq`` tokens, timed per phase; the
    timed iterations sit in NVTX ranges named ``train_step``."""
    from graspo_b200.models.fused import AttnMeta, FusedQwen3
    from graspo_b200.ops._ext import check_errors, ext

    model = _step_model(args)
    f = FusedQwen3(model)
    B, S = args.rows, args.seq
    g = torch.Generator().manual_seed(0)
    seq = torch.randint(0, 150000, (B, S), generator=g).cuda()
    mask = torch.ones(B, S, dtype=torch.bool, device="cuda")
    for b in range(B):  # left padding in half the rows, right padding in the others
        if b % 2:
            mask[b, : 37 * b] = False
        else:
            mask[b, S - 53 * (b + 1):] = False
    tgt = torch.zeros_like(seq)
    tgt[:, :-1] = seq[:, 1:]
    tgt = tgt.reshape(-1)
    w = torch.randn(B * S, device="cuda") * 1e-3

    def fwd():
        meta = AttnMeta.from_mask(mask)
        x, inputs = f.stage_forward(f.embed(seq), meta, train=True, seed=1, keep_inputs=True)
        hn, rstd = f.final_norm(x)
        lp, lse = f.token_logprobs(hn, tgt)
        return meta, x, inputs, hn, rstd, lse

    def bwd(state):
        meta, x, inputs, hn, rstd, lse = state
        dhn = f.token_logprobs_backward(hn, tgt, lse, w)
        dx = torch.empty_like(x)
        ext().rmsnorm_bwd(dhn, x, model.norm, rstd, None, dx, model.cfg.rms_norm_eps)
        f.stage_backward(inputs, dx, meta, train=True, seed=1)

    for _ in range(2):
        bwd(fwd())
    torch.cuda.synchronize()
    ev = [torch.cuda.Event(enable_timing=True) for _ in range(3)]
    times = []
    for _ in range(args.iters):
        torch.cuda.nvtx.range_push("train_step")
        ev[0].record()
        st = fwd()
        ev[1].record()
        bwd(st)
        ev[2].record()
        torch.cuda.nvtx.range_pop()
        torch.cuda.synchronize()
        times.append((ev[0].elapsed_time(ev[1]), ev[1].elapsed_time(ev[2])))
    check_errors()
    times.sort(key=lambda t: t[0] + t[1])
    fw, bw = times[len(times) // 2]
    tokens = B * S
    print(json.dumps({
        "kernel": "train_microbatch", "layers": args.layers, "rows": B, "seq": S, "dropout": args.dropout,
        "fwd_ms": round(fw, 2), "bwd_ms": round(bw, 2),
        "fwd_ms_per_layer": round(fw / args.layers, 3), "bwd_ms_per_layer": round(bw / args.layers, 3),
        "tokens": tokens,
    }), flush=True)


def bench_hybrid(args) -> None:
    """Training micro-batch of the Qwen3.5 hybrid family (``--layers`` layers of
    the 9B shape, every fourth a gated-attention layer; ``--tiny`` for the test
    shape): autograd forward to the selected-token log-probs with LoRA r=16 on
    every linear of the decoder, then the backward into the LoRA factors, on
    ``--rows`` x ``--seq`` tokens.  CUDA-event timed on a GPU, wall-clock
    otherwise."""
    import time

    from graspo_b200.models.config import load_decoder_config, lora_available_targets
    from graspo_b200.models.loader import SafetensorIndex
    from graspo_b200.models.qwen3 import EagerLoRA
    from graspo_b200.models.qwen35 import Qwen35Model
    from graspo_b200.parallel.state import ParallelState
    from graspo_b200.utils.synth import QWEN35_9B, QWEN35_TINY, write_qwen35_checkpoint

    cuda = torch.cuda.is_available()
    dev = torch.device("cuda", 0) if cuda else torch.device("cpu")
    dims = dict(QWEN35_TINY if args.tiny else QWEN35_9B, num_hidden_layers=args.layers)
    name = f"qwen35-{'tiny' if args.tiny else '9b'}-{args.layers}l"
    path = write_qwen35_checkpoint(Path(args.ckpt) / name, dims, seed=7, with_tokenizer=False)
    cfg = load_decoder_config(path)
    model = Qwen35Model(cfg, SafetensorIndex(path), ps=ParallelState(device=dev),
                        lora_targets=set(lora_available_targets(cfg)), lora_r=16, lora_alpha=32,
                        lora_dropout=args.dropout, dtype=torch.bfloat16 if cuda else torch.float32, device=dev,
                        seed=1)
    B, S = args.rows, args.seq
    g = torch.Generator().manual_seed(0)
    ids = torch.randint(0, dims["vocab_size"] - 8, (B, S), generator=g).to(dev)
    mask = torch.ones(B, S, dtype=torch.bool, device=dev)
    if not args.no_pad:
        mask[0, : S // 8] = False        # a left-padded first row
    w = (torch.randn(B, S - 1, generator=g) * 1e-3).to(dev)

    def mark():
        if cuda:
            e = torch.cuda.Event(enable_timing=True)
            e.record()
            return e
        return time.perf_counter()

    def ms(a, b):
        return a.elapsed_time(b) if cuda else (b - a) * 1e3

    def step():
        lora = EagerLoRA(model.lora, requires_grad=True)
        lp = model.sequence_logprobs(ids, mask, lora=lora, training=True)
        mid = mark()
        (lp.float() * w).sum().backward()
        lora.accumulate_grads()
        return mid

    for _ in range(2):
        step()
    if cuda:
        torch.cuda.synchronize()
    times = []
    for _ in range(args.iters):
        t0 = mark()
        t1 = step()
        t2 = mark()
        if cuda:
            torch.cuda.synchronize()
        times.append((ms(t0, t1), ms(t1, t2)))
    times.sort(key=lambda t: t[0] + t[1])
    fw, bw = times[len(times) // 2]
    if args.torch_profile and cuda:
        # one more step under torch.profiler: a per-kernel breakdown, not a timing
        from torch.profiler import ProfilerActivity, profile

        with profile(activities=[ProfilerActivity.CUDA]) as prof:
            step()
            torch.cuda.synchronize()
        print(prof.key_averages().table(sort_by="cuda_time_total", row_limit=30, max_name_column_width=70),
              flush=True)
    print(json.dumps({
        "kernel": "hybrid_train_microbatch", "shape": "tiny" if args.tiny else "qwen3.5-9b", "layers": args.layers,
        "rows": B, "seq": S, "padded_first_row": not args.no_pad, "device": str(dev), "fwd_ms": round(fw, 2),
        "bwd_ms": round(bw, 2), "fwd_ms_per_layer": round(fw / args.layers, 3),
        "bwd_ms_per_layer": round(bw / args.layers, 3), "tokens_per_s": round(B * S / ((fw + bw) / 1e3), 1),
    }), flush=True)


def bench_profile(args) -> None:
    """Small, fixed launches of one kernel family for an ncu capture (no timing).

    ``--kernel``: ``gemm`` (training gate/up projection with the SwiGLU
    epilogue, 8192 tokens), ``gemm_mn`` (dgrad against the stored weight,
    MN-major B), ``decode_attn`` (64 rows, 2048 keys, shared 1024-key prompt
    per group of 8), ``flash_fwd`` / ``flash_bwd`` (4 x 3072 tokens, 32/8 heads).
    """
    from graspo_b200.ops._ext import check_errors, ext
    from graspo_b200.ops.gemm import gemm

    k = args.kernel
    runs = []
    if k == "gemm":
        x, w = torch.randn(8192, 4096, device="cuda").bfloat16(), torch.randn(24576, 4096, device="cuda").bfloat16()
        runs.append(lambda: gemm(x, w, epilogue="swiglu"))
    elif k in ("gemm_gu_decode", "gemm_gu_decode_s1"):
        # decode gate/up: 64 tokens, swap layout, SwiGLU epilogue, split-K 3 (or 1)
        splits = 1 if k.endswith("_s1") else 3
        w, x = torch.randn(24576, 4096, device="cuda").bfloat16(), torch.randn(64, 4096, device="cuda").bfloat16()
        out = torch.empty(64, 12288, device="cuda", dtype=torch.bfloat16)
        ws = torch.empty(splits * 64 * 24576, device="cuda")
        ctr = torch.zeros(192, device="cuda", dtype=torch.int32)
        kw = dict(aux=ws, tile_ctr=ctr) if splits > 1 else {}
        runs.append(lambda: gemm(w, x, out, swap=True, epilogue="swiglu", splits=splits, **kw))
    elif k in ("lse", "softmax_grad"):
        # LM head over the full vocabulary: per-tile log-sum-exp partials + target logit (old log-probs,
        # 8192 tokens), or the softmax-grad epilogue of its backward
        T, H, V = 8192, 4096, 151936
        h = torch.randn(T, H, device="cuda").bfloat16()
        head = (torch.randn(V, H, device="cuda") * 0.02).bfloat16()
        tgt = torch.randint(0, V, (T,), device="cuda")
        nblk = -(-V // 256)
        part = torch.empty(T, nblk * 2, device="cuda")
        tl = torch.zeros(T, device="cuda")
        if k == "lse":
            runs.append(lambda: gemm(h, head, torch.empty(0, device="cuda"), epilogue="lse", aux=part, targets=tgt,
                                     tgt_logit=tl, bn=256))
        else:
            lse = torch.full((T,), 12.0, device="cuda")
            g = torch.full((T,), 1e-3, device="cuda")
            runs.append(lambda: gemm(h, head, epilogue="softmax_grad", targets=tgt, row_lse=lse, row_scale=g))
    elif k in ("gemm_push_peer", "tp_reduce"):
        # one process, two GPUs: the training o_proj GEMM at TP=2 (24576 tokens x 4096 x 2048) whose
        # epilogue stores every bf16 tile into this GPU's own slot and into the slot on GPU 1
        # (NVLink), then the rank-order sum of the two slots with the residual
        if not ext().enable_peer_access(0, 1):
            raise SystemExit("GPU 0 cannot reach GPU 1")
        T, H, K = 24576, 4096, 2048
        a = torch.randn(T, K, device="cuda:0").bfloat16()
        w = (torch.randn(H, K, device="cuda:0") * 0.02).bfloat16()
        own = torch.empty(T, H, device="cuda:0", dtype=torch.bfloat16)
        peer = torch.empty(T, H, device="cuda:1", dtype=torch.bfloat16)
        ctr = torch.zeros(2, device="cuda:1", dtype=torch.int64)
        push = {"push_out": torch.tensor([own.data_ptr(), peer.data_ptr()], dtype=torch.int64),
                "push_sig": torch.tensor([0, ctr.data_ptr()], dtype=torch.int64), "push_self": 0, "push_rows": 0}
        if k == "gemm_push_peer":
            runs.append(lambda: gemm(a, w, own, push=dict(push)))
        else:
            from graspo_b200.ops._ext import err_word

            other = torch.randn(T, H, device="cuda:0").bfloat16()
            res = torch.randn(T, H, device="cuda:0").bfloat16()
            out = torch.empty(T, H, device="cuda:0", dtype=torch.bfloat16)
            done = torch.ones(1, device="cuda:0", dtype=torch.int64)  # every arrival already counted
            srcs = torch.tensor([own.data_ptr(), other.data_ptr()], dtype=torch.int64)
            runs.append(lambda: ext().tp_reduce(srcs, done.data_ptr(), 1, res, out, H, err_word(out.device), 0))
    elif k == "gemm_qkv_decode":
        # decode q/k/v projection with its LoRA A rows: 64 tokens, swap layout, split-K 3, fp32 atomics
        w, x = torch.randn(6144 + 64, 4096, device="cuda").bfloat16(), torch.randn(64, 4096, device="cuda").bfloat16()
        ws = torch.zeros(64, 6144 + 64, device="cuda")
        runs.append(lambda: gemm(w, x, ws, swap=True, epilogue="atomic", splits=3))
    elif k == "adamw":
        # clipped AdamW over the flat LoRA buffer of the Qwen3-8B config (r=16, all linears)
        n = 43646976
        p, g = torch.randn(n, device="cuda") * 0.01, torch.randn(n, device="cuda") * 1e-3
        m1, m2 = torch.zeros(n, device="cuda"), torch.zeros(n, device="cuda")
        sumsq, loss = torch.ones(1, device="cuda"), torch.zeros(1, device="cuda")
        skipped = torch.zeros(1, dtype=torch.int32, device="cuda")
        runs.append(lambda: ext().adamw(p, g, m1, m2, 5e-6, 0.9, 0.999, 1e-8, 0.01, 1, sumsq, 1.0, loss, skipped))
    elif k == "sample":
        # Gumbel-max sampling + decode-state update, 64 rows x 151936 vocabulary (top-p 1 and 0.9)
        rows, V = 64, 151936
        logits = torch.randn(rows, V, device="cuda") * 3
        st = dict(next_ids=torch.zeros(rows, dtype=torch.long, device="cuda"),
                  slot=torch.full((rows,), 1023, dtype=torch.long, device="cuda"),
                  pos=torch.zeros(rows, dtype=torch.long, device="cuda"),
                  kv_len=torch.full((rows,), 1024, dtype=torch.int32, device="cuda"),
                  finished=torch.zeros(rows, dtype=torch.uint8, device="cuda"),
                  out=torch.zeros(rows, 4096, dtype=torch.long, device="cuda"))
        for top_p in (1.0, 0.9):
            runs.append(lambda top_p=top_p: ext().sample_append(
                logits, 1.0, top_p, 7, st["next_ids"], st["slot"], st["pos"], st["kv_len"], st["finished"],
                st["out"], 1024, -1, 0, True, None))
    elif k == "gemm_mn":
        dy, w = torch.randn(8192, 24576, device="cuda").bfloat16(), torch.randn(24576, 4096, device="cuda").bfloat16()
        runs.append(lambda: gemm(dy, w, b_mn=True))
    elif k == "decode_attn":
        rows, nq, nkv, D, page, P, ctx, G = 64, 32, 8, 128, 64, 1024, 2048, 8
        n = rows // G
        pp, gp = P // page, (ctx - P) // page
        num_pages = n * pp + rows * gp
        kp = torch.randn(num_pages, nkv, page, D, device="cuda").bfloat16()
        vp = torch.randn_like(kp)
        bt = torch.empty(rows, pp + gp, dtype=torch.int32)
        for r in range(rows):
            bt[r, :pp] = torch.arange((r // G) * pp, (r // G + 1) * pp)
            bt[r, pp:] = torch.arange(n * pp + r * gp, n * pp + (r + 1) * gp)
        bt = bt.cuda()
        q = torch.randn(rows, nq, D, device="cuda").bfloat16()
        start = torch.zeros(rows, device="cuda", dtype=torch.int32)
        ln = torch.full((rows,), ctx, device="cuda", dtype=torch.int32)
        out = torch.empty(rows, nq * D, device="cuda", dtype=torch.bfloat16)
        scratch = torch.zeros(rows * nq * 12 * (D + 2) + rows * nkv, device="cuda")
        runs.append(lambda: ext().paged_decode_attention(q, kp, vp, bt, start, ln, out, 1 / math.sqrt(D), 4, scratch,
                                                         P, G, 2))
    elif k in ("flash_fwd", "flash_bwd", "flash_fwd_tc", "flash_bwd_tc"):
        from graspo_b200.ops._ext import err_word

        B, S, nq, nkv, D = 4, 3072, 32, 8, 128
        T = B * S
        q = torch.randn(T, nq, D, device="cuda").bfloat16()
        kk = torch.randn(T, nkv, D, device="cuda").bfloat16()
        v = torch.randn(T, nkv, D, device="cuda").bfloat16()
        start = torch.zeros(B, device="cuda", dtype=torch.int32)
        end = torch.full((B,), S, device="cuda", dtype=torch.int32)
        o = torch.empty_like(q)
        lse = torch.empty(T, nq, device="cuda")
        ew = err_word(q.device)
        ext().flash_attn_fwd_tc(q, kk, v, o, lse, start, end, B, S, 1 / math.sqrt(D), ew)
        if k in ("flash_fwd", "flash_fwd_tc"):
            runs.append(lambda: ext().flash_attn_fwd_tc(q, kk, v, o, lse, start, end, B, S, 1 / math.sqrt(D), ew))
        else:
            do = torch.randn_like(q)
            dq, dk, dv = torch.empty_like(q), torch.empty_like(kk), torch.empty_like(v)
            runs.append(lambda: ext().flash_attn_bwd_tc(do, q, kk, v, o, lse, dq, dk, dv, start, end, B, S,
                                                        1 / math.sqrt(D), ew))
    else:
        raise SystemExit(f"unknown kernel {k}")
    for _ in range(args.iters):
        for fn in runs:
            fn()
    torch.cuda.synchronize()
    check_errors()
    print(json.dumps({"profile": k, "launches": args.iters * len(runs)}), flush=True)


def main(argv: list[str] | None = None) -> None:
    parser = argparse.ArgumentParser()
    parser.add_argument("what", choices=["gemm", "decode", "dsweep", "attn", "push", "step", "train", "hybrid",
                                         "profile", "all"])
    parser.add_argument("--kernel", default="gemm")
    parser.add_argument("--iters", type=int, default=10)
    parser.add_argument("--tokens", type=int, default=64)
    parser.add_argument("--layers", type=int, default=4)
    parser.add_argument("--prompts", type=int, default=8)
    parser.add_argument("--group", type=int, default=8)
    parser.add_argument("--prompt-len", type=int, default=1024)
    parser.add_argument("--new", type=int, default=64)
    parser.add_argument("--configs", default="gn,gp,en", help="decode-step configs: g/e = graph/eager, n/p = no prefix / shared-prefix attention")
    parser.add_argument("--ckpt", default="/tmp/graspo_b200_bench")
    parser.add_argument("--rows", type=int, default=8)
    parser.add_argument("--seq", type=int, default=3072)
    parser.add_argument("--dropout", type=float, default=0.1)
    parser.add_argument("--tiny", action="store_true", help="hybrid: the small test shape")
    parser.add_argument("--no-pad", action="store_true", help="hybrid: no left-padded row")
    parser.add_argument("--torch-profile", action="store_true", help="hybrid: print a torch.profiler kernel table")
    args = parser.parse_args(argv)
    if args.what in ("gemm", "all"):
        bench_gemm(args)
    if args.what in ("decode", "all"):
        bench_decode(args)
    if args.what == "attn":
        bench_attn(args)
    if args.what == "push":
        bench_push(args)
    if args.what == "dsweep":
        bench_dsweep(args)
    if args.what == "step":
        bench_step(args)
    if args.what == "train":
        bench_train(args)
    if args.what == "hybrid":
        bench_hybrid(args)
    if args.what == "profile":
        bench_profile(args)


if __name__ == "__main__":
    main()
