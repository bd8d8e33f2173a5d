"""GRASPO step throughput: tokens/sec for the Qwen3-8B-shaped LoRA config.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]

One GRASPO step = rollout of B prompts x G completions (prefill + fixed-length
decode), rule-based reward + group advantages, old log-probs, and
``train_batch`` (PPO-clip loss, backward, clipped AdamW on the LoRA
adapters).  Tokens per step = sum over completions of (prompt + generated
tokens).  Both arms run through their framework's own public runtime API
(``generate_groups`` from chat messages, ``sequence_log_probs``,
``train_batch``) on the same synthetic random-init checkpoint and the same
seeded JSON-extraction prompts.

Benchmark mode: random weights never produce a parseable answer, so every
group would be rejected and nothing trained.  The harness therefore scores
each completion with the real reward and adds a seeded per-completion
perturbation (a hash of prompt id and completion index, in [0, 0.5)) before
the group advantages, which makes every group trainable in both arms.

Timing: W untimed steps, then K steps bracketed by a barrier and
``torch.cuda.synchronize()``; CUDA events on the launching stream; the max
over ranks.  ``value`` counts only the device phases (rollout, old
log-probs, training, each including its host<->device copies); ``e2e`` is
the whole step through the public API including chat-template rendering,
tokenization, detokenization and reward scoring on the host.
"""

from __future__ import annotations

import argparse
import hashlib
import json
import os
import sys
import time
from pathlib import Path

import torch

ROOT = Path(__file__).resolve().parent
CKPT_ROOT = Path(os.environ.get("GRASPO_BENCH_DIR", "/tmp/graspo_bench"))
PROMPT_LEN = 1024
MAX_NEW = 2048
GROUP = 8
PROMPTS_PER_REPLICA_PER_TP = 8
BASELINE_VALUE = None  # the reference publishes no throughput number
MIN_WARMUP = 3
# wall-clock budget of one run (set-up + warm-up + timed steps); see StepBudget
TIME_BUDGET_S = 760.0
_T_IMPORT = time.time()


def layout(n: int) -> tuple[int, int]:
    """(tp, dp) for n GPUs: TP=2 x DP=n/2 from 2 GPUs up (config 1 is TP=2 x DP=4 on 8)."""
    if n == 1:
        return 1, 1
    return 2, n // 2


def dist_env() -> tuple[int, int, int]:
    return int(os.environ.get("RANK", 0)), int(os.environ.get("WORLD_SIZE", 1)), int(os.environ.get("LOCAL_RANK", 0))


def ensure_checkpoint(model: str, local_rank: int) -> Path:
    from graspo_b200.utils.synth import QWEN3_8B, TINY, write_qwen3_checkpoint

    dims = QWEN3_8B if model == "qwen3-8b" else TINY
    path = CKPT_ROOT / model
    marker = path / ".complete"
    if local_rank == 0 and not marker.exists():
        write_qwen3_checkpoint(path, dims, seed=1234, device="cuda" if torch.cuda.is_available() else "cpu")
    deadline = time.time() + 1800
    while not marker.exists():
        if time.time() > deadline:
            raise TimeoutError("synthetic checkpoint was not written in time")
        time.sleep(2)
    return path


def perturbation(prompt_id: str, idx: int) -> float:
    digest = hashlib.sha256(f"{prompt_id}:{idx}".encode()).digest()
    return int.from_bytes(digest[:4], "little") / 2**32 * 0.5


def records(total: int) -> list[dict]:
    from graspo_b200.utils.synth import synthetic_json_records

    # ~1500 characters of user text -> truncated to exactly PROMPT_LEN byte tokens
    return synthetic_json_records(total, seed=20261201, pad_words_to=260)


def base_config(args, tp: int, dp: int, model_path: Path, out_dir: Path, n_prompts: int) -> dict:
    return {
        "train_method": "graspo",
        "model": {"model_path": str(model_path), "torch_dtype": "bfloat16", "gradient_checkpointing": True},
        "data": {"train_path": "", "max_prompt_length": args.prompt_len},
        # all seven linears of the dense decoder, named explicitly: the reference's
        # "language_all_linear" preset also lists hybrid-model modules and is
        # rejected for a dense qwen3 checkpoint
        "lora": {"r": 16, "alpha": 32, "dropout": 0.1, "target_modules": [
            "language.self_attn.q_proj", "language.self_attn.k_proj", "language.self_attn.v_proj",
            "language.self_attn.o_proj", "language.mlp.gate_proj", "language.mlp.up_proj",
            "language.mlp.down_proj"]},
        "reward": {},
        "training": {
            "output_dir": str(out_dir), "run_name": "bench", "seed": 42,
            "rollout_group_size": args.group, "optimize_prompt_batch_size": args.group,
            "optimize_iterations_per_step": args.iters, "learning_rate": 5e-6, "weight_decay": 0.01,
            "max_grad_norm": 1.0, "policy_ratio_clip_eps": 0.2, "max_new_tokens": args.max_new,
            "temperature": 1.0, "top_p": 1.0,
        },
        "graspoflow": {
            "tp_size": tp, "pp_size": 1, "forward_batch_size": n_prompts * args.group,
            "use_kv_cache_for_rollout": True, "raw_log_enabled": False, "readable_log_enabled": False,
        },
    }


class PhaseTimer:
    """CUDA-event timing of device phases on the current stream."""

    def __init__(self, cuda: bool) -> None:
        self.cuda = cuda
        self.device_ms = 0.0
        self.total_ms = 0.0
        self.phases: dict[str, float] = {}

    def add(self, name: str, ms: float) -> None:
        self.device_ms += ms
        self.phases[name] = self.phases.get(name, 0.0) + ms

    def event(self):
        if self.cuda:
            e = torch.cuda.Event(enable_timing=True)
            e.record()
            return e
        return time.perf_counter()

    def elapsed(self, a, b) -> float:
        if self.cuda:
            b.synchronize()
            return a.elapsed_time(b)
        return (b - a) * 1e3


class StepBudget:
    """Fits the warm-up and timed steps into a wall-clock budget for the whole run.

    The budget counts from the process start (model set-up included).  Every
    rank takes the slowest rank's step time (a MAX all-reduce), so all ranks
    agree on the number of steps.  At least ``MIN_WARMUP`` warm-up steps and
    one timed step always run; steps are never shortened, only counted.
    """

    def __init__(self, budget_s: float, cuda: bool) -> None:
        self.budget_s = float(budget_s)
        self.cuda = cuda
        self.last_step_s = 0.0

    @staticmethod
    def elapsed() -> float:
        try:
            import psutil

            return time.time() - psutil.Process().create_time()
        except Exception:  # noqa: BLE001 - psutil missing: count from import
            return time.time() - _T_IMPORT

    def _agree(self, values: list[float]) -> list[float]:
        import torch.distributed as dist

        if not (dist.is_available() and dist.is_initialized()):
            return values
        t = torch.tensor(values, dtype=torch.float64, device="cuda" if self.cuda else "cpu")
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        return [float(v) for v in t.tolist()]

    def step_done(self, seconds: float) -> None:
        self.last_step_s, self._elapsed = self._agree([seconds, self.elapsed()])

    def room_for(self, n_steps: int) -> bool:
        if self.budget_s <= 0:
            return True
        return self._elapsed + n_steps * self.last_step_s <= self.budget_s

    def timed_steps(self, requested: int) -> int:
        if self.budget_s <= 0 or self.last_step_s <= 0:
            return requested
        fit = int((self.budget_s - self._elapsed) // self.last_step_s)
        return max(1, min(requested, fit))


def grpo_step(api, samples, reward, *, group: int, max_new: int, prompt_len: int, iters: int, timer: PhaseTimer,
              reward_cls_adv, experience_cls, counters: dict) -> int:
    """One GRASPO step through ``api`` (this framework's or the reference's runtime)."""
    t_start = timer.event()
    a = timer.event()
    gens = api.generate_groups(
        message_batches=[s.messages for s in samples], tool_batches=[s.tools for s in samples],
        rollout_group_size=group, max_new_tokens=max_new, max_prompt_length=prompt_len,
        temperature=1.0, top_p=1.0, chat_template_kwargs={},
    )
    b = timer.event()
    timer.add("rollout", timer.elapsed(a, b))
    meta = gens[0].metadata or {}
    n = len(gens)
    timer.phases["prefill_s"] = timer.phases.get("prefill_s", 0.0) + float(meta.get("prefill_sec", 0.0)) * n
    timer.phases["decode_s"] = timer.phases.get("decode_s", 0.0) + float(meta.get("decode_sec", 0.0)) * n
    tokens = 0
    experiences = []
    for sample, gen in zip(samples, gens, strict=True):
        seqs = gen.sequences
        counters["d2h"] += seqs.numel() * seqs.element_size()
        rewards = []
        for j, text in enumerate(gen.completions):
            parsed = api.parse_completion(text, sample)
            res = reward.score_parsed(parsed, sample.targets, is_tool_call=sample.expects_tool_calls)
            rewards.append(float(res.reward) + perturbation(str(sample.metadata.get("id")), j))
        adv = reward_cls_adv(rewards)
        a = timer.event()
        old = api.sequence_log_probs(gen.sequences, gen.attention_mask)
        old = old.detach().float().cpu()
        b = timer.event()
        timer.add("old_logprob", timer.elapsed(a, b))
        counters["h2d"] += seqs.numel() * seqs.element_size() + gen.attention_mask.numel()
        counters["d2h"] += old.numel() * 4
        prompt_len_tok = int(gen.prompt_len)
        for j in range(seqs.shape[0]):
            n_tok = int(seqs.shape[1])
            tokens += n_tok
            experiences.append(experience_cls(
                sequences=seqs[j].cpu(), old_log_probs=old[j], advantages=torch.full((n_tok - 1,), adv[j]),
                attention_mask=gen.attention_mask[j].cpu(), action_mask=gen.action_mask[j].cpu(),
                rewards=torch.tensor(rewards[j]), metadata={"prompt_len": prompt_len_tok},
            ))
    a = timer.event()
    metrics = api.train_batch(experiences, policy_ratio_clip_eps=0.2, optimize_iterations_per_step=iters,
                              max_grad_norm=1.0)
    b = timer.event()
    timer.add("train", timer.elapsed(a, b))
    for e in experiences:
        counters["h2d"] += (e.sequences.numel() * 8 + e.old_log_probs.numel() * 4 + e.advantages.numel() * 4
                            + e.attention_mask.numel() + e.action_mask.numel()) * iters
    counters["d2h"] += 4 * max(1, int(metrics.get("optimizer_steps") or 1))
    t_end = timer.event()
    timer.total_ms += timer.elapsed(t_start, t_end)
    return tokens


def run(args) -> dict:
    rank, world, local_rank = dist_env()
    if torch.cuda.is_available():
        torch.cuda.set_device(local_rank)
    tp, dp = layout(world) if args.impl == "ours" else (world, 1)
    if args.tp and args.impl == "ours":
        if world % args.tp:
            raise SystemExit(f"--tp {args.tp} does not divide {world} GPUs")
        tp, dp = args.tp, world // args.tp
    model_path = ensure_checkpoint(args.model, local_rank)
    per_replica = PROMPTS_PER_REPLICA_PER_TP * tp if args.prompts is None else args.prompts
    n_total = per_replica * (dp if args.impl == "ours" else 1)
    all_records = records(n_total * (max(args.warmup, MIN_WARMUP) + args.steps))
    out_dir = CKPT_ROOT / f"run_{args.impl}_{world}"
    # the runtimes append per-rank JSONL under <output_dir>/logs (normally created
    # by the trainer's logging setup, which the harness does not run)
    (out_dir / "logs").mkdir(parents=True, exist_ok=True)

    if args.impl == "ours":
        sys.path.insert(0, str(ROOT))
        from graspo_b200.core.buffer import Experience
        from graspo_b200.core.data import sample_from_record
        from graspo_b200.core.decisions import group_advantages
        from graspo_b200.core.reward import GraspoReward
        from graspo_b200.core.schema import GraspoConfig
        from graspo_b200.engine.runtime import GraspoFlowRuntime
        from graspo_b200.ops._ext import launches

        cfg_dict = base_config(args, tp, dp, model_path, out_dir, per_replica)
        cfg_dict["graspoflow"].update({"dp_size": dp, "benchmark_ignore_eos": True, "advantage_eps": 1e-8,
                                       "pg_timeout_sec": 300.0})
        cfg = GraspoConfig.from_dict(cfg_dict)
        api = GraspoFlowRuntime.from_config(cfg)
        api.setup()
        dp_rank = api.ps.dp_rank
        reward = GraspoReward(cfg.reward)
        adv_fn = lambda r: group_advantages(r, eps=cfg.graspoflow.advantage_eps)  # noqa: E731
    else:
        ref = ROOT / "baseline" / "_ref"
        if not (ref / "graspo").exists():
            return {"impl": "reference", "unavailable": "reference not installed in baseline/_ref"}
        sys.path.insert(0, str(ref))
        from graspo.backends.graspoflow.runtime import GraspoFlowRuntime  # type: ignore
        from graspo.core.buffer import Experience  # type: ignore
        from graspo.core.data import sample_from_record  # type: ignore
        from graspo.core.graspo_parity import group_advantages  # type: ignore
        from graspo.core.reward import GraspoReward  # type: ignore
        from graspo.core.schema import GraspoConfig  # type: ignore

        cfg_dict = base_config(args, tp, 1, model_path, out_dir, per_replica)
        cfg = GraspoConfig.from_dict(cfg_dict)  # default adapter: the reference's stock path
        api = GraspoFlowRuntime.from_config(cfg)
        api.setup()
        dp_rank = 0
        reward = GraspoReward(cfg.reward)
        adv_fn = lambda r: group_advantages(r)  # noqa: E731
        launches = None

    import torch.distributed as dist

    def step_samples(step: int) -> list:
        base = step * n_total + dp_rank * per_replica
        return [sample_from_record(r) for r in all_records[base : base + per_replica]]

    cuda = torch.cuda.is_available()
    counters = {"h2d": 0, "d2h": 0}
    kw = dict(group=args.group, max_new=args.max_new, prompt_len=args.prompt_len, iters=args.iters,
              reward_cls_adv=adv_fn, experience_cls=Experience)
    budget = StepBudget(args.time_budget, cuda)
    warm_done = 0
    while warm_done < args.warmup:
        wt = PhaseTimer(cuda)
        t0 = time.monotonic()
        grpo_step(api, step_samples(warm_done), reward, timer=wt, counters={"h2d": 0, "d2h": 0}, **kw)
        warm_done += 1
        if rank == 0:
            phases = {k: round(v / 1e3 if not k.endswith("_s") else v, 2) for k, v in wt.phases.items()}
            print(f"[bench] warm-up step {warm_done}/{args.warmup}: {phases}", file=sys.stderr, flush=True)
        budget.step_done(time.monotonic() - t0)
        if warm_done >= MIN_WARMUP and warm_done < args.warmup and not budget.room_for(2):
            # one more warm-up and one timed step would not fit: stop warming up
            break
    steps = budget.timed_steps(args.steps)
    if rank == 0 and (steps != args.steps or warm_done != args.warmup):
        print(f"[bench] time budget {args.time_budget:.0f} s: {warm_done} warm-up and {steps} timed steps "
              f"(requested {args.warmup} and {args.steps})", file=sys.stderr, flush=True)

    from graspo_b200.bench.clocks import ClockSampler

    if dist.is_available() and dist.is_initialized():
        dist.barrier()
    if cuda:
        torch.cuda.synchronize()
    if launches is not None:
        launches.reset()
    timer = PhaseTimer(cuda)
    tokens = 0
    with ClockSampler(gpu_index=None) as clocks:
        for k in range(steps):
            tokens += grpo_step(api, step_samples(warm_done + k), reward, timer=timer, counters=counters, **kw)
        if cuda:
            torch.cuda.synchronize()
    if dist.is_available() and dist.is_initialized():
        dist.barrier()
    gpu_launches = launches.reset() if launches is not None else 0
    if rank == 0:
        phases = {k: round(v / 1e3 if not k.endswith("_s") else v, 2) for k, v in timer.phases.items()}
        print(f"[bench] timed phases (s): {phases}", file=sys.stderr, flush=True)
    stats = torch.tensor([timer.device_ms, timer.total_ms, float(tokens), float(gpu_launches)],
                         dtype=torch.float64, device="cuda" if cuda else "cpu")
    if dist.is_available() and dist.is_initialized():
        maxes = stats.clone()
        dist.all_reduce(maxes, op=dist.ReduceOp.MAX)
        sums = stats.clone()
        dist.all_reduce(sums, op=dist.ReduceOp.SUM)
    else:
        maxes = sums = stats
    device_ms, total_ms = float(maxes[0]), float(maxes[1])
    # each DP replica generates its own prompts; TP ranks of a replica share them
    job_tokens = float(sums[2]) / (tp if args.impl == "ours" else world)
    value = job_tokens / (device_ms / 1e3)
    e2e = job_tokens / (total_ms / 1e3)
    result = {
        "metric": "GRASPO step tokens/sec/box (rollout+train), Qwen3-8B LoRA",
        "value": round(value, 2),
        "unit": "tokens/s",
        "n_gpus": world,
        "steps": steps,
        "warmup": warm_done,
        "requested_steps": args.steps,
        "requested_warmup": args.warmup,
        "time_budget_s": args.time_budget,
        "ms_per_step": round(device_ms / steps, 2),
        "higher_is_better": True,
        "scaling": "weak",
        "vs_baseline": None if BASELINE_VALUE is None else round(value / BASELINE_VALUE, 4),
        "dtype": "bf16",
        "data": "synthetic (seeded JSON-extraction prompts, random-init N(0,0.02) Qwen3-8B-shaped weights)",
        "config": {
            "model": args.model, "global_batch": n_total * args.group, "seq_len": args.prompt_len + args.max_new,
            "prompt_len": args.prompt_len, "max_new_tokens": args.max_new, "group_size": args.group,
            "prompts": n_total, "optimize_iterations_per_step": args.iters, "lora_r": 16,
            "lora_targets": "all linear", "parallelism": f"tp{tp}" + (f"xdp{dp}" if dp > 1 else ""),
            "l2": "inputs larger than L2 (weights 16 GB, KV cache > 10 GB per step)",
            "fixed_length_decode": args.impl == "ours",
        },
        "e2e": {"value": round(e2e, 2), "unit": "tokens/s", "h2d_bytes_per_step": counters["h2d"] // max(1, steps),
                "d2h_bytes_per_step": counters["d2h"] // max(1, steps)},
        "gpu_launches": int(float(maxes[3])),
        "clocks": clocks.summary() if rank == 0 else None,
    }
    if args.impl == "reference":
        result["impl"] = "reference"
    return result


def main() -> None:
    p = argparse.ArgumentParser()
    p.add_argument("--gpus", type=int, default=1)
    p.add_argument("--steps", type=int, default=1)
    p.add_argument("--warmup", type=int, default=3)
    p.add_argument("--impl", choices=["ours", "reference"], default="ours")
    p.add_argument("--model", default="qwen3-8b", choices=["qwen3-8b", "tiny"])
    p.add_argument("--prompts", type=int, default=None, help="prompts per data-parallel replica")
    p.add_argument("--group", type=int, default=GROUP)
    p.add_argument("--prompt-len", type=int, default=PROMPT_LEN)
    p.add_argument("--max-new", type=int, default=MAX_NEW)
    p.add_argument("--iters", type=int, default=1, help="optimize_iterations_per_step")
    p.add_argument("--tp", type=int, default=0,
                   help="tensor-parallel size of this framework's arm (default: 1 on one GPU, else 2; DP = N / TP)")
    p.add_argument("--time-budget", type=float, default=TIME_BUDGET_S,
                   help="wall-clock seconds for the whole run; fewer timed steps (>= 1) run when the requested "
                        "ones would not fit, and warm-up stops early (after at least 3); 0 disables")
    args = p.parse_args()
    if args.warmup < MIN_WARMUP:
        print(f"[bench] warm-up raised to {MIN_WARMUP} steps", file=sys.stderr)
        args.warmup = MIN_WARMUP
    rank, world, _ = dist_env()
    if args.gpus != world:
        print(f"[bench] --gpus {args.gpus} but WORLD_SIZE={world}; using WORLD_SIZE", file=sys.stderr)
    try:
        result = run(args)
    except Exception as exc:  # noqa: BLE001 - the reference arm reports unavailability as a line
        if args.impl == "reference":
            result = {"impl": "reference", "unavailable": f"{type(exc).__name__}: {str(exc)[:200]}"}
        else:
            raise
    if rank == 0:
        print(json.dumps(result), flush=True)
    import torch.distributed as dist

    if dist.is_available() and dist.is_initialized():
        dist.destroy_process_group()


if __name__ == "__main__":
    main()
