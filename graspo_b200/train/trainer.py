"""The GRASPO training loop (reference: trainer/trainer.py, rollout.py, optimize.py).

Per epoch the samples are shuffled with ``seed + epoch`` and consumed in
queues of ``optimize_prompt_batch_size`` prompts (per data-parallel replica:
replica r takes the r-th slice of each global queue).  A queue is rolled out
(G completions per prompt), scored, and every group is classified; RETRY
groups are rolled out again (up to ``rollout_max_retries``).  Trainable
groups get old log-probs and group-normalised advantages and enter the
replay buffer; when every replica holds at least B x G experiences an
optimize step runs (all replicas train on the same number of experiences so
their collectives line up).  Checkpoints: ``step_N`` every ``save_steps``,
``epoch_N`` at epoch end (after a forced flush of the replay buffer),
``final`` at the end or when ``max_steps`` is reached.

Host-side fault injection (tests, never a GPU fault): ``GRASPO_FAULT`` =
``<phase>:<count>`` raises ``InjectedFault`` the ``count``-th time ``phase``
(``rollout``, ``reward``, ``optimize``, ``checkpoint``) is entered, and
``GRASPO_FAULT_RANK`` restricts it to one rank.
"""

from __future__ import annotations

import json
import logging
import os
import random
import sys
import time
from collections import deque
from dataclasses import asdict, dataclass, field
from datetime import datetime
from pathlib import Path
from typing import Any

import torch

from graspo_b200.core.buffer import Experience, ReplayBuffer
from graspo_b200.core.completion import raw_parsed_completion
from graspo_b200.core.data import load_jsonl
from graspo_b200.core.decisions import classify_group, group_advantages, has_reward_variance, lower_median
from graspo_b200.core.logging import setup_logging
from graspo_b200.core.reward import GraspoReward
from graspo_b200.core.schema import GraspoConfig
from graspo_b200.engine.runtime import GraspoFlowRuntime, validate_graspoflow_runtime_config
from graspo_b200.train.logger import RolloutLogger, append_event
from graspo_b200.train.summary import (
    compact_batch_summary,
    compact_decisions,
    compact_optimize_metrics,
    compact_timing_summary,
    monitor_group,
    reward_batch_summary,
    reward_window_summary,
    round_timing_details,
    scalar_generation_timing,
    training_health,
)

log = logging.getLogger("graspo.trainer")


class InjectedFault(RuntimeError):
    """Raised by the host-side fault injector (``GRASPO_FAULT``)."""


class FaultInjector:
    def __init__(self, rank: int = 0) -> None:
        spec = os.environ.get("GRASPO_FAULT", "")
        only = os.environ.get("GRASPO_FAULT_RANK")
        self.phase, self.at = None, 0
        if spec and (only is None or int(only) == rank):
            phase, _, count = spec.partition(":")
            self.phase, self.at = phase, int(count or 1)
        self.seen: dict[str, int] = {}

    def hit(self, phase: str) -> None:
        self.seen[phase] = self.seen.get(phase, 0) + 1
        if phase == self.phase and self.seen[phase] == self.at:
            raise InjectedFault(f"injected fault in {phase} (occurrence {self.at})")


@dataclass
class TrainStats:
    total_groups: int = 0
    perfect_skipped: int = 0
    retries: int = 0
    invalid: int = 0
    invalid_no_preference_gap: int = 0
    trainable: int = 0
    trainable_max_correct: int = 0
    trainable_not_correct: int = 0
    optimized_steps: int = 0


@dataclass
class EpochStats:
    epoch: int = 0
    samples_seen: int = 0
    attempt_groups: int = 0
    completion_count: int = 0
    perfect_skipped: int = 0
    retries: int = 0
    invalid: int = 0
    invalid_no_preference_gap: int = 0
    trainable: int = 0
    trainable_max_correct: int = 0
    trainable_not_correct: int = 0
    reward_mean_sum: float = 0.0
    content_mean_sum: float = 0.0
    best_reward: float = 0.0


@dataclass
class _Queued:
    sample: Any
    retry_count: int = 0
    attempts: list[dict[str, Any]] = field(default_factory=list)


def _timestamp() -> str:
    return datetime.now().astimezone().isoformat(timespec="seconds")


def reward_detail(result) -> dict[str, Any]:
    extracted = dict(result.extracted)
    valid = None
    answer = extracted.get("answer")
    if isinstance(answer, str) and answer.strip():
        try:
            json.loads(answer.strip())
            valid = True
        except (TypeError, ValueError):
            valid = False
    return {
        "raw_score": float(result.raw_score), "max_score": float(result.max_score), "extracted": extracted,
        "parsed_tool_calls": extracted.get("tool_calls"), "parser": extracted.get("parser"),
        "parse_errors": extracted.get("parse_errors"), "extra_text": extracted.get("extra_text"),
        "matched_target_index": result.matched_target_index, "matched_target_id": result.matched_target_id,
        "target_scores": result.target_scores, "useless_text_length": len(result.useless_text),
        "valid_extracted_json": valid,
    }


def group_stats(rewards: list[float]) -> dict[str, Any]:
    if not rewards:
        return {"count": 0, "min": 0.0, "median": 0.0, "max": 0.0, "mean": 0.0, "range": 0.0}
    return {"count": len(rewards), "min": min(rewards), "median": lower_median(rewards), "max": max(rewards),
            "mean": sum(rewards) / len(rewards), "range": max(rewards) - min(rewards)}


class GraspoTrainer:
    def __init__(self, config: GraspoConfig, runtime=None, selection: Any | None = None) -> None:
        self.config = config
        self.runtime = runtime or GraspoFlowRuntime.from_config(config)
        self.selection = selection
        self.reward = GraspoReward(config.reward)
        self.replay_buffer = ReplayBuffer()
        self.stats = TrainStats()
        self.epoch_stats = EpochStats()
        self.global_step = 0
        self.sample_index = 0
        self.total_samples = 0
        self.started_at = time.monotonic()
        self.recent_groups: deque[dict[str, Any]] = deque(maxlen=50)
        self.pending_attempts: list[dict[str, Any]] = []
        self.pending_timings: list[dict[str, Any]] = []
        self.resume_info: dict[str, Any] | None = None
        flow = config.graspoflow
        self.logger = RolloutLogger(config.training.output_dir, readable_enabled=flow.readable_log_enabled,
                                    raw_enabled=flow.raw_log_enabled)
        self.faults = FaultInjector()

    # ------------------------------------------------------------ plumbing
    @property
    def ps(self):
        return getattr(self.runtime, "ps", None)

    def _now(self) -> float:
        """Phase clock; with ``graspoflow.synchronize_cuda_timing`` the device is
        synchronised first so each phase owns its GPU work (reference:
        transformer_adapter.py:685-691)."""
        if self.config.graspoflow.synchronize_cuda_timing and torch.cuda.is_available():
            torch.cuda.synchronize()
        return time.monotonic()

    def _is_primary(self) -> bool:
        fn = getattr(self.runtime, "is_primary", None)
        return bool(fn()) if callable(fn) else True

    def _emit(self, payload: dict[str, Any]) -> None:
        if self._is_primary():
            print(json.dumps(payload, ensure_ascii=False, default=str), flush=True)
            append_event(self.config.training.output_dir, payload)

    def _dp(self) -> tuple[int, int]:
        ps = self.ps
        return (ps.dp_rank, ps.dp_size) if ps is not None else (0, 1)

    def _all_min(self, value: int) -> int:
        ps = self.ps
        if ps is None or not ps.distributed:
            return int(value)
        import torch.distributed as dist

        t = torch.tensor([int(value)], dtype=torch.long, device=ps.device)
        dist.all_reduce(t, op=dist.ReduceOp.MIN)
        return int(t.item())

    # ------------------------------------------------------------ main loop
    def train(self) -> None:
        validate_graspoflow_runtime_config(self.config)
        self.runtime.validate()
        self.runtime.setup()
        self.faults = FaultInjector(int(getattr(self.runtime, "rank", 0)))
        setup_logging(self.config.training.output_dir, rank=int(getattr(self.runtime, "rank", 0)))
        cfg, tr = self.config, self.config.training
        self._emit({
            "timestamp": _timestamp(), "event": "backend_selected", "backend": "graspoflow",
            "reason": getattr(self.selection, "reason", "configured"),
            "dependency_boundary": "PyTorch + sm_100a kernels + NCCL; no NeMo/vLLM/Ray/DeepSpeed/FSDP/DDP/Accelerate",
            "model_path": cfg.model.model_path, "train_path": cfg.data.train_path,
            "completion_parser": "qwen_tool_call", "tp_size": cfg.graspoflow.tp_size,
        })
        samples = load_jsonl(cfg.data.train_path)
        self.total_samples = len(samples)
        out = Path(tr.output_dir)
        out.mkdir(parents=True, exist_ok=True)
        self._resume_if_requested()
        if self.resume_info is None and self._is_primary():
            import yaml

            (out / "config.yaml").write_text(yaml.dump(cfg.model_dump(), allow_unicode=True, sort_keys=False),
                                             encoding="utf-8")
        self._emit({
            "timestamp": _timestamp(), "event": "run_start", "backend": "graspoflow",
            "samples_total": self.total_samples, "resume": self.resume_info,
            "config": {
                "rollout_group_size": tr.rollout_group_size, "optimize_prompt_batch_size": tr.optimize_prompt_batch_size,
                "optimize_iterations_per_step": tr.optimize_iterations_per_step,
                "replay_buffer_optimize_threshold": tr.replay_buffer_optimize_threshold,
                "rollout_max_retries": tr.rollout_max_retries, "max_epochs": tr.max_epochs, "max_steps": tr.max_steps,
                "max_new_tokens": tr.max_new_tokens, "save_steps": tr.save_steps,
                "lora_target_modules": list(cfg.lora.target_modules or [cfg.lora.target_preset]),
                "forward_batch_size": cfg.graspoflow.forward_batch_size, "dp_size": self._dp()[1],
            },
        })
        dp_rank, dp_size = self._dp()
        try:
            start_epoch = self.epoch_stats.epoch
            if self.total_samples and self.epoch_stats.samples_seen >= self.total_samples:
                start_epoch += 1
            for epoch in range(start_epoch, tr.max_epochs):
                if epoch != start_epoch or self.epoch_stats.samples_seen == 0:
                    self.epoch_stats = EpochStats(epoch=epoch)
                order = list(samples)
                random.Random(int(tr.seed) + epoch).shuffle(order)
                offset = self.epoch_stats.samples_seen if epoch == start_epoch else 0
                pending = order[offset:]
                q = max(1, int(tr.optimize_prompt_batch_size))
                for start in range(0, len(pending), q * dp_size):
                    chunk = pending[start : start + q * dp_size]
                    mine = chunk[dp_rank * q : (dp_rank + 1) * q]
                    if self._run_queue(mine, epoch=epoch, global_count=len(chunk)):
                        self._save_checkpoint(out / "final", epoch=epoch)
                        return
                self._emit({"timestamp": _timestamp(), "event": "epoch_summary",
                            "elapsed_sec": round(time.monotonic() - self.started_at, 3),
                            "epoch": self._epoch_summary(), "run": self._run_summary()})
                if tr.save_checkpoint_every_epoch:
                    self._maybe_optimize(epoch=epoch, force=True)
                    self._save_checkpoint(out / f"epoch_{epoch}", epoch=epoch)
            self._maybe_optimize(epoch=tr.max_epochs - 1, force=True)
            self._save_checkpoint(out / "final", epoch=tr.max_epochs - 1)
        finally:
            if sys.exc_info()[0] is not None:
                # failing: do not wait at a checkpoint barrier the other ranks may never reach
                abandon = getattr(self.runtime, "abandon_checkpoints", None)
                if callable(abandon):
                    try:
                        abandon()
                    except RuntimeError:
                        pass
            self.runtime.close()

    # ------------------------------------------------------------ rollout
    def _run_queue(self, samples: list[Any], *, epoch: int, global_count: int) -> bool:
        active = [_Queued(s) for s in samples]
        finished: list[_Queued] = []
        max_attempts = self.config.training.rollout_max_retries + 1
        while True:
            # Rollout collectives stay inside a replica's TP group; the only
            # world-wide call is the "everyone done?" check below, which every
            # rank makes once per iteration, so replicas that finish early keep
            # looping (without work) until the last replica is done.
            records = self._rollout_attempt(active, epoch=epoch) if active else []
            nxt = []
            for st, rec in zip(active, records, strict=True):
                st.attempts.append(rec)
                if rec["decision"].should_retry:
                    st.retry_count += 1
                    if st.retry_count >= max_attempts:
                        raise RuntimeError("GRASPO retry state exceeded configured max attempts")
                    nxt.append(st)
                else:
                    finished.append(st)
            active = nxt
            if self._all_min(1 if not active else 0) == 1:
                break
        stop = False
        for st in finished:
            stop = self._finalize(st, epoch=epoch) or stop
        # replicas may have counted different numbers of samples; advance by the global chunk
        self.epoch_stats.samples_seen += global_count - len(finished)
        if self._maybe_optimize(epoch=epoch):
            stop = stop or 0 < self.config.training.max_steps <= self.global_step
        return stop

    def _rollout_attempt(self, active: list[_Queued], *, epoch: int) -> list[dict[str, Any]]:
        tr = self.config.training
        self.faults.hit("rollout")
        t0 = self._now()
        gens = self.runtime.generate_sample_groups(
            samples=[s.sample for s in active], rollout_group_size=tr.rollout_group_size,
            max_new_tokens=tr.max_new_tokens, max_prompt_length=self.config.data.max_prompt_length,
            temperature=tr.temperature, top_p=tr.top_p, chat_template_kwargs=self.config.model.chat_template_kwargs,
        )
        if len(gens) != len(active):
            raise RuntimeError(f"generate_sample_groups returned {len(gens)} groups for {len(active)} samples")
        per_prompt = (self._now() - t0) / max(1, len(gens))
        records = []
        self.faults.hit("reward")
        for st, gen in zip(active, gens, strict=True):
            t1 = self._now()
            parse = getattr(self.runtime, "parse_completion", None)
            parsed = [parse(t, st.sample) if callable(parse) else raw_parsed_completion(t) for t in gen.completions]
            results = [self.reward.score_parsed(p, st.sample.targets, is_tool_call=st.sample.expects_tool_calls)
                       for p in parsed]
            reward_sec = self._now() - t1
            rewards = [float(r.reward) for r in results]
            content = [float(r.content_score) for r in results]
            best = max(range(len(rewards)), key=lambda i: rewards[i])
            bp = parsed[best]
            bad = bool(bp.parse_errors)
            if st.sample.expects_tool_calls and st.sample.targets and not bad:
                calls = (st.sample.targets[0].get("output") or {}).get("tool_calls")
                expected = len(calls) if isinstance(calls, list) else 0
                bad = expected > 0 and len(bp.tool_calls) != expected
            decision = classify_group(
                rewards, content, retry_count=st.retry_count, rollout_max_retries=tr.rollout_max_retries,
                perfect_skip_reward_threshold=tr.perfect_skip_reward_threshold,
                best_completion_has_parse_error=bad, reject_unparseable_groups=tr.reject_unparseable_groups,
            )
            self.stats.total_groups += 1
            if decision.should_retry:
                self.stats.retries += 1
            gen_tokens = [int(x) for x in gen.action_mask.sum(dim=1).tolist()]
            readable = {
                "event": "graspo_group", "backend": "graspoflow", "epoch": epoch, "step": self.global_step,
                "sample_index": self.sample_index, "messages": st.sample.messages, "tools": st.sample.tools,
                "prompt_preview": st.sample.prompt_preview, "targets": st.sample.targets,
                "metadata": {k: v for k, v in st.sample.metadata.items() if k not in ("image", "images", "video", "videos")},
                "completions": gen.completions, "parsed_completions": [p.to_dict() for p in parsed],
                "rewards": rewards, "content_scores": content, "all_right": [bool(r.all_right) for r in results],
                "reward_details": [reward_detail(r) for r in results], "generated_tokens": gen_tokens,
                "decision": decision.decision.value, "attempt_index": st.retry_count + 1,
                "max_attempts": tr.rollout_max_retries + 1, "retry_count": st.retry_count,
                "group_stats": group_stats(rewards), "reward_max_median_gap": decision.reward_max_median_gap,
                "generation_metadata": {k: v for k, v in (gen.metadata or {}).items() if not str(k).startswith("_")},
            }
            if decision.decision.value == "invalid_no_preference_gap":
                readable["invalid_reason"] = "no_preference_gap"
            if self._is_primary():
                self.logger.write_readable(readable)
            timing = {
                "rollout_sec": per_prompt, "reward_cpu_sec": reward_sec, "decision_sec": 0.0,
                "old_logprob_sec": 0.0, "replay_append_sec": 0.0, "decision": decision.decision.value,
                "retry_count": st.retry_count, "completion_count": len(gen.completions),
                "sequence_len": int(gen.sequences.shape[1]), "generated_tokens_max": max(gen_tokens, default=0),
                **scalar_generation_timing(gen.metadata or {}),
            }
            records.append({"generation": gen, "rewards": rewards, "content": content, "decision": decision,
                            "readable": readable, "timing": timing})
        return records

    def _finalize(self, st: _Queued, *, epoch: int) -> bool:
        rec = st.attempts[-1]
        gen, rewards, decision, readable, timing = (rec["generation"], rec["rewards"], rec["decision"],
                                                    rec["readable"], rec["timing"])
        trainable = decision.should_train and has_reward_variance(rewards)
        if not trainable:
            kind = decision.decision.value
            if kind == "perfect_skip":
                self.stats.perfect_skipped += 1
            elif kind == "invalid_no_preference_gap":
                self.stats.invalid_no_preference_gap += 1
            else:
                self.stats.invalid += 1
                self.logger.write_error({"event": "group_decision", "decision": "invalid",
                                         "reason": kind if decision.should_train is False else "no_reward_variance",
                                         "sample_index": self.sample_index, "global_step": self.global_step,
                                         "prompt_preview": readable.get("prompt_preview"),
                                         "group_stats": readable.get("group_stats")})
        else:
            t0 = self._now()
            old = self.runtime.sequence_log_probs(gen.sequences, gen.attention_mask, metadata=gen.metadata)
            old = old.detach().float().cpu()
            timing["old_logprob_sec"] = self._now() - t0
            adv = group_advantages(rewards, eps=self.config.graspoflow.advantage_eps)
            items = []
            for j in range(len(rewards)):
                items.append(Experience(
                    sequences=gen.sequences[j].detach().cpu(), old_log_probs=old[j],
                    advantages=torch.full_like(old[j], float(adv[j])),
                    attention_mask=gen.attention_mask[j].detach().cpu(), action_mask=gen.action_mask[j].detach().cpu(),
                    rewards=torch.tensor(rewards[j]),
                    # image references travel with the experience so training re-encodes them
                    metadata=({"_media": gen.metadata["_media_rows"][j]}
                              if (gen.metadata or {}).get("_media_rows") else None),
                ))
            self.replay_buffer.append_many(items)
            self.stats.trainable += 1
            if decision.decision.value == "trainable_max_correct":
                self.stats.trainable_max_correct += 1
            else:
                self.stats.trainable_not_correct += 1
        if self._is_primary():
            self.logger.write_raw({**readable, "raw": {"sequences": gen.sequences, "attention_mask": gen.attention_mask,
                                                       "action_mask": gen.action_mask, "prompt_len": gen.prompt_len}})
        for r in st.attempts:
            self.recent_groups.append(monitor_group(r["readable"]))
            self.pending_attempts.append(r["readable"])
            self._record_epoch_attempt(r["readable"])
            self.pending_timings.append(r["timing"])
            if self._is_primary():
                self.logger.write_timing_event(self._timing_event("rollout_attempt", r["timing"], epoch))
        self.epoch_stats.samples_seen += 1
        self.sample_index += 1
        return False

    def _record_epoch_attempt(self, payload: dict[str, Any]) -> None:
        es = self.epoch_stats
        rewards = [float(v) for v in payload.get("rewards", [])]
        content = [float(v) for v in payload.get("content_scores", [])]
        es.attempt_groups += 1
        es.completion_count += len(rewards)
        if rewards:
            es.reward_mean_sum += sum(rewards) / len(rewards)
            es.best_reward = max(es.best_reward, max(rewards))
        if content:
            es.content_mean_sum += sum(content) / len(content)
        d = str(payload.get("decision"))
        field_name = {"retry": "retries", "perfect_skip": "perfect_skipped", "invalid": "invalid",
                      "invalid_no_preference_gap": "invalid_no_preference_gap"}.get(d)
        if field_name:
            setattr(es, field_name, getattr(es, field_name) + 1)
        elif d in ("trainable_max_correct", "trainable_not_correct"):
            es.trainable += 1
            key = "trainable_max_correct" if d == "trainable_max_correct" else "trainable_not_correct"
            setattr(es, key, getattr(es, key) + 1)

    def _timing_event(self, phase: str, details: dict[str, Any], epoch: int) -> dict[str, Any]:
        return {"timestamp": _timestamp(), "elapsed_sec": round(time.monotonic() - self.started_at, 6),
                "phase": phase, "duration_sec": round(float(details.get("attempt_total_sec") or sum(
                    float(details.get(k) or 0) for k in ("rollout_sec", "reward_cpu_sec", "old_logprob_sec"))), 6),
                "step": self.global_step, "epoch": epoch, "sample_index": self.sample_index,
                "rank": int(getattr(self.runtime, "rank", 0)), "details": round_timing_details(details)}

    # ------------------------------------------------------------ optimize
    def _maybe_optimize(self, *, epoch: int, force: bool = False) -> bool:
        tr = self.config.training
        threshold = tr.replay_buffer_optimize_threshold
        usable = self._all_min(len(self.replay_buffer) if force else (threshold if len(self.replay_buffer) >= threshold else 0))
        if usable <= 0:
            return False
        self.faults.hit("optimize")
        data = self.replay_buffer.take(usable)
        t0 = self._now()
        metrics = self.runtime.train_batch(data, policy_ratio_clip_eps=tr.policy_ratio_clip_eps,
                                           optimize_iterations_per_step=tr.optimize_iterations_per_step,
                                           max_grad_norm=tr.max_grad_norm)
        optimize_sec = self._now() - t0
        batch = reward_batch_summary(self.pending_attempts, rollout_group_size=tr.rollout_group_size,
                                     optimize_prompt_batch_size=tr.optimize_prompt_batch_size)
        metrics.update({
            "replay_buffer_optimize_threshold": threshold, "replay_buffer_trainable_completion_count": usable,
            "replay_buffer_trainable_group_count": usable / max(tr.rollout_group_size, 1),
            "optimize_prompt_batch_size": tr.optimize_prompt_batch_size,
            "optimize_iterations_per_step": tr.optimize_iterations_per_step, "force_flush": bool(force),
        })
        self.replay_buffer.consume(usable)
        attempts, timings = list(self.pending_attempts), list(self.pending_timings)
        self.pending_attempts.clear()
        self.pending_timings.clear()
        self.global_step += 1
        self.stats.optimized_steps += 1
        ckpt_sec, ckpt_dir = 0.0, None
        if tr.save_steps > 0 and self.global_step % tr.save_steps == 0:
            ckpt_dir = Path(tr.output_dir) / f"step_{self.global_step}"
            t1 = self._now()
            self._save_checkpoint(ckpt_dir, epoch=epoch)
            ckpt_sec = self._now() - t1
        window = reward_window_summary(self.recent_groups)
        health = training_health(metrics, batch, window)
        optimize = compact_optimize_metrics(metrics)
        compact = compact_batch_summary(batch)
        timing = compact_timing_summary(timings, optimize_sec=optimize_sec, checkpoint_sec=ckpt_sec, metrics=metrics)
        if self._is_primary():
            self.logger.write_train_batch_readable({"backend": "graspoflow", "epoch": epoch, "step": self.global_step,
                                                    "timestamp": _timestamp(), "batch": compact, "optimize": optimize,
                                                    "health": health, "timing": timing, "attempts": attempts})
            self.logger.write_timing_event(self._timing_event("optimize", {**timing, "attempt_total_sec":
                                                                           optimize_sec + ckpt_sec}, epoch))
        self._emit({"timestamp": _timestamp(), "event": "train_step", "backend": "graspoflow", "step": self.global_step,
                    "elapsed_sec": round(time.monotonic() - self.started_at, 3), "run": self._run_summary(),
                    "epoch": self._epoch_summary(), "batch": compact, "optimize": optimize, "timing": timing,
                    "health": health})
        if ckpt_dir is not None:
            self._emit({"timestamp": _timestamp(), "event": "checkpoint_saved", "step": self.global_step,
                        "path": str(ckpt_dir), "checkpoint_save_sec": round(ckpt_sec, 6)})
        return True

    def _run_summary(self) -> dict[str, Any]:
        s = self.stats
        return {"attempt_groups": s.total_groups,
                "completions": s.total_groups * int(self.config.training.rollout_group_size),
                "decisions": compact_decisions(perfect_skip=s.perfect_skipped, trainable_max_correct=s.trainable_max_correct,
                                               trainable_not_correct=s.trainable_not_correct, invalid=s.invalid,
                                               invalid_no_preference_gap=s.invalid_no_preference_gap,
                                               retry_attempts=s.retries),
                "optimized_steps": s.optimized_steps}

    def _epoch_summary(self) -> dict[str, Any]:
        es = self.epoch_stats
        n = max(es.attempt_groups, 1)
        return {"epoch": es.epoch, "samples_seen": es.samples_seen, "samples_total": self.total_samples,
                "progress": es.samples_seen / self.total_samples if self.total_samples else 0.0,
                "attempt_groups": es.attempt_groups, "completions": es.completion_count,
                "decisions": compact_decisions(perfect_skip=es.perfect_skipped,
                                               trainable_max_correct=es.trainable_max_correct,
                                               trainable_not_correct=es.trainable_not_correct, invalid=es.invalid,
                                               invalid_no_preference_gap=es.invalid_no_preference_gap,
                                               retry_attempts=es.retries),
                "reward_mean": es.reward_mean_sum / n if es.attempt_groups else 0.0,
                "content_mean": es.content_mean_sum / n if es.attempt_groups else 0.0,
                "best_reward": es.best_reward}

    # ------------------------------------------------------------ checkpoints
    def trainer_state(self, epoch: int) -> dict[str, Any]:
        if len(self.replay_buffer):
            raise RuntimeError("Cannot checkpoint a recoverable trainer state with a non-empty replay buffer")
        tr = self.config.training
        return {"format": "graspoflow-trainer-state", "version": 1, "global_step": self.global_step,
                "sample_index": self.sample_index, "total_samples": self.total_samples, "epoch": epoch,
                "run_stats": asdict(self.stats), "epoch_stats": asdict(self.epoch_stats),
                "config_snapshot": {"seed": tr.seed, "rollout_group_size": tr.rollout_group_size,
                                    "optimize_prompt_batch_size": tr.optimize_prompt_batch_size,
                                    "train_path": self.config.data.train_path, "max_epochs": tr.max_epochs}}

    def _save_checkpoint(self, path: Path, *, epoch: int) -> None:
        self.faults.hit("checkpoint")
        self.runtime.save_checkpoint(path, trainer_state=self.trainer_state(epoch))
        self._emit({"timestamp": _timestamp(), "event": "checkpoint_saved", "step": self.global_step, "path": str(path)})
        formats = list(self.config.export.final_formats or [])
        if path.name == "final" and formats and self._is_primary():
            from graspo_b200.models.lora_io import export_from_checkpoint

            for fmt in formats:
                dest = path / fmt
                export_from_checkpoint(path, dest, export_format=fmt, base_model_path=self.config.model.model_path)
                self._emit({"timestamp": _timestamp(), "event": "checkpoint_exported", "format": fmt, "path": str(dest)})

    def _resume_if_requested(self) -> None:
        path = self.config.training.resume_from_checkpoint
        if not path:
            return
        state = self.runtime.load_checkpoint(path)
        if not state:
            raise RuntimeError(f"checkpoint {path} has no trainer state to resume from")
        if state.get("format") != "graspoflow-trainer-state":
            raise ValueError("unrecognised trainer state format")
        snap = state.get("config_snapshot") or {}
        tr = self.config.training
        for key in ("seed", "rollout_group_size", "optimize_prompt_batch_size"):
            if key in snap and snap[key] != getattr(tr, key):
                raise ValueError(f"resume: training.{key} changed from {snap[key]} to {getattr(tr, key)}")
        self.global_step = int(state["global_step"])
        self.sample_index = int(state["sample_index"])
        self.stats = TrainStats(**state["run_stats"])
        self.epoch_stats = EpochStats(**state["epoch_stats"])
        self.resume_info = {"path": str(path), "global_step": self.global_step, "epoch": self.epoch_stats.epoch,
                            "samples_seen": self.epoch_stats.samples_seen}
        self._emit({"timestamp": _timestamp(), "event": "checkpoint_resumed", **self.resume_info})


# reference-compatible name
GraspoFlowTrainer = GraspoTrainer
