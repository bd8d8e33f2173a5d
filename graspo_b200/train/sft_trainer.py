"""Supervised fine-tuning of the LoRA adapter on the JSONL targets.

Each sample becomes ``prompt (as rendered for rollout) + primary target +
EOS`` with labels masked on the prompt (``core.data.sft_tokenize``).  Batches
of ``optimize_prompt_batch_size`` samples go to ``runtime.train_batch_sft``;
checkpoints follow ``save_steps`` / ``save_checkpoint_every_epoch`` / final
(reference: trainer/sft_trainer.py:26-172).  Data-parallel replicas take
disjoint slices of every global batch.
"""

from __future__ import annotations

import json
import logging
import random
import time
from datetime import datetime
from pathlib import Path

from graspo_b200.core.data import load_jsonl, sft_tokenize
from graspo_b200.core.logging import setup_logging
from graspo_b200.train.logger import append_event
from graspo_b200.engine.runtime import GraspoFlowRuntime

log = logging.getLogger("graspo.sft")


class SFTTrainer:
    def __init__(self, config, runtime=None) -> None:
        self.config = config
        self.runtime = runtime or GraspoFlowRuntime.from_config(config)
        self.global_step = 0

    def _emit(self, payload: dict) -> None:
        if self.runtime.is_primary():
            print(json.dumps(payload, ensure_ascii=False, default=str), flush=True)
            append_event(self.config.training.output_dir, payload)

    def _checkpoint(self, path: Path, epoch: int) -> None:
        state = {"format": "graspoflow-trainer-state", "version": 1, "global_step": self.global_step,
                 "sample_index": 0, "total_samples": 0, "epoch": epoch, "run_stats": {}, "epoch_stats": {},
                 "train_method": "sft"}
        self.runtime.save_checkpoint(path, trainer_state=state)
        self._emit({"timestamp": datetime.now().astimezone().isoformat(timespec="seconds"),
                    "event": "checkpoint_saved", "step": self.global_step, "path": str(path)})

    def train(self) -> None:
        cfg, tr = self.config, self.config.training
        self.runtime.validate()
        self.runtime.setup()
        setup_logging(tr.output_dir, rank=int(getattr(self.runtime, "rank", 0)))
        out = Path(tr.output_dir)
        out.mkdir(parents=True, exist_ok=True)
        tok = self.runtime.tokenizer
        samples = load_jsonl(cfg.data.train_path)
        max_len = int(cfg.data.max_prompt_length) + int(tr.max_new_tokens)
        data = [sft_tokenize(s, tok, max_seq_length=max_len, chat_template_kwargs=cfg.model.chat_template_kwargs)
                for s in samples]
        ps = getattr(self.runtime, "ps", None)
        dp_rank, dp_size = (ps.dp_rank, ps.dp_size) if ps is not None else (0, 1)
        bs = max(1, int(tr.optimize_prompt_batch_size))
        log.info("SFT: %d samples, batch %d x dp %d, epochs %d", len(data), bs, dp_size, tr.max_epochs)
        try:
            for epoch in range(int(tr.max_epochs)):
                order = list(data)
                random.Random(int(tr.seed) + epoch).shuffle(order)
                for b, start in enumerate(range(0, len(order) - bs * dp_size + 1, bs * dp_size)):
                    batch = order[start + dp_rank * bs : start + (dp_rank + 1) * bs]
                    t0 = time.monotonic()
                    metrics = self.runtime.train_batch_sft(batch, optimize_iterations_per_step=tr.optimize_iterations_per_step,
                                                           max_grad_norm=tr.max_grad_norm)
                    self.global_step += 1
                    self._emit({"event": "sft_step", "step": self.global_step, "epoch": epoch, "batch": b,
                                "loss": metrics.get("global_loss_mean", metrics.get("loss_mean")),
                                "lr": metrics.get("current_lr"), "batch_sec": round(time.monotonic() - t0, 3)})
                    if tr.save_steps > 0 and self.global_step % tr.save_steps == 0:
                        self._checkpoint(out / f"step_{self.global_step}", epoch)
                    if 0 < tr.max_steps <= self.global_step:
                        self._checkpoint(out / "final", epoch)
                        return
                if tr.save_checkpoint_every_epoch:
                    self._checkpoint(out / f"epoch_{epoch}", epoch)
            self._checkpoint(out / "final", int(tr.max_epochs) - 1)
        finally:
            self.runtime.close()
