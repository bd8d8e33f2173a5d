"""Recoverable per-rank LoRA training checkpoints.

Layout (reference: transformer_adapter.py:295-425, trainer/checkpoint.py)::

    <dir>/rank_{rank:05d}_tp_{tp:02d}_pp_{pp:02d}.pt   one per (tp, pp) cell
    <dir>/manifest.json                                written by rank 0

Payload keys: ``adapter, rank, tp_rank, tp_size, pp_rank, pp_size, placement,
lora_target_signature, lora_tensor_metadata, lora_state_dict,
optimizer_state_dict, scheduler_state_dict, torch_rng_state, cuda_rng_state,
adapter_state, trainer_state, config``.  Additions: ``dp_size`` in payload and
manifest; only data-parallel replica 0 writes (replicas hold identical LoRA
state), under its own rank number so file names stay those of a dp=1 run.
Files are written to a temporary name and renamed, so a crash mid-save never
leaves a truncated shard; the manifest is written last, after a barrier.
"""

from __future__ import annotations

import json
import os
from pathlib import Path
from typing import Any

import torch
import torch.distributed as dist

from graspo_b200.parallel.placement import placement_summary


def rank_file_name(rank: int, tp_rank: int, pp_rank: int) -> str:
    return f"rank_{rank:05d}_tp_{tp_rank:02d}_pp_{pp_rank:02d}.pt"


def _atomic_save(obj: Any, path: Path) -> None:
    tmp = path.with_name(path.name + f".tmp{os.getpid()}")
    torch.save(obj, tmp)
    os.replace(tmp, path)


def _atomic_write_text(path: Path, text: str) -> None:
    tmp = path.with_name(path.name + f".tmp{os.getpid()}")
    tmp.write_text(text, encoding="utf-8")
    os.replace(tmp, path)


def _to_cpu(obj: Any) -> Any:
    """Deep copy with every tensor cloned to host memory (a snapshot that later
    training steps cannot change)."""
    if isinstance(obj, torch.Tensor):
        return obj.detach().to("cpu", copy=True)
    if isinstance(obj, dict):
        return {k: _to_cpu(v) for k, v in obj.items()}
    if isinstance(obj, (list, tuple)):
        return type(obj)(_to_cpu(v) for v in obj)
    return obj


def build_rank_payload(adapter, trainer_state: dict | None) -> dict | None:
    """This rank's shard payload (None on data-parallel replicas other than 0)."""
    ps = adapter.ps
    model = adapter.model
    cell_rank = ps.rank_of(tp=ps.tp_rank, pp=ps.pp_rank, dp=0)
    if ps.dp_rank == 0:
        return {
            "adapter": "graspoflow",
            "rank": cell_rank,
            "tp_rank": ps.tp_rank,
            "tp_size": ps.tp_size,
            "pp_rank": ps.pp_rank,
            "pp_size": ps.pp_size,
            "dp_size": ps.dp_size,
            "placement": placement_summary(adapter.placement),
            "lora_target_signature": model.lora_target_signature(),
            "lora_tensor_metadata": model.lora_tensor_metadata(),
            "lora_state_dict": model.lora_state_dict(),
            "optimizer_state_dict": adapter.optimizer.state_dict() if adapter.optimizer else None,
            "scheduler_state_dict": {"step": adapter.optimizer.step_count} if adapter.optimizer else None,
            "torch_rng_state": torch.get_rng_state(),
            "cuda_rng_state": torch.cuda.get_rng_state(ps.device) if ps.device.type == "cuda" else None,
            "adapter_state": {"train_batch_call_index": adapter._train_batch_call_index},
            "trainer_state": trainer_state,
            "config": adapter.config.model_dump(),
        }
    return None


def shard_path(adapter, path: Path) -> Path:
    ps = adapter.ps
    cell_rank = ps.rank_of(tp=ps.tp_rank, pp=ps.pp_rank, dp=0)
    return path / rank_file_name(cell_rank, ps.tp_rank, ps.pp_rank)


def save_rank_checkpoint(adapter, path: Path, *, trainer_state: dict | None = None) -> None:
    path.mkdir(parents=True, exist_ok=True)
    payload = build_rank_payload(adapter, trainer_state)
    if payload is not None:
        _atomic_save(payload, shard_path(adapter, path))
    finish_checkpoint(adapter, path, has_trainer_state=trainer_state is not None)


def finish_checkpoint(adapter, path: Path, *, has_trainer_state: bool) -> None:
    """Barrier over every rank, then rank 0 writes the manifest (the checkpoint
    counts as complete only once the manifest exists)."""
    ps = adapter.ps
    model = adapter.model
    if ps.distributed:
        dist.barrier()
    if ps.rank == 0:
        manifest = {
            "format": "graspoflow-lora",
            "tp_size": ps.tp_size,
            "pp_size": ps.pp_size,
            "dp_size": ps.dp_size,
            "placement": placement_summary(adapter.placement),
            "lora_target_signature": model.lora_target_signature(),
            "world_size": ps.tp_size * ps.pp_size,
            "checkpoint_type": "recoverable_lora_training_state",
            "has_trainer_state": bool(has_trainer_state),
        }
        _atomic_write_text(path / "manifest.json", json.dumps(manifest, ensure_ascii=False, indent=2))


class AsyncCheckpointWriter:
    """Background shard writer (``graspoflow.async_checkpoint``).

    ``submit`` snapshots the shard payload into host memory on the calling
    thread (so later optimizer steps cannot leak into it) and serialises it on
    a worker thread while training continues.  ``wait`` joins the worker, then
    runs the cross-rank barrier and the manifest write of ``finish_checkpoint``;
    every rank calls it at the same program points (the next save, the final
    save, shutdown), so at most one checkpoint is in flight and a checkpoint
    without its manifest is never taken for a finished one."""

    def __init__(self) -> None:
        self._thread = None
        self._error: BaseException | None = None
        self._pending: tuple[Path, bool] | None = None

    def submit(self, adapter, path: Path, *, trainer_state: dict | None = None) -> None:
        import threading

        self.wait(adapter)
        path.mkdir(parents=True, exist_ok=True)
        payload = build_rank_payload(adapter, trainer_state)
        payload = _to_cpu(payload) if payload is not None else None
        target = shard_path(adapter, path)

        def work() -> None:
            try:
                if payload is not None:
                    _atomic_save(payload, target)
            except BaseException as exc:  # noqa: BLE001 - re-raised by wait()
                self._error = exc

        self._thread = threading.Thread(target=work, name="graspo-checkpoint", daemon=True)
        self._thread.start()
        self._pending = (path, trainer_state is not None)

    @property
    def pending(self) -> bool:
        return self._pending is not None

    def abandon(self) -> None:
        """Join the worker without the barrier and manifest (error paths: the other
        ranks may never reach the barrier); the directory stays without a manifest."""
        if self._thread is not None:
            self._thread.join()
        self._thread, self._pending, self._error = None, None, None

    def wait(self, adapter) -> None:
        if self._pending is None:
            return
        self._thread.join()
        path, has_state = self._pending
        self._pending, self._thread = None, None
        if self._error is not None:
            err, self._error = self._error, None
            raise RuntimeError(f"background checkpoint write to {path} failed") from err
        finish_checkpoint(adapter, path, has_trainer_state=has_state)


def load_rank_checkpoint(adapter, path: Path) -> dict | None:
    ps = adapter.ps
    model = adapter.model
    cell_rank = ps.rank_of(tp=ps.tp_rank, pp=ps.pp_rank, dp=0)
    shard = path / rank_file_name(cell_rank, ps.tp_rank, ps.pp_rank)
    if not shard.exists():
        raise FileNotFoundError(
            f"Missing GRASPO checkpoint shard for rank={cell_rank} tp_rank={ps.tp_rank} pp_rank={ps.pp_rank}: {shard}"
        )
    payload = torch.load(shard, map_location="cpu", weights_only=False)
    if int(payload.get("tp_size", ps.tp_size)) != ps.tp_size:
        raise ValueError(f"Checkpoint TP size {payload.get('tp_size')} does not match runtime TP size {ps.tp_size}")
    if int(payload.get("pp_size", ps.pp_size)) != ps.pp_size:
        raise ValueError(f"Checkpoint PP size {payload.get('pp_size')} does not match runtime PP size {ps.pp_size}")
    sig = payload.get("lora_target_signature")
    if sig is not None and sig != model.lora_target_signature():
        raise ValueError(
            "Checkpoint LoRA target signature does not match runtime configuration: "
            f"checkpoint={sig}, runtime={model.lora_target_signature()}"
        )
    model.lora.load_state_dict(payload["lora_state_dict"], strict=True)
    opt = payload.get("optimizer_state_dict")
    if adapter.optimizer is not None:
        if opt is None:
            raise RuntimeError("Checkpoint shard is missing optimizer state for a trainable rank")
        adapter.optimizer.load_state_dict(opt)
    torch.set_rng_state(payload["torch_rng_state"].cpu())
    if payload.get("cuda_rng_state") is not None and ps.device.type == "cuda":
        torch.cuda.set_rng_state(payload["cuda_rng_state"].cpu(), ps.device)
    adapter._train_batch_call_index = int((payload.get("adapter_state") or {}).get("train_batch_call_index") or 0)
    return payload.get("trainer_state")


def read_manifest(path: str | Path) -> dict:
    return json.loads((Path(path) / "manifest.json").read_text(encoding="utf-8"))
