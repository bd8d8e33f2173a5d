"""Pipeline schedules as pure plan generators.

A schedule turns (stage, number of micro-batches) into an ordered list of
``forward(i)`` / ``backward(i)`` steps; the pipeline executor decides how to
compute and communicate (reference: backends/graspoflow/schedule.py:19-207).

* GPipe (``simple``/``gpipe``): all forwards, then all backwards in reverse.
* 1F1B (``one_f_one_b``/``1f1b``): ``warmup = min(pp - rank - 1, chunks,
  max_inflight)`` forwards, then alternating forward(k + warmup) /
  backward(k), then the remaining backwards; at most ``warmup + 1``
  micro-batches hold activations on a stage.
* ``async_1f1b``: the 1F1B order under its own name (the reference's async
  variant is a placeholder).  Every schedule's executor already posts each
  receive one step ahead and sends without blocking, on one communicator per
  direction, so transfers overlap the neighbouring compute steps.
"""

from __future__ import annotations

from dataclasses import dataclass
from enum import StrEnum


class PipelineAction(StrEnum):
    FORWARD = "forward"
    BACKWARD = "backward"


@dataclass(frozen=True, slots=True)
class SchedulerStep:
    action: PipelineAction
    microbatch_idx: int

    def __repr__(self) -> str:
        return f"{self.action.value}({self.microbatch_idx})"


class PipelineScheduler:
    overlap_comm = False

    def __init__(self, *, pp_size: int, pp_rank: int) -> None:
        if pp_size < 1:
            raise ValueError("pp_size must be >= 1")
        if not 0 <= pp_rank < pp_size:
            raise ValueError(f"pp_rank {pp_rank} out of range [0, {pp_size})")
        self.pp_size, self.pp_rank = pp_size, pp_rank

    @property
    def is_pipeline(self) -> bool:
        return self.pp_size > 1

    @property
    def is_first_stage(self) -> bool:
        return self.pp_rank == 0

    @property
    def is_last_stage(self) -> bool:
        return self.pp_rank == self.pp_size - 1

    def plan(self, chunk_count: int, *, max_inflight: int | None = None) -> list[SchedulerStep]:
        raise NotImplementedError

    def plan_phases(self, chunk_count: int, *, max_inflight: int | None = None) -> dict[str, list[SchedulerStep]]:
        return {"all": self.plan(chunk_count, max_inflight=max_inflight)}


F, B = PipelineAction.FORWARD, PipelineAction.BACKWARD


class GPipeScheduler(PipelineScheduler):
    def plan_phases(self, chunk_count, *, max_inflight=None):
        return {"forward": [SchedulerStep(F, i) for i in range(chunk_count)],
                "backward": [SchedulerStep(B, i) for i in reversed(range(chunk_count))]}

    def plan(self, chunk_count, *, max_inflight=None):
        phases = self.plan_phases(chunk_count)
        return phases["forward"] + phases["backward"]


class OneFOneBScheduler(PipelineScheduler):
    def warmup(self, chunk_count: int, max_inflight: int | None = None) -> int:
        n = max(0, min(self.pp_size - self.pp_rank - 1, chunk_count))
        return min(n, max_inflight) if max_inflight else n

    def plan_phases(self, chunk_count, *, max_inflight=None):
        w = self.warmup(chunk_count, max_inflight)
        rest = chunk_count - w
        steady = []
        for k in range(rest):
            steady += [SchedulerStep(F, k + w), SchedulerStep(B, k)]
        return {"fill": [SchedulerStep(F, i) for i in range(w)], "steady": steady,
                "drain": [SchedulerStep(B, i) for i in range(rest, chunk_count)]}

    def plan(self, chunk_count, *, max_inflight=None):
        p = self.plan_phases(chunk_count, max_inflight=max_inflight)
        return p["fill"] + p["steady"] + p["drain"]


class AsyncOneFOneBScheduler(OneFOneBScheduler):
    overlap_comm = True


_REGISTRY: dict[str, type[PipelineScheduler]] = {
    "simple": GPipeScheduler,
    "gpipe": GPipeScheduler,
    "one_f_one_b": OneFOneBScheduler,
    "1f1b": OneFOneBScheduler,
    "async_1f1b": AsyncOneFOneBScheduler,
}


def get_scheduler(name: str, *, pp_size: int, pp_rank: int) -> PipelineScheduler:
    key = name.lower().strip()
    cls = _REGISTRY.get(key)
    if cls is None:
        raise ValueError(f"Unknown pipeline scheduler: {name!r}. Available: {', '.join(sorted(_REGISTRY))}")
    return cls(pp_size=pp_size, pp_rank=pp_rank)


def peak_inflight(plan: list[SchedulerStep]) -> int:
    """Most micro-batches whose forward ran but whose backward has not."""
    live, peak = set(), 0
    for step in plan:
        if step.action == F:
            live.add(step.microbatch_idx)
            peak = max(peak, len(live))
        else:
            live.discard(step.microbatch_idx)
    return peak
