"""Dataflow building blocks for pipelined execution.

* ``Microbatch`` -- one slice of a batch moving through the stages, with its
  tensors and per-stage bookkeeping.
* ``OpBuffer`` -- a bounded FIFO between operators; ``push`` refuses when full
  (back-pressure) instead of growing.
* ``ComputeOperator`` -- one stage's compute (forward / backward of a set of
  layers); subclasses own the tensors saved between them.
* ``PipelineGraph`` -- wires operators through buffers and executes a plan
  from ``parallel.schedule`` on this rank.

(Reference: backends/graspoflow/operator.py:19-239, graph.py:29-168.)
"""

from __future__ import annotations

from collections import deque
from dataclasses import dataclass, field
from typing import Any

import torch

from graspo_b200.parallel.schedule import PipelineAction, SchedulerStep


@dataclass
class Microbatch:
    idx: int
    tensors: dict[str, torch.Tensor] = field(default_factory=dict)
    meta: dict[str, Any] = field(default_factory=dict)
    retry: int = 0

    @property
    def batch_size(self) -> int:
        for t in self.tensors.values():
            if isinstance(t, torch.Tensor) and t.dim() > 0:
                return int(t.shape[0])
        return 0

    @property
    def seq_len(self) -> int:
        for t in self.tensors.values():
            if isinstance(t, torch.Tensor) and t.dim() > 1:
                return int(t.shape[1])
        return 0

    def clone_for_retry(self, idx: int | None = None) -> Microbatch:
        return Microbatch(idx=self.idx if idx is None else idx, tensors=dict(self.tensors), meta=dict(self.meta),
                          retry=self.retry + 1)


@dataclass(frozen=True)
class OpMemoryProfile:
    activation_bytes: int = 0
    kv_bytes: int = 0
    workspace_bytes: int = 0

    @property
    def total_per_microbatch(self) -> int:
        return self.activation_bytes + self.kv_bytes + self.workspace_bytes


class OpBuffer:
    def __init__(self, max_slots: int, name: str = "") -> None:
        if max_slots < 1:
            raise ValueError("OpBuffer needs at least one slot")
        self.max_slots = int(max_slots)
        self.name = name
        self._q: deque[Microbatch] = deque()

    @property
    def is_full(self) -> bool:
        return len(self._q) >= self.max_slots

    @property
    def is_empty(self) -> bool:
        return not self._q

    @property
    def size(self) -> int:
        return len(self._q)

    @property
    def waterlevel(self) -> float:
        return len(self._q) / self.max_slots

    def push(self, mb: Microbatch) -> bool:
        if self.is_full:
            return False
        self._q.append(mb)
        return True

    def pop(self) -> Microbatch | None:
        return self._q.popleft() if self._q else None

    def peek(self) -> Microbatch | None:
        return self._q[0] if self._q else None

    def clear(self) -> None:
        self._q.clear()

    def __len__(self) -> int:
        return len(self._q)

    def __repr__(self) -> str:
        return f"OpBuffer({self.name!r}, {len(self._q)}/{self.max_slots})"


class ComputeOperator:
    """One stage's compute.  Override ``forward`` / ``backward``."""

    def __init__(self, *, name: str, tp_size: int = 1) -> None:
        self.name = name
        self.tp_size = tp_size
        self.input_buffer: OpBuffer | None = None
        self.output_buffer: OpBuffer | None = None
        self.forward_count = 0
        self.backward_count = 0

    def attach_buffers(self, input_buffer: OpBuffer | None, output_buffer: OpBuffer | None) -> None:
        self.input_buffer, self.output_buffer = input_buffer, output_buffer

    def forward(self, mb: Microbatch) -> Microbatch:
        raise NotImplementedError

    def backward(self, mb: Microbatch) -> Microbatch:
        raise NotImplementedError

    def memory_profile(self) -> OpMemoryProfile:
        return OpMemoryProfile()

    def trainable_parameters(self) -> list[torch.Tensor]:
        return []

    def done(self) -> None:
        """Release per-chunk state (called when a plan finishes)."""

    def __repr__(self) -> str:
        return f"{type(self).__name__}({self.name!r})"


class PipelineGraph:
    """Operators of this rank chained through bounded buffers."""

    def __init__(self, operators: list[ComputeOperator], *, buffer_slots: int = 2) -> None:
        if not operators:
            raise ValueError("PipelineGraph needs at least one operator")
        self.operators = list(operators)
        self.buffers = [OpBuffer(buffer_slots, f"buf{i}") for i in range(len(operators) + 1)]
        for i, op in enumerate(self.operators):
            op.attach_buffers(self.buffers[i], self.buffers[i + 1])
        self._inflight: dict[int, Microbatch] = {}

    @property
    def first_op(self) -> ComputeOperator:
        return self.operators[0]

    @property
    def last_op(self) -> ComputeOperator:
        return self.operators[-1]

    def push_input(self, mb: Microbatch) -> bool:
        return self.buffers[0].push(mb)

    def collect_output(self) -> Microbatch | None:
        return self.buffers[-1].pop()

    def execute_plan(self, plan: list[SchedulerStep], inputs: dict[int, Microbatch]) -> dict[int, Microbatch]:
        """Run forward/backward steps; returns the forward outputs by index."""
        outputs: dict[int, Microbatch] = {}
        for step in plan:
            if step.action == PipelineAction.FORWARD:
                mb = inputs[step.microbatch_idx]
                for op in self.operators:
                    mb = op.forward(mb)
                    op.forward_count += 1
                self._inflight[step.microbatch_idx] = mb
                outputs[step.microbatch_idx] = mb
            else:
                mb = self._inflight.pop(step.microbatch_idx)
                for op in reversed(self.operators):
                    mb = op.backward(mb)
                    op.backward_count += 1
        return outputs

    def shutdown(self) -> None:
        for op in self.operators:
            op.done()
        for buf in self.buffers:
            buf.clear()
        self._inflight.clear()
