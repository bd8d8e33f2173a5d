"""Point-to-point transfers between neighbouring pipeline stages.

Stage ``s`` of a pipeline column talks to ``s - 1`` (global rank ``rank - tp``)
and ``s + 1`` (``rank + tp``); every TP rank of a stage exchanges its own
(replicated) hidden state with the same TP rank of the neighbour stage
(reference: backends/graspoflow/transformer_op.py:85-97, training.py:509-565).

Sends are non-blocking (``isend``) and kept until ``flush``; receives block
the issuing stream (NCCL) or the host (gloo).  With sends never blocking, any
schedule in which both sides post matching operations in the same order --
GPipe, 1F1B -- cannot deadlock.  On GPUs the NCCL transfers run on NCCL's
stream, ordered after the compute that produced the tensor.
"""

from __future__ import annotations

import torch
import torch.distributed as dist


class StageComm:
    def __init__(self, ps) -> None:
        self.ps = ps
        self._pending: list[tuple[object, torch.Tensor]] = []

    @property
    def active(self) -> bool:
        return self.ps.pp_size > 1 and self.ps.distributed

    def _send(self, t: torch.Tensor, dst: int) -> None:
        t = t.contiguous()
        self._pending.append((dist.isend(t, dst), t))

    def send_next(self, t: torch.Tensor) -> None:
        if self.ps.next_rank is not None:
            self._send(t, self.ps.next_rank)

    def send_prev(self, t: torch.Tensor) -> None:
        if self.ps.prev_rank is not None:
            self._send(t, self.ps.prev_rank)

    def _recv(self, shape, dtype, src: int, out: torch.Tensor | None = None) -> torch.Tensor:
        buf = out if out is not None else torch.empty(shape, dtype=dtype, device=self.ps.device)
        dist.recv(buf, src)
        return buf

    def recv_prev(self, shape, dtype, out: torch.Tensor | None = None) -> torch.Tensor:
        return self._recv(shape, dtype, self.ps.prev_rank, out)

    def recv_next(self, shape, dtype, out: torch.Tensor | None = None) -> torch.Tensor:
        return self._recv(shape, dtype, self.ps.next_rank, out)

    def flush(self) -> None:
        for work, _ in self._pending:
            work.wait()
        self._pending.clear()

    def last_stage_rank(self) -> int:
        return self.ps.pp_ranks[-1]

    def broadcast_from_last(self, t: torch.Tensor) -> torch.Tensor:
        """Make ``t`` on every stage of the column equal to the last stage's."""
        if self.active:
            dist.broadcast(t, src=self.last_stage_rank(), group=self.ps.pp_group)
        return t
