"""Point-to-point transfers between neighbouring pipeline stages.

Stage ``s`` of a pipeline column talks to ``s - 1`` (global rank ``rank - tp``)
and ``s + 1`` (``rank + tp``); every TP rank of a stage exchanges its own
(replicated) hidden state with the same TP rank of the neighbour stage
(reference: backends/graspoflow/transformer_op.py:85-97, training.py:509-565,
where every transfer is a blocking call between the stage computations).

Each boundary has one process group per direction (``ParallelState.stage_groups``):
activations travel forward on one, their gradients backward on the other.
Both ends of a group post their operations in the same order (the schedule's
order), and a group carries one direction only, so no send can sit in front of
a receive that its peer needs first -- the head-to-head wait that a single
shared stream has under 1F1B once a message outgrows NCCL's staging buffer.

Sends are non-blocking and kept alive until they complete.  Receives can be
posted ahead of need (``prefetch_prev`` / ``prefetch_next``): the pipeline
posts the next receive before it computes the current micro-batch, so the
transfer runs on NCCL's stream under that computation, and ``recv_*`` then
takes the oldest posted receive of its direction.  On GPUs the transfers are
ordered after the compute that produced (or allocated) their tensors and the
consumer's stream waits only on its own transfer.
"""

from __future__ import annotations

from collections import deque

import torch
import torch.distributed as dist


class StageComm:
    def __init__(self, ps) -> None:
        self.ps = ps
        self._sends: list[tuple[object, torch.Tensor]] = []
        # receives posted ahead of need, oldest first, per direction
        self._posted: dict[str, deque] = {"prev": deque(), "next": deque()}

    @property
    def active(self) -> bool:
        return self.ps.pp_size > 1 and self.ps.distributed

    def _link(self, name: str):
        """The direction's process group (None: the default group)."""
        return (getattr(self.ps, "stage_groups", None) or {}).get(name)

    # ------------------------------------------------------------------ sends
    def _send(self, t: torch.Tensor, dst: int, link: str) -> None:
        t = t.contiguous()
        self._sends.append((dist.isend(t, dst, group=self._link(link)), t))
        if len(self._sends) > 8:  # release the buffers of sends that have finished
            self._sends = [(w, x) for w, x in self._sends if not w.is_completed()]

    def send_next(self, t: torch.Tensor) -> None:
        if self.ps.next_rank is not None:
            self._send(t, self.ps.next_rank, "send_next")

    def send_prev(self, t: torch.Tensor) -> None:
        if self.ps.prev_rank is not None:
            self._send(t, self.ps.prev_rank, "send_prev")

    # --------------------------------------------------------------- receives
    def _post(self, side: str, shape, dtype, out: torch.Tensor | None) -> None:
        src = self.ps.prev_rank if side == "prev" else self.ps.next_rank
        buf = out if out is not None else torch.empty(shape, dtype=dtype, device=self.ps.device)
        work = dist.irecv(buf, src, group=self._link("recv_prev" if side == "prev" else "recv_next"))
        self._posted[side].append((work, buf))

    def _take(self, side: str, shape, dtype, out: torch.Tensor | None) -> torch.Tensor:
        q = self._posted[side]
        if not q:
            self._post(side, shape, dtype, out)
        work, buf = q.popleft()
        if tuple(buf.shape) != tuple(shape) or buf.dtype != dtype:
            raise RuntimeError(f"posted receive from the {side} stage holds {tuple(buf.shape)} {buf.dtype}, "
                               f"the schedule expects {tuple(shape)} {dtype}")
        work.wait()
        if out is not None and out.data_ptr() != buf.data_ptr():
            out.copy_(buf)
            return out
        return buf

    def prefetch_prev(self, shape, dtype) -> None:
        """Post the next receive from the previous stage now; ``recv_prev`` returns it."""
        if self.ps.prev_rank is not None:
            self._post("prev", shape, dtype, None)

    def prefetch_next(self, shape, dtype) -> None:
        """Post the next receive from the next stage now; ``recv_next`` returns it."""
        if self.ps.next_rank is not None:
            self._post("next", shape, dtype, None)

    def recv_prev(self, shape, dtype, out: torch.Tensor | None = None) -> torch.Tensor:
        return self._take("prev", shape, dtype, out)

    def recv_next(self, shape, dtype, out: torch.Tensor | None = None) -> torch.Tensor:
        return self._take("next", shape, dtype, out)

    # ------------------------------------------------------------------ misc
    def flush(self) -> None:
        """Wait for every send; a receive still posted here is a schedule error."""
        for work, _ in self._sends:
            work.wait()
        self._sends.clear()
        left = {side: len(q) for side, q in self._posted.items() if q}
        if left:
            raise RuntimeError(f"receives posted but never taken: {left}")

    def last_stage_rank(self) -> int:
        return self.ps.pp_ranks[-1]

    def broadcast_from_last(self, t: torch.Tensor) -> torch.Tensor:
        """Make ``t`` on every stage of the column equal to the last stage's."""
        if self.active:
            dist.broadcast(t, src=self.last_stage_rank(), group=self.ps.pp_group)
        return t
