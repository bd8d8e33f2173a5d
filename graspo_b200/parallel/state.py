"""Process groups for tensor x pipeline x data parallelism.

Rank layout (TP innermost, then PP, then DP)::

    rank = dp_rank * (pp * tp) + pp_rank * tp + tp_rank

With ``dp == 1`` this is exactly the reference layout (``pp_rank = rank // tp``,
``tp_rank = rank % tp``; reference: parallel_state.py:45-61), so per-rank
checkpoint files line up.  Pipeline neighbours are ``rank -/+ tp``.  NCCL is
used on GPUs, gloo on CPU; every group gets a finite timeout so a dead peer
ends collectives with an error rather than a hang.
"""

from __future__ import annotations

import datetime
import os
from dataclasses import dataclass, field

import torch
import torch.distributed as dist


@dataclass
class ParallelState:
    rank: int = 0
    world_size: int = 1
    local_rank: int = 0
    tp_size: int = 1
    pp_size: int = 1
    dp_size: int = 1
    tp_rank: int = 0
    pp_rank: int = 0
    dp_rank: int = 0
    device: torch.device = field(default_factory=lambda: torch.device("cpu"))
    backend: str = "none"
    tp_group: object | None = None
    pp_group: object | None = None
    dp_group: object | None = None
    tp_ranks: list[int] = field(default_factory=list)
    pp_ranks: list[int] = field(default_factory=list)
    dp_ranks: list[int] = field(default_factory=list)
    # one two-rank group per stage boundary and direction: "send_next" /
    # "recv_prev" carry activations forward, "send_prev" / "recv_next" carry
    # their gradients back (see ``initialize``)
    stage_groups: dict[str, object] = field(default_factory=dict)
    owns_process_group: bool = False

    @property
    def is_first_stage(self) -> bool:
        return self.pp_rank == 0

    @property
    def is_last_stage(self) -> bool:
        return self.pp_rank == self.pp_size - 1

    @property
    def prev_rank(self) -> int | None:
        return self.rank - self.tp_size if self.pp_rank > 0 else None

    @property
    def next_rank(self) -> int | None:
        return self.rank + self.tp_size if self.pp_rank < self.pp_size - 1 else None

    @property
    def distributed(self) -> bool:
        return self.world_size > 1 and dist.is_available() and dist.is_initialized()

    def rank_of(self, *, tp: int, pp: int, dp: int) -> int:
        return dp * (self.pp_size * self.tp_size) + pp * self.tp_size + tp


_STATE: ParallelState | None = None


def get_state() -> ParallelState:
    global _STATE
    if _STATE is None:
        _STATE = ParallelState()
    return _STATE


def initialize(
    tp_size: int = 1,
    pp_size: int = 1,
    dp_size: int = 0,
    *,
    timeout_sec: float = 600.0,
    device: str | None = None,
) -> ParallelState:
    """Create (or adopt) the default process group and the TP/PP/DP subgroups."""
    global _STATE
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local_rank = int(os.environ.get("LOCAL_RANK", "0"))
    if dist.is_available() and dist.is_initialized():
        world, rank = dist.get_world_size(), dist.get_rank()
    tp, pp = int(tp_size), int(pp_size)
    if tp < 1 or pp < 1:
        raise ValueError("tp_size and pp_size must be >= 1")
    if world % (tp * pp):
        raise ValueError(f"WORLD_SIZE={world} is not divisible by tp*pp={tp * pp}")
    dp = int(dp_size) or world // (tp * pp)
    if tp * pp * dp != world:
        raise ValueError(f"WORLD_SIZE={world} must equal tp*pp*dp={tp}*{pp}*{dp}")

    use_cuda = torch.cuda.is_available() and device != "cpu"
    if use_cuda:
        torch.cuda.set_device(local_rank)
        dev = torch.device("cuda", local_rank)
    else:
        dev = torch.device("cpu")
    owns = False
    backend = "none"
    if world > 1:
        if not dist.is_initialized():
            backend = "nccl" if use_cuda else "gloo"
            kwargs = {"backend": backend, "timeout": datetime.timedelta(seconds=timeout_sec)}
            if use_cuda:
                kwargs["device_id"] = dev
            dist.init_process_group(**kwargs)
            owns = True
        backend = dist.get_backend()

    state = ParallelState(
        rank=rank, world_size=world, local_rank=local_rank, tp_size=tp, pp_size=pp, dp_size=dp,
        device=dev, backend=backend, owns_process_group=owns,
    )
    state.tp_rank = rank % tp
    state.pp_rank = (rank // tp) % pp
    state.dp_rank = rank // (tp * pp)
    if world > 1:
        timeout = datetime.timedelta(seconds=timeout_sec)
        # every rank creates every group, in the same order
        for d in range(dp):
            for p in range(pp):
                ranks = [state.rank_of(tp=t, pp=p, dp=d) for t in range(tp)]
                group = dist.new_group(ranks, timeout=timeout)
                if rank in ranks:
                    state.tp_group, state.tp_ranks = group, ranks
        for d in range(dp):
            for t in range(tp):
                ranks = [state.rank_of(tp=t, pp=p, dp=d) for p in range(pp)]
                group = dist.new_group(ranks, timeout=timeout)
                if rank in ranks:
                    state.pp_group, state.pp_ranks = group, ranks
        for p in range(pp):
            for t in range(tp):
                ranks = [state.rank_of(tp=t, pp=p, dp=d) for d in range(dp)]
                group = dist.new_group(ranks, timeout=timeout)
                if rank in ranks:
                    state.dp_group, state.dp_ranks = group, ranks
        # Stage-boundary links.  Each boundary of each pipeline column gets two
        # groups, one per direction, so the activations going forward and the
        # gradients coming back queue on different NCCL streams.  On one
        # stream, a large send posted ahead of a receive that the peer must
        # complete first (1F1B: stage s sends micro-batch i+1 forward while
        # stage s+1 sends the gradient of micro-batch i back) waits forever;
        # with one direction per stream both ends post in the same order.
        for d in range(dp):
            for t in range(tp):
                for p in range(pp - 1):
                    pair = [state.rank_of(tp=t, pp=p, dp=d), state.rank_of(tp=t, pp=p + 1, dp=d)]
                    fwd = dist.new_group(pair, timeout=timeout)
                    bwd = dist.new_group(pair, timeout=timeout)
                    if rank == pair[0]:
                        state.stage_groups["send_next"] = fwd
                        state.stage_groups["recv_next"] = bwd
                    elif rank == pair[1]:
                        state.stage_groups["recv_prev"] = fwd
                        state.stage_groups["send_prev"] = bwd
    else:
        state.tp_ranks, state.pp_ranks, state.dp_ranks = [0], [0], [0]
    _STATE = state
    return state


def destroy() -> None:
    global _STATE
    state = _STATE
    if state is not None and state.owns_process_group and dist.is_initialized():
        try:
            dist.barrier()
        finally:
            dist.destroy_process_group()
    _STATE = None


def replica_mismatches(tensor: torch.Tensor, group, *, name: str = "tensor") -> list[str]:
    """Debug check that a tensor meant to be replicated over ``group`` holds the
    same bits on every member: all-gathers a 64-bit digest of its bytes and
    returns one message per rank that disagrees with the group's first rank
    (empty when consistent or when the group has one member)."""
    if group is None or not dist.is_available() or not dist.is_initialized():
        return []
    n = dist.get_world_size(group)
    if n <= 1:
        return []
    flat = tensor.detach().contiguous().view(-1)
    words = flat.view(torch.int32) if flat.element_size() == 4 else flat.float().view(torch.int32)
    w = words.to(torch.int64)
    idx = torch.arange(w.numel(), device=w.device, dtype=torch.int64)
    digest = torch.stack([(w * (idx % 8191 + 1)).sum(), (w ^ (idx * 2654435761 % (1 << 31))).sum()])
    gathered = [torch.empty_like(digest) for _ in range(n)]
    dist.all_gather(gathered, digest, group=group)
    ranks = dist.get_process_group_ranks(group)
    return [f"{name}: rank {ranks[i]} differs from rank {ranks[0]}" for i in range(1, n)
            if not torch.equal(gathered[i], gathered[0])]
