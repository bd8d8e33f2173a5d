"""Stage transfers under the 1F1B and GPipe plans: every stage receives exactly
the tensor its neighbour sent for that micro-batch, with receives posted one
receiving step early.  CPU ranks over gloo; the GPU case uses messages far
larger than NCCL's staging buffer, where forward and backward transfers that
shared one stream would wait on each other."""

import pytest
import torch

from tests.dist_util import run_world


def _expected(c: int, stage: int, backward: bool) -> float:
    # forward: micro-batch c leaves stage s carrying c * 16 + s + 1;
    # backward: its gradient leaves stage s carrying -(c * 16 + s + 1)
    # (small integers, exact in bf16)
    v = float(c * 16 + stage + 1)
    return -v if backward else v


def _schedule_worker(rank, world, tp, pp, numel, schedule, cuda):
    from graspo_b200.engine.pipeline import _plan_needs, _RecvAhead
    from graspo_b200.parallel import state as pstate
    from graspo_b200.parallel.p2p import StageComm
    from graspo_b200.parallel.schedule import PipelineAction, get_scheduler
    from graspo_b200.utils.timing import schedule_phases

    if cuda:
        import os

        os.environ["NCCL_NVLS_ENABLE"] = "0"
    ps = pstate.initialize(tp, pp, 0, timeout_sec=60, device=None if cuda else "cpu")
    assert ps.stage_groups, "pipeline ranks get per-direction stage groups"
    comm = StageComm(ps)
    chunks = [slice(i, i + 1) for i in range(5)]
    plan = schedule_phases(get_scheduler(schedule, pp_size=pp, pp_rank=ps.pp_rank), len(chunks))
    dtype = torch.bfloat16 if cuda else torch.float32
    ahead = _RecvAhead(comm, _plan_needs(plan, chunks, ps, lambda rows: (rows * numel,)), dtype)
    s = ps.pp_rank
    for k, (_, step) in enumerate(plan):
        c = step.microbatch_idx
        ahead.advance(k)
        if step.action == PipelineAction.FORWARD:
            if s > 0:
                x = comm.recv_prev((numel,), dtype)
                assert torch.all(x == _expected(c, s - 1, False)), (rank, "fwd", c)
            comm.send_next(torch.full((numel,), _expected(c, s, False), dtype=dtype, device=ps.device))
        else:
            if s < pp - 1:
                g = comm.recv_next((numel,), dtype)
                assert torch.all(g == _expected(c, s + 1, True)), (rank, "bwd", c)
            comm.send_prev(torch.full((numel,), _expected(c, s, True), dtype=dtype, device=ps.device))
    comm.flush()
    if cuda:
        torch.cuda.synchronize()
    pstate.destroy()


@pytest.mark.parametrize("tp,pp,schedule", [(1, 2, "one_f_one_b"), (1, 4, "one_f_one_b"), (2, 2, "one_f_one_b"),
                                             (1, 3, "gpipe")])
def test_stage_transfers_follow_the_plan(tp, pp, schedule):
    run_world(tp * pp, _schedule_worker, tp, pp, 4096, schedule, False, timeout=180)


def test_posted_receive_must_be_taken():
    from types import SimpleNamespace

    from graspo_b200.parallel.p2p import StageComm

    comm = StageComm(SimpleNamespace(pp_size=1, prev_rank=None, next_rank=None, stage_groups={}))
    comm.prefetch_prev((4,), torch.float32)  # no previous stage: nothing is posted
    comm.flush()


@pytest.mark.gpu
@pytest.mark.skipif(torch.cuda.device_count() < 2, reason="needs 2 GPUs")
def test_stage_transfers_large_messages_on_gpus():
    # 64 MiB per transfer (bf16), about 16x NCCL's default staging buffer
    run_world(2, _schedule_worker, 1, 2, 32 << 20, "one_f_one_b", True, timeout=300)


# ---------------------------------------------------------------------------
# Rendezvous model of the transfer queues.  A send completes only together with
# its matching receive, and each queue runs its operations strictly in order
# (a large NCCL send cannot finish before the peer's receive runs).  A rank
# posts receives ahead, then blocks on taking them, as ``_RecvAhead`` does.


class _Recorder:
    """StageComm stand-in that records each rank's issue order."""

    def __init__(self, pp_rank, pp):
        self.s, self.pp, self.program = pp_rank, pp, []
        self.counts = {"prev": 0, "next": 0}
        self.taken = {"prev": 0, "next": 0}

    def prefetch_prev(self, shape, dtype):
        self._post("prev")

    def prefetch_next(self, shape, dtype):
        self._post("next")

    def _post(self, side):
        if (side == "prev" and self.s == 0) or (side == "next" and self.s == self.pp - 1):
            return
        self.program.append(("post", side, self.counts[side]))
        self.counts[side] += 1

    def take(self, side):
        if self.taken[side] == self.counts[side]:
            self._post(side)
        self.program.append(("take", side, self.taken[side]))
        self.taken[side] += 1

    def send(self, side):
        self.program.append(("send", side, None))


def _programs(pp, n_micro, schedule, max_inflight=0):
    from graspo_b200.engine.pipeline import _plan_needs, _RecvAhead
    from graspo_b200.parallel.schedule import PipelineAction, get_scheduler
    from graspo_b200.utils.timing import schedule_phases

    progs = []
    chunks = [slice(i, i + 1) for i in range(n_micro)]
    for s in range(pp):
        rec = _Recorder(s, pp)
        ps = type("PS", (), {"is_first_stage": s == 0, "is_last_stage": s == pp - 1})()
        plan = schedule_phases(get_scheduler(schedule, pp_size=pp, pp_rank=s), n_micro, max_inflight)
        ahead = _RecvAhead(rec, _plan_needs(plan, chunks, ps, lambda rows: (rows,)), torch.float32)
        for k, (_, step) in enumerate(plan):
            ahead.advance(k)
            if step.action == PipelineAction.FORWARD:
                if s > 0:
                    rec.take("prev")
                if s < pp - 1:
                    rec.send("next")
            else:
                if s < pp - 1:
                    rec.take("next")
                if s > 0:
                    rec.send("prev")
        progs.append(rec.program)
    return progs


def _runs_to_completion(progs, per_direction: bool) -> bool:
    """Simulate the queues; True when every operation completes."""
    pp = len(progs)
    pc = [0] * pp
    queues: dict[tuple, list] = {}  # (rank, queue key) -> [op id, ...] in issue order
    done: set = set()
    sends = {}  # (src, dst) -> sends issued so far (one direction per neighbour)

    def key(r, peer, direction):
        lo, hi = min(r, peer), max(r, peer)
        return (lo, hi, direction) if per_direction else (lo, hi)

    progress = True
    while progress:
        progress = False
        # issue what each host can issue without blocking
        for r in range(pp):
            while pc[r] < len(progs[r]):
                kind, side, idx = progs[r][pc[r]]
                peer = r - 1 if side == "prev" else r + 1
                direction = "fwd" if (side == "prev") == (kind != "send") else "bwd"
                if kind == "take":
                    if ("recv", r, side, idx) not in done:
                        break
                elif kind == "post":
                    queues.setdefault((r, key(r, peer, direction)), []).append(("recv", r, side, idx))
                else:
                    n = sends.get((r, peer), 0)
                    sends[(r, peer)] = n + 1
                    queues.setdefault((r, key(r, peer, direction)), []).append(("send", r, side, n))
                pc[r] += 1
                progress = True
        # complete matching queue heads
        for (r, k), q in list(queues.items()):
            if not q or q[0][0] != "send":
                continue
            _, src, side, n = q[0]
            dst = src + 1 if side == "next" else src - 1
            peer_side = "prev" if side == "next" else "next"
            q2 = queues.get((dst, k), [])
            if q2 and q2[0] == ("recv", dst, peer_side, n):
                q.pop(0)
                q2.pop(0)
                done.add(("recv", dst, peer_side, n))
                progress = True
    return all(pc[r] == len(progs[r]) for r in range(pp)) and not any(queues.values())


@pytest.mark.parametrize("pp,n_micro", [(2, 4), (4, 8), (8, 16), (4, 3)])
def test_direction_queues_cannot_deadlock(pp, n_micro):
    for schedule in ("one_f_one_b", "gpipe"):
        assert _runs_to_completion(_programs(pp, n_micro, schedule), per_direction=True), schedule
    # graspoflow.pp_max_inflight_microbatches caps the 1F1B warm-up
    for cap in (1, 2):
        assert _runs_to_completion(_programs(pp, n_micro, "one_f_one_b", cap), per_direction=True), cap


def test_inflight_cap_bounds_live_microbatches():
    from graspo_b200.parallel.schedule import get_scheduler, peak_inflight
    from graspo_b200.utils.timing import schedule_phases

    for cap in (1, 2, 3):
        plan = [step for _, step in schedule_phases(get_scheduler("one_f_one_b", pp_size=8, pp_rank=0), 16, cap)]
        assert peak_inflight(plan) == cap + 1
        assert sorted((s.action, s.microbatch_idx) for s in plan) == sorted(
            [(a, i) for a in ("forward", "backward") for i in range(16)])


def test_one_shared_queue_per_boundary_deadlocks_under_1f1b():
    # the reason for two groups per boundary: with receives posted ahead and a
    # single queue, 1F1B stalls (stage 0's gradient receive sits in front of
    # its next forward send while stage 1 waits for that send)
    assert not _runs_to_completion(_programs(2, 4, "one_f_one_b"), per_direction=False)


def _leaving_stage_worker(rank, world, timeout_sec):
    """Stage 1 leaves between steps (exits without posting its receive); stage 0's
    next transfer with it must end with an error, not wait for ever."""
    import time

    from graspo_b200.parallel import state as pstate
    from graspo_b200.parallel.p2p import StageComm

    ps = pstate.initialize(1, 2, 0, timeout_sec=timeout_sec, device="cpu")
    comm = StageComm(ps)
    comm.send_next(torch.ones(8))                    # one completed step
    if rank == 1:
        assert torch.equal(comm.recv_prev((8,), torch.float32), torch.ones(8))
        return                                       # leaves; no destroy, no further collectives
    comm.flush()
    t0 = time.monotonic()
    try:
        comm.recv_next((1 << 16,), torch.float32)    # the gradient that never comes
    except RuntimeError:
        elapsed = time.monotonic() - t0
        assert elapsed < timeout_sec + 30, elapsed
        return
    raise AssertionError("a receive from a stage that left returned normally")


def test_stage_that_leaves_ends_the_neighbours_transfer():
    run_world(2, _leaving_stage_worker, 10.0, timeout=120)
