"""bench.py's wall-clock budget: whole steps only, at least three warm-ups and one timed step,
and as many timed steps as fit."""

import importlib.util
from pathlib import Path

ROOT = Path(__file__).resolve().parents[1]


def _bench():
    spec = importlib.util.spec_from_file_location("bench_module", ROOT / "bench.py")
    mod = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(mod)
    return mod


def _budget(mod, budget, elapsed_seq):
    b = mod.StepBudget(budget, cuda=False)
    it = iter(elapsed_seq)
    b.elapsed = lambda: next(it)  # process wall clock at each warm-up step's end
    return b


def test_fast_steps_keep_the_requested_counts():
    mod = _bench()
    b = _budget(mod, 760.0, [60, 90, 120, 150, 180])
    for _ in range(5):
        b.step_done(30.0)
    assert b.room_for(2)
    assert b.timed_steps(20) == 19  # 180 s spent, 580 s left, 30 s per step
    assert b.timed_steps(10) == 10


def test_slow_steps_run_one_timed_step_after_three_warmups():
    mod = _bench()
    b = _budget(mod, 760.0, [500, 760, 1020])
    warm = 0
    while warm < 5:
        b.step_done(260.0)
        warm += 1
        if warm >= mod.MIN_WARMUP and warm < 5 and not b.room_for(2):
            break
    assert warm == mod.MIN_WARMUP
    assert b.timed_steps(20) == 1


def test_disabled_budget():
    mod = _bench()
    b = _budget(mod, 0.0, [10_000])
    b.step_done(500.0)
    assert b.room_for(100)
    assert b.timed_steps(20) == 20
