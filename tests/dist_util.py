"""Spawn a small gloo world on CPU for multi-rank tests."""

import os
import socket
import traceback

import torch.multiprocessing as mp


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _entry(rank, world, port, fn, args, errq):
    os.environ.update({"MASTER_ADDR": "127.0.0.1", "MASTER_PORT": str(port), "RANK": str(rank),
                       "WORLD_SIZE": str(world), "LOCAL_RANK": str(rank)})
    try:
        fn(rank, world, *args)
    except BaseException:  # noqa: BLE001 - reported to the parent
        errq.put((rank, traceback.format_exc()))
        raise


def run_world(world: int, fn, *args, timeout: float = 300.0) -> None:
    ctx = mp.get_context("spawn")
    errq = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_entry, args=(r, world, port, fn, args, errq)) for r in range(world)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(timeout)
    alive = [p for p in procs if p.is_alive()]
    for p in alive:
        p.kill()
    errors = []
    while not errq.empty():
        errors.append(errq.get())
    if errors:
        raise AssertionError("\n".join(f"rank {r}:\n{tb}" for r, tb in errors))
    if alive:
        raise AssertionError(f"{len(alive)} rank(s) timed out")
    bad = [p.exitcode for p in procs if p.exitcode != 0]
    if bad:
        raise AssertionError(f"ranks exited with {bad}")
