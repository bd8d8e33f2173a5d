"""The ``graspo`` standard-library logging channel (reference: ``logs/training.log``,
described at lines 491-513 of the reference project's own README).

Console output (INFO) on every rank; ``<output_dir>/logs/training.log`` (DEBUG)
on rank 0.  Calling it again for the same directory is harmless.
"""

from __future__ import annotations

import logging
import sys
from pathlib import Path

_FILE_HANDLERS: set[str] = set()


def setup_logging(output_dir: str | Path, *, rank: int = 0) -> logging.Logger:
    root = logging.getLogger("graspo")
    root.setLevel(logging.DEBUG)
    if not any(type(h) is logging.StreamHandler for h in root.handlers):
        console = logging.StreamHandler(sys.stdout)
        console.setLevel(logging.INFO)
        console.setFormatter(logging.Formatter("%(message)s"))
        root.addHandler(console)
    key = str(Path(output_dir).resolve())
    if rank == 0 and key not in _FILE_HANDLERS:
        log_dir = Path(output_dir) / "logs"
        log_dir.mkdir(parents=True, exist_ok=True)
        handler = logging.FileHandler(log_dir / "training.log", encoding="utf-8")
        handler.setLevel(logging.DEBUG)
        handler.setFormatter(
            logging.Formatter(
                "%(asctime)s [%(levelname)-5s] %(name)s: %(message)s", datefmt="%Y-%m-%d %H:%M:%S"
            )
        )
        root.addHandler(handler)
        _FILE_HANDLERS.add(key)
    return root
