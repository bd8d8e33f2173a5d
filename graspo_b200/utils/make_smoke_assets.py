"""Create the tiny random-init model and the 16-record JSONL of the CPU smoke config.

    python -m graspo_b200.utils.make_smoke_assets <dir>
"""

from __future__ import annotations

import sys
from pathlib import Path

from graspo_b200.utils.synth import TINY, synthetic_json_records, write_jsonl_records, write_qwen3_checkpoint


def make(root: str | Path) -> Path:
    root = Path(root)
    write_qwen3_checkpoint(root / "tiny-qwen3", TINY, seed=0, device="cpu", dtype=__import__("torch").float32)
    write_jsonl_records(synthetic_json_records(16, seed=0), root / "train.jsonl")
    return root


if __name__ == "__main__":
    print(make(sys.argv[1] if len(sys.argv) > 1 else "outputs/smoke_assets"))
