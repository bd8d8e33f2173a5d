"""Record GPU memory / utilisation while a run is going (read-only queries).

    python -m graspo_b200.analysis.gpu_memory --gpus 0,1 --output-dir OUTPUT_DIR/gpu_memory \
        [--interval-sec 2] [--duration-sec N] [--tag NAME]

Samples ``nvidia-smi --query-gpu`` (index, uuid, memory used / free / total,
utilisation, temperature, power) every interval into ``gpu_memory.jsonl`` and
writes ``gpu_memory_summary.json`` (peak / p95 / mean memory, mean
utilisation per GPU) when stopped (SIGINT / SIGTERM or the duration).  It only
reads device state; it changes no GPU setting.  Reference behaviour:
scripts/record_gpu_memory.py:27-83.
"""

from __future__ import annotations

import argparse
import json
import signal
import subprocess
import time
from collections.abc import Callable
from datetime import datetime, timezone
from pathlib import Path
from statistics import mean
from typing import Any

FIELDS = ("index", "uuid", "memory.used", "memory.free", "memory.total", "utilization.gpu", "temperature.gpu",
          "power.draw")
KEYS = ("gpu_index", "gpu_uuid", "memory_used_mib", "memory_free_mib", "memory_total_mib", "utilization_gpu_pct",
        "temperature_c", "power_w")


def _num(text: str) -> float | None:
    try:
        return float(text)
    except ValueError:
        return None


def parse_query_csv(text: str) -> list[dict[str, Any]]:
    """Rows of ``nvidia-smi --query-gpu=<FIELDS> --format=csv,noheader,nounits``."""
    rows = []
    for line in text.splitlines():
        parts = [p.strip() for p in line.split(",")]
        if len(parts) != len(FIELDS):
            continue
        row: dict[str, Any] = {"gpu_index": parts[0], "gpu_uuid": parts[1]}
        for key, val in zip(KEYS[2:], parts[2:], strict=True):
            row[key] = _num(val)
        rows.append(row)
    return rows


def query_nvidia_smi(gpus: list[str]) -> list[dict[str, Any]]:
    cmd = ["nvidia-smi", f"--query-gpu={','.join(FIELDS)}", "--format=csv,noheader,nounits"]
    if gpus:
        cmd.append(f"--id={','.join(gpus)}")
    out = subprocess.run(cmd, capture_output=True, text=True, timeout=30, check=False)
    return parse_query_csv(out.stdout) if out.returncode == 0 else []


def _p95(values: list[float]) -> float:
    ordered = sorted(values)
    return ordered[min(len(ordered) - 1, int(round(0.95 * (len(ordered) - 1))))]


def summarize_samples(samples: list[dict[str, Any]]) -> dict[str, Any]:
    by_gpu: dict[str, list[dict[str, Any]]] = {}
    for row in samples:
        by_gpu.setdefault(str(row.get("gpu_index")), []).append(row)
    per_gpu = {}
    for gpu, rows in sorted(by_gpu.items()):
        mem = [float(r["memory_used_mib"]) for r in rows if r.get("memory_used_mib") is not None]
        util = [float(r["utilization_gpu_pct"]) for r in rows if r.get("utilization_gpu_pct") is not None]
        per_gpu[gpu] = {
            "samples": len(rows),
            "memory_used_mib_peak": max(mem) if mem else None,
            "memory_used_mib_p95": _p95(mem) if mem else None,
            "memory_used_mib_mean": mean(mem) if mem else None,
            "utilization_gpu_pct_mean": mean(util) if util else None,
        }
    return {"sample_count": len(samples), "per_gpu": per_gpu}


def record(output_dir: str | Path, *, gpus: list[str], interval_sec: float = 2.0, duration_sec: float | None = None,
           tag: str = "", query: Callable[[list[str]], list[dict[str, Any]]] = query_nvidia_smi,
           stop: Callable[[], bool] | None = None) -> dict[str, Any]:
    out = Path(output_dir)
    out.mkdir(parents=True, exist_ok=True)
    rows_path = out / "gpu_memory.jsonl"
    samples: list[dict[str, Any]] = []
    started = time.monotonic()
    with rows_path.open("a", encoding="utf-8") as fh:
        while not (stop is not None and stop()):
            stamp = datetime.now(timezone.utc).isoformat(timespec="seconds")
            for row in query(gpus):
                row.update(timestamp=stamp, tag=tag)
                samples.append(row)
                fh.write(json.dumps(row) + "\n")
            fh.flush()
            if duration_sec is not None and time.monotonic() - started >= duration_sec:
                break
            time.sleep(interval_sec)
    summary = summarize_samples(samples)
    summary.update(tag=tag, gpus=gpus, interval_sec=interval_sec)
    (out / "gpu_memory_summary.json").write_text(json.dumps(summary, indent=2) + "\n", encoding="utf-8")
    return summary


def main(argv: list[str] | None = None) -> int:
    p = argparse.ArgumentParser(description="Record GPU memory / utilisation to JSONL (read-only).")
    p.add_argument("--gpus", default="0")
    p.add_argument("--output-dir", required=True)
    p.add_argument("--interval-sec", type=float, default=2.0)
    p.add_argument("--duration-sec", type=float, default=None)
    p.add_argument("--tag", default="")
    args = p.parse_args(argv)
    flag = {"stop": False}
    for sig in (signal.SIGINT, signal.SIGTERM):
        signal.signal(sig, lambda *_: flag.__setitem__("stop", True))
    gpus = [g.strip() for g in args.gpus.split(",") if g.strip()]
    record(args.output_dir, gpus=gpus, interval_sec=args.interval_sec, duration_sec=args.duration_sec, tag=args.tag,
           stop=lambda: flag["stop"])
    return 0


if __name__ == "__main__":
    raise SystemExit(main())
