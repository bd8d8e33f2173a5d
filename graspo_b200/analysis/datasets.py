"""Dataset helpers: a seeded train / eval split and a synthetic image dataset.

    python -m graspo_b200.analysis.datasets split SOURCE.jsonl --train OUT/train.jsonl \
        --eval OUT/eval.jsonl [--eval-count 48] [--seed 42]
    python -m graspo_b200.analysis.datasets synth-images OUT_DIR [--train-count 240] [--eval-count 80]

``split`` shuffles record lines with the seed, writes the first ``eval-count``
to the eval file and the rest to the train file, plus a manifest with the
counts and the seed (reference: scripts/split_train_eval_jsonl.sh).
``synth-images`` draws status-panel images (PIL) whose printed fields are the
JSON extraction target, in the messages / targets JSONL format with image
parts (reference: scripts/generate_synthetic_multimodal_dataset.py).
"""

from __future__ import annotations

import argparse
import json
import random
from pathlib import Path

STATUSES = ("ok", "warning", "failed", "pending")


def split_jsonl(source: str | Path, train: str | Path, eval_: str | Path, *, eval_count: int = 48,
                seed: int = 42, manifest: str | Path | None = None) -> dict:
    lines = [ln for ln in Path(source).read_text(encoding="utf-8").splitlines() if ln.strip()]
    if eval_count >= len(lines):
        raise ValueError(f"eval_count {eval_count} leaves no training records out of {len(lines)}")
    order = list(range(len(lines)))
    random.Random(seed).shuffle(order)
    ev, tr = sorted(order[:eval_count]), sorted(order[eval_count:])
    for path, idx in ((train, tr), (eval_, ev)):
        Path(path).parent.mkdir(parents=True, exist_ok=True)
        Path(path).write_text("".join(lines[i] + "\n" for i in idx), encoding="utf-8")
    info = {"source": str(source), "train": str(train), "eval": str(eval_), "train_count": len(tr),
            "eval_count": len(ev), "seed": seed, "eval_indices": ev}
    if manifest is not None:
        Path(manifest).write_text(json.dumps(info, indent=2) + "\n", encoding="utf-8")
    return info


def _panel(path: Path, values: dict, rng: random.Random) -> None:
    from PIL import Image, ImageDraw

    w, h = 320, 192
    bg = {"ok": (220, 245, 220), "warning": (250, 240, 200), "failed": (250, 215, 215), "pending": (225, 230, 245)}
    img = Image.new("RGB", (w, h), bg[values["status"]])
    d = ImageDraw.Draw(img)
    d.rectangle([4, 4, w - 5, h - 5], outline=(40, 40, 40), width=2)
    y = 16
    for key in ("ticket", "status", "priority", "count"):
        d.text((16, y), f"{key}: {values[key]}", fill=(0, 0, 0))
        y += 36
    for _ in range(rng.randint(2, 6)):  # clutter that is not part of the answer
        x0, y0 = rng.randint(200, 290), rng.randint(20, 160)
        d.ellipse([x0, y0, x0 + 12, y0 + 12], outline=(90, 90, 90))
    img.save(path)


def synth_image_records(out_dir: str | Path, *, train_count: int = 240, eval_count: int = 80,
                        seed: int = 20260606) -> dict:
    out = Path(out_dir)
    (out / "images").mkdir(parents=True, exist_ok=True)
    rng = random.Random(seed)
    rows = []
    for i in range(train_count + eval_count):
        status = rng.choice(STATUSES)
        values = {"ticket": f"T-{rng.randint(1000, 9999)}", "status": status,
                  "priority": "high" if status == "failed" else rng.choice(("low", "medium", "high")),
                  "count": rng.randint(0, 99)}
        img = out / "images" / f"panel_{i:05d}.png"
        _panel(img, values, rng)
        rows.append({
            "messages": [
                {"role": "system", "content": "Read the status panel and answer with one JSON object."},
                {"role": "user", "content": [{"type": "image", "image": str(img)},
                                             {"type": "text", "text": "Return ticket, status, priority and count."}]},
            ],
            "targets": [{"id": "panel", "output": {"content": values}}],
            "source": "synthetic_panel",
        })
    train, ev = rows[:train_count], rows[train_count:]
    for name, part in (("train.jsonl", train), ("eval.jsonl", ev)):
        (out / name).write_text("".join(json.dumps(r) + "\n" for r in part), encoding="utf-8")
    return {"train": str(out / "train.jsonl"), "eval": str(out / "eval.jsonl"), "train_count": len(train),
            "eval_count": len(ev)}


def main(argv: list[str] | None = None) -> int:
    p = argparse.ArgumentParser(description="Dataset helpers.")
    sub = p.add_subparsers(dest="cmd", required=True)
    sp = sub.add_parser("split")
    sp.add_argument("source")
    sp.add_argument("--train", required=True)
    sp.add_argument("--eval", required=True)
    sp.add_argument("--eval-count", type=int, default=48)
    sp.add_argument("--seed", type=int, default=42)
    sp.add_argument("--manifest")
    si = sub.add_parser("synth-images")
    si.add_argument("out_dir")
    si.add_argument("--train-count", type=int, default=240)
    si.add_argument("--eval-count", type=int, default=80)
    si.add_argument("--seed", type=int, default=20260606)
    args = p.parse_args(argv)
    if args.cmd == "split":
        info = split_jsonl(args.source, args.train, args.eval, eval_count=args.eval_count, seed=args.seed,
                           manifest=args.manifest)
    else:
        info = synth_image_records(args.out_dir, train_count=args.train_count, eval_count=args.eval_count,
                                   seed=args.seed)
    print(json.dumps({k: v for k, v in info.items() if k != "eval_indices"}))
    return 0


if __name__ == "__main__":
    raise SystemExit(main())
