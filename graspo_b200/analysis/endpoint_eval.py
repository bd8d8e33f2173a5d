"""Score a served model through an OpenAI-compatible chat-completions endpoint.

    python -m graspo_b200.analysis.endpoint_eval --config run.yaml --data eval.jsonl \
        --base-url http://127.0.0.1:8000/v1 --model NAME --output-dir OUT \
        [--samples-per-prompt K] [--limit N] [--temperature T] [--top-p P] [--max-tokens M] \
        [--seed S] [--chat-template-kwargs JSON] [--timeout SEC]

For each record the messages (image parts become ``image_url`` parts with
base64 data URLs; relative paths resolve against the JSONL's folder) and the
record's tools go to ``<base-url>/chat/completions``, one request per
completion with seed ``S + k``.  A reply's structured ``tool_calls`` are
scored as the tool calls; otherwise its text goes through the Qwen tool-call
parser.  Scores use the run's reward; ``completions.jsonl`` and
``summary.json`` have the same layout as the native evaluator's.
Reference behaviour: scripts/evaluate_vllm_reward.py, scripts/vllm_eval.py.
"""

from __future__ import annotations

import argparse
import base64
import json
import mimetypes
import time
import urllib.error
import urllib.request
from pathlib import Path
from typing import Any

from graspo_b200.analysis.scoring import score_row, summarize, write_report
from graspo_b200.core.completion import ParsedCompletion
from graspo_b200.core.reward import GraspoReward
from graspo_b200.core.tool_parser import parse_qwen_tool_completion


def _image_url(part: dict[str, Any], base_dir: Path) -> dict[str, Any]:
    ref = part.get("image") or part.get("path") or part.get("url")
    if isinstance(part.get("image_url"), dict):
        ref = part["image_url"].get("url") or ref
    if not isinstance(ref, str):
        return dict(part)
    if not ref.startswith(("data:", "http://", "https://")):
        path = Path(ref) if Path(ref).is_absolute() else base_dir / ref
        mime = mimetypes.guess_type(path.name)[0] or "image/png"
        ref = f"data:{mime};base64,{base64.b64encode(path.read_bytes()).decode('ascii')}"
    return {"type": "image_url", "image_url": {"url": ref}}


def openai_messages(messages: list[dict[str, Any]], base_dir: Path) -> list[dict[str, Any]]:
    """Record messages in the chat-completions wire format."""
    out = []
    for msg in messages:
        item = dict(msg)
        if isinstance(item.get("content"), list):
            item["content"] = [
                _image_url(p, base_dir) if isinstance(p, dict) and str(p.get("type", "")).lower() in ("image", "image_url")
                else p
                for p in item["content"]
            ]
        out.append(item)
    return out


class EndpointClient:
    """Minimal client of ``POST <base_url>/chat/completions``."""

    def __init__(self, base_url: str, model: str, *, timeout: float = 600.0, api_key: str = "none") -> None:
        self.url = base_url.rstrip("/") + "/chat/completions"
        self.model, self.timeout, self.api_key = model, float(timeout), api_key

    def chat(self, messages, *, tools=None, **sampling) -> dict[str, Any]:
        body = {"model": self.model, "messages": messages, **{k: v for k, v in sampling.items() if v is not None}}
        if tools:
            body["tools"] = tools
        req = urllib.request.Request(self.url, data=json.dumps(body, ensure_ascii=False).encode("utf-8"),
                                     headers={"Content-Type": "application/json",
                                              "Authorization": f"Bearer {self.api_key}"}, method="POST")
        try:
            with urllib.request.urlopen(req, timeout=self.timeout) as resp:
                reply = json.loads(resp.read().decode("utf-8"))
        except urllib.error.HTTPError as exc:
            raise RuntimeError(f"endpoint returned HTTP {exc.code}: "
                               f"{exc.read().decode('utf-8', errors='replace')[:2000]}") from exc
        choices = reply.get("choices") or []
        if not choices:
            raise RuntimeError(f"endpoint reply has no choices: {str(reply)[:500]}")
        return choices[0].get("message") or {}


def parse_reply(message: dict[str, Any], sample) -> ParsedCompletion:
    """Structured tool calls of the reply when it has any, else the text parsed
    as a Qwen completion."""
    text = str(message.get("content") or "")
    calls = []
    for call in message.get("tool_calls") or []:
        fn = call.get("function") if isinstance(call, dict) else None
        if not isinstance(fn, dict) or not isinstance(fn.get("name"), str):
            continue
        args = fn.get("arguments")
        if isinstance(args, str):
            try:
                args = json.loads(args)
            except ValueError:
                args = None
        if isinstance(args, dict):
            calls.append({"name": fn["name"], "arguments": args})
    if calls:
        return ParsedCompletion(raw_text=text, tool_calls=calls, answer_text=text, parser_name="endpoint_tool_calls",
                                extra_text=text)
    return parse_qwen_tool_completion(text, expect_tool_calls=sample.expects_tool_calls, tools=sample.tools)


def evaluate_endpoint(config, samples: list, client: EndpointClient, output_dir: str | Path, *,
                      base_dir: Path, samples_per_prompt: int = 1, seed: int = 42,
                      chat_template_kwargs: dict | None = None) -> dict[str, Any]:
    tr = config.training
    reward = GraspoReward(config.reward)
    t0 = time.monotonic()
    rows = []
    for idx, sample in enumerate(samples):
        messages = openai_messages(sample.messages, base_dir)
        for k in range(max(1, int(samples_per_prompt))):
            extra = {"chat_template_kwargs": chat_template_kwargs} if chat_template_kwargs else {}
            message = client.chat(messages, tools=sample.tools, temperature=tr.temperature, top_p=tr.top_p,
                                  max_tokens=tr.max_new_tokens, seed=seed + k, **extra)
            rows.append(score_row(reward, parse_reply(message, sample), sample, sample_index=idx, completion_index=k))
    summary = summarize(rows, len(samples), base_url=client.url, model=client.model,
                        samples_per_prompt=int(samples_per_prompt), elapsed_sec=round(time.monotonic() - t0, 3))
    write_report(output_dir, rows, summary)
    return summary


def main(argv: list[str] | None = None) -> int:
    p = argparse.ArgumentParser(description="Score an OpenAI-compatible chat endpoint with the GRASPO reward.")
    p.add_argument("--config", required=True, help="run YAML (reward and sampling settings)")
    p.add_argument("--data", required=True)
    p.add_argument("--base-url", required=True, help="e.g. http://127.0.0.1:8000/v1")
    p.add_argument("--model", required=True)
    p.add_argument("--output-dir", required=True)
    p.add_argument("--samples-per-prompt", type=int, default=1)
    p.add_argument("--limit", type=int, default=0)
    p.add_argument("--temperature", type=float)
    p.add_argument("--top-p", type=float)
    p.add_argument("--max-tokens", type=int)
    p.add_argument("--seed", type=int, default=42)
    p.add_argument("--chat-template-kwargs", help="JSON object sent as chat_template_kwargs")
    p.add_argument("--timeout", type=float, default=600.0)
    args = p.parse_args(argv)

    from graspo_b200.core.data import load_jsonl
    from graspo_b200.core.schema import GraspoConfig

    config = GraspoConfig.from_yaml(args.config)
    for key, value in (("temperature", args.temperature), ("top_p", args.top_p), ("max_new_tokens", args.max_tokens)):
        if value is not None:
            setattr(config.training, key, value)
    samples = load_jsonl(args.data)
    if args.limit > 0:
        samples = samples[: args.limit]
    summary = evaluate_endpoint(
        config, samples, EndpointClient(args.base_url, args.model, timeout=args.timeout), args.output_dir,
        base_dir=Path(args.data).resolve().parent, samples_per_prompt=args.samples_per_prompt, seed=args.seed,
        chat_template_kwargs=json.loads(args.chat_template_kwargs) if args.chat_template_kwargs else None)
    print(json.dumps(summary, ensure_ascii=False))
    return 0


if __name__ == "__main__":
    raise SystemExit(main())
