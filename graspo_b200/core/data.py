"""JSONL data layer: strict record validation, media extraction, SFT targets.

Record format (reference: src/graspo/core/data.py:13-413)::

    {"messages": [{"role": ..., "content": ...}, ...],   # prompt/context only
     "tools": [{"type": "function", "function": {...}}], # optional
     "targets": [{"id": ..., "output": {"content": {...}} | {"tool_calls": [...]}}],
     ...extra keys become metadata}

Rejected: the removed fields ``prompt``/``image(s)``/``video(s)``/``ground_truth``,
a final assistant message (it would leak the answer), raw ``<tool_call>`` /
``<function=`` / ``<parameter=`` markers in assistant text, tool-call targets that
name undeclared tools, miss ``required`` arguments or break an ``enum``.
"""

from __future__ import annotations

import json
import re
from pathlib import Path
from typing import Any

from graspo_b200.core.reward import normalize_targets
from graspo_b200.core.schema import Sample

_RAW_TOOL_MARKER = re.compile(r"<(?:tool_call|function=|parameter=)")
_REMOVED_FIELDS = ("image", "images", "prompt", "video", "videos")


def sample_from_record(record: dict[str, Any]) -> Sample:
    removed = sorted(f for f in _REMOVED_FIELDS if f in record)
    if removed:
        raise ValueError(
            "removed input field(s): "
            + ", ".join(removed)
            + "; use messages + optional tools + targets JSONL"
        )
    if "ground_truth" in record:
        raise ValueError("record field 'ground_truth' was removed; use targets[].output")
    messages = _validate_messages(record.get("messages"))
    if "targets" not in record:
        raise ValueError("record must contain 'targets'")
    tools = _validate_tools(record.get("tools"))
    targets = normalize_targets(record["targets"])
    if tools is not None:
        _check_tool_call_targets(targets, tools)
    media: list[dict[str, Any]] = []
    seen: set[tuple[str, str]] = set()
    for message in messages:
        for item in content_to_text_and_media(message.get("content", ""))[1]:
            key = (str(item.get("type") or ""), str(item.get("path") or ""))
            if key not in seen:
                seen.add(key)
                media.append(item)
    metadata = {k: v for k, v in record.items() if k not in ("messages", "targets", "tools")}
    return Sample(messages=messages, targets=targets, tools=tools, metadata=metadata, media=media)


def _validate_messages(value: Any) -> list[dict[str, Any]]:
    if not isinstance(value, list) or not value:
        raise ValueError("record must contain a non-empty 'messages' list")
    messages = []
    for i, message in enumerate(value):
        if not isinstance(message, dict):
            raise ValueError(f"messages[{i}] must be an object")
        if not str(message.get("role") or "").strip():
            raise ValueError(f"messages[{i}].role is required")
        if "content" not in message:
            raise ValueError(f"messages[{i}].content is required")
        messages.append(dict(message))
    if str(messages[-1].get("role") or "").lower() == "assistant":
        raise ValueError("messages must be prompt/context only; final assistant messages leak the target")
    for i, message in enumerate(messages):
        if str(message.get("role") or "").lower() == "assistant":
            _check_assistant_message(i, message)
    return messages


def _assistant_texts(content: Any) -> list[str]:
    if isinstance(content, str):
        return [content]
    texts = []
    if isinstance(content, list):
        for block in content:
            if isinstance(block, str):
                texts.append(block)
            elif isinstance(block, dict) and str(block.get("type") or "").lower() == "text":
                texts.append(str(block.get("text") or ""))
    return texts


def _check_assistant_message(index: int, message: dict[str, Any]) -> None:
    for text in _assistant_texts(message.get("content", "")):
        if _RAW_TOOL_MARKER.search(text):
            raise ValueError(
                f"messages[{index}] (assistant) has raw tool-call text in content. "
                "Use the structured 'tool_calls' field instead: "
                '{"tool_calls": [{"name": "...", "arguments": {...}}]}. '
                f"Found in content: {text.strip()[:200]!r}"
            )
    calls = message.get("tool_calls")
    if calls is None:
        return
    path = f"messages[{index}].tool_calls"
    if not isinstance(calls, list) or not calls:
        raise ValueError(f"{path} must be a non-empty list")
    for j, call in enumerate(calls):
        if not isinstance(call, dict):
            raise ValueError(f"{path}[{j}] must be a JSON object")
        name, args = call.get("name"), call.get("arguments")
        if not isinstance(name, str) or not name.strip():
            raise ValueError(f"{path}[{j}].name must be a non-empty string")
        if not isinstance(args, dict):
            raise ValueError(f"{path}[{j}].arguments must be a JSON object")
        for key, val in args.items():
            if isinstance(val, str) and _RAW_TOOL_MARKER.search(val):
                raise ValueError(
                    f"{path}[{j}].arguments.{key} contains raw tool-call markers in its string "
                    f"value; use structured JSON values instead: {val!r}"
                )


def _validate_tools(value: Any) -> list[dict[str, Any]] | None:
    if value is None:
        return None
    if not isinstance(value, list):
        raise ValueError("record 'tools' must be a list of JSON objects")
    for i, tool in enumerate(value):
        if not isinstance(tool, dict):
            raise ValueError(f"tools[{i}] must be an object")
    return [dict(tool) for tool in value]


def _declared_function(tools: list[dict[str, Any]], name: str) -> dict[str, Any] | None:
    for tool in tools:
        fn = tool.get("function")
        if isinstance(fn, dict) and fn.get("name") == name:
            return fn
    return None


def _check_tool_call_targets(targets: list[dict[str, Any]], tools: list[dict[str, Any]]) -> None:
    declared = {
        str(tool["function"]["name"])
        for tool in tools
        if isinstance(tool.get("function"), dict) and tool["function"].get("name")
    }
    for t_idx, target in enumerate(targets):
        calls = target["output"].get("tool_calls")
        if not isinstance(calls, list):
            continue
        for call in calls:
            name = str(call["name"])
            if declared and name not in declared:
                raise ValueError(f"targets[{t_idx}].output.tool_calls name {name!r} is not declared in tools")
            fn = _declared_function(tools, name)
            params = fn.get("parameters") if fn is not None else None
            if not isinstance(params, dict):
                continue
            args = call["arguments"]
            required = params.get("required")
            if isinstance(required, list):
                missing = [str(k) for k in required if k not in args]
                if missing:
                    raise ValueError(
                        f"targets[{t_idx}].output.tool_calls missing required argument(s): "
                        + ", ".join(missing)
                    )
            props = params.get("properties")
            if not isinstance(props, dict):
                continue
            for key, val in args.items():
                spec = props.get(key)
                allowed = spec.get("enum") if isinstance(spec, dict) else None
                if isinstance(allowed, list) and val not in allowed:
                    raise ValueError(
                        f"targets[{t_idx}].output.tool_calls argument {key!r} value {val!r} is not in enum"
                    )


def _media_path(item: dict[str, Any], kind: str) -> str | None:
    path = item.get(kind) or item.get("path") or item.get("url")
    nested = item.get(f"{kind}_url")
    if isinstance(nested, dict):
        path = nested.get("url") or path
    return str(path) if path else None


def content_to_text_and_media(content: Any) -> tuple[str, list[dict[str, Any]]]:
    """Flatten message content to text; images/videos become placeholders + refs."""
    if isinstance(content, str):
        return content, []
    if not isinstance(content, list):
        return str(content or ""), []
    parts: list[str] = []
    media: list[dict[str, Any]] = []
    for item in content:
        if not isinstance(item, dict):
            parts.append(str(item))
            continue
        kind = str(item.get("type") or "").lower()
        if kind == "text":
            parts.append(str(item.get("text") or ""))
        elif kind in ("image", "image_url", "video", "video_url"):
            base = kind.split("_")[0]
            path = _media_path(item, base)
            if path:
                media.append({"type": base, "path": path})
            parts.append(f"<{base}>")
        else:
            raise ValueError(f"unsupported multimodal content type: {kind!r}")
    return "\n".join(p for p in parts if p), media


def load_jsonl(path: str | Path) -> list[Sample]:
    samples = []
    with Path(path).open("r", encoding="utf-8") as handle:
        for line_no, line in enumerate(handle, start=1):
            if not line.strip():
                continue
            try:
                samples.append(sample_from_record(json.loads(line)))
            except Exception as exc:  # noqa: BLE001 - re-raised with location
                raise ValueError(f"invalid JSONL record at {path}:{line_no}: {exc}") from exc
    return samples


def sample_to_record(sample: Sample) -> dict[str, Any]:
    """The JSONL record that ``sample_from_record`` turns back into ``sample``:
    metadata keys return to the top level and media (derived from the
    messages) is not written."""
    record: dict[str, Any] = {"messages": sample.messages, "targets": sample.targets}
    if sample.tools is not None:
        record["tools"] = sample.tools
    record.update(sample.metadata or {})
    return record


def write_jsonl(samples: list[Sample], path: str | Path) -> None:
    out = Path(path)
    out.parent.mkdir(parents=True, exist_ok=True)
    with out.open("w", encoding="utf-8") as handle:
        for sample in samples:
            handle.write(json.dumps(sample_to_record(sample), ensure_ascii=False) + "\n")


# --------------------------------------------------------------------------
# SFT
# --------------------------------------------------------------------------


def _xml_value(value: Any) -> str:
    if isinstance(value, bool):
        return "true" if value else "false"
    if isinstance(value, float) and value == value and value == int(value):
        return str(int(value))
    return str(value)


def build_sft_target_text(target_output: dict[str, Any]) -> str:
    """Text the model should produce for a target: Qwen XML tool calls or fenced JSON."""
    calls = target_output.get("tool_calls")
    if isinstance(calls, list) and calls:
        blocks = []
        for call in calls:
            params = "".join(
                f"<parameter={k}>{_xml_value(v)}</parameter>" for k, v in call["arguments"].items()
            )
            blocks.append(f"<tool_call>\n<function={call['name']}>\n{params}\n</function>\n</tool_call>")
        return "\n".join(blocks)
    content = target_output.get("content")
    if isinstance(content, dict):
        return "```json\n" + json.dumps(content, ensure_ascii=False, indent=2) + "\n```"
    return ""


def sft_tokenize(
    sample: Sample,
    tokenizer: Any,
    *,
    max_seq_length: int = 4096,
    chat_template_kwargs: dict[str, Any] | None = None,
) -> dict[str, Any]:
    """Prompt (as rendered for rollout) + primary target + EOS; prompt labels = -100."""
    import torch

    target_text = build_sft_target_text(sample.targets[0]["output"])
    if not target_text:
        raise ValueError("primary target has no content or tool_calls")
    kwargs = dict(chat_template_kwargs or {})
    kwargs.setdefault("enable_thinking", False)
    if sample.expects_tool_calls and sample.tools is not None:
        kwargs["tools"] = sample.tools
    prompt = tokenizer.apply_chat_template(
        sample.messages, tokenize=False, add_generation_prompt=True, **kwargs
    )
    full_ids = tokenizer.encode(prompt + target_text + tokenizer.eos_token, add_special_tokens=False)
    prompt_ids = tokenizer.encode(prompt, add_special_tokens=False)
    full_ids = full_ids[:max_seq_length]
    prompt_len = min(len(prompt_ids), len(full_ids))
    labels = [-100] * prompt_len + full_ids[prompt_len:]
    input_ids = torch.tensor(full_ids, dtype=torch.long)
    out: dict[str, Any] = {
        "input_ids": input_ids,
        "labels": torch.tensor(labels, dtype=torch.long),
        "attention_mask": torch.ones_like(input_ids),
        "prompt_len": prompt_len,
        "metadata": dict(sample.metadata or {}),
    }
    if sample.media:
        out["_multimodal_row"] = {"messages": sample.messages, "tools": sample.tools, "media": sample.media}
        out["_target_text"] = target_text
    return out
