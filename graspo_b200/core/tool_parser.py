"""Parse Qwen-style tool calls out of a completion.

Recognised forms (reference: src/graspo/backends/graspoflow/tool_parser.py:14-180):

* ``<think>...</think>`` blocks are collected as think text.
* ``<tool_call>BODY</tool_call>`` where BODY is canonical JSON
  (``{"name", "arguments"}`` or a list of them) or Qwen XML
  ``<function=NAME><parameter=KEY>VALUE</parameter>...</function>``.
* A bare ``<function=...>`` outside any ``<tool_call>`` wrapper, used only when
  no wrapped call parsed.

XML values are strings unless the declared tool schema says ``integer``,
``number`` or ``boolean``; a value that does not fit its declared type is kept
as text and recorded in ``parse_errors``.  Whatever remains after removing the
think, tool-call and function blocks is ``extra_text``.
"""

from __future__ import annotations

import json
import math
import re
from typing import Any

from graspo_b200.core.completion import ParsedCompletion

_THINK = re.compile(r"<think>(.*?)</think>", re.DOTALL)
_CALL = re.compile(r"<tool_call>(.*?)</tool_call>", re.DOTALL)
_FUNC = re.compile(r"<function=([^>\n]+)>(.*?)</function>", re.DOTALL)
_PARAM = re.compile(r"<parameter=([^>\n]+)>(.*?)</parameter>", re.DOTALL)
_INT = re.compile(r"[+-]?\d+")


def canonical_tool_call(value: Any) -> dict[str, Any] | None:
    if not isinstance(value, dict):
        return None
    name, args = value.get("name"), value.get("arguments")
    if not isinstance(name, str) or not isinstance(args, dict):
        return None
    return {"name": name, "arguments": dict(args)}


def try_parse_json_tool_call(text: str) -> list[dict[str, Any]] | None:
    """Canonical JSON body -> list of calls, or None when it is not one."""
    try:
        value = json.loads(text)
    except (TypeError, ValueError):
        return None
    calls = []
    for item in value if isinstance(value, list) else [value]:
        call = canonical_tool_call(item)
        if call is None:
            return None
        calls.append(call)
    return calls


def tool_argument_schema_type(
    tools: list[dict[str, Any]] | None, tool_name: str, param_name: str
) -> str | None:
    """JSON-schema type declared for ``tool_name(param_name)`` (first non-null)."""
    for tool in tools or []:
        fn = tool.get("function") if isinstance(tool, dict) else None
        if not isinstance(fn, dict) or fn.get("name") != tool_name:
            continue
        params = fn.get("parameters")
        props = params.get("properties") if isinstance(params, dict) else None
        spec = props.get(param_name) if isinstance(props, dict) else None
        if not isinstance(spec, dict):
            return None
        kind = spec.get("type")
        if isinstance(kind, str):
            return kind
        if isinstance(kind, list):
            return next((k for k in kind if isinstance(k, str) and k != "null"), None)
        return None
    return None


def coerce_xml_tool_argument(
    tool_name: str,
    param_name: str,
    raw_value: str,
    *,
    tools: list[dict[str, Any]] | None,
) -> tuple[Any, str | None]:
    kind = tool_argument_schema_type(tools, tool_name, param_name)
    if kind == "integer":
        return (int(raw_value), None) if _INT.fullmatch(raw_value) else (raw_value, "expected integer")
    if kind == "number":
        try:
            number = float(raw_value)
        except ValueError:
            return raw_value, "expected number"
        return (number, None) if math.isfinite(number) else (raw_value, "expected finite number")
    if kind == "boolean":
        lowered = raw_value.lower()
        if lowered in ("true", "false"):
            return lowered == "true", None
        return raw_value, "expected boolean"
    return raw_value, None


def try_parse_qwen_xml_tool_call(
    text: str,
    *,
    tools: list[dict[str, Any]] | None = None,
    error_prefix: str = "tool_call",
) -> tuple[list[dict[str, Any]], list[str]]:
    calls: list[dict[str, Any]] = []
    errors: list[str] = []
    for fn in _FUNC.finditer(text):
        name = fn.group(1).strip()
        args: dict[str, Any] = {}
        for param in _PARAM.finditer(fn.group(2)):
            key = param.group(1).strip()
            value, err = coerce_xml_tool_argument(name, key, param.group(2).strip(), tools=tools)
            args[key] = value
            if err:
                errors.append(f"{error_prefix}.arguments.{key} {err}")
        if name and args:
            calls.append({"name": name, "arguments": args})
    return calls, errors


def parse_qwen_tool_completion(
    text: str,
    *,
    expect_tool_calls: bool = False,
    tools: list[dict[str, Any]] | None = None,
) -> ParsedCompletion:
    think = [m.group(1).strip() for m in _THINK.finditer(text)]
    calls: list[dict[str, Any]] = []
    errors: list[str] = []
    parsers: set[str] = set()
    for idx, wrapped in enumerate(_CALL.finditer(text)):
        body = wrapped.group(1).strip()
        as_json = try_parse_json_tool_call(body)
        if as_json is not None:
            calls += as_json
            parsers.add("qwen_json_tool_call")
            continue
        as_xml, xml_errors = try_parse_qwen_xml_tool_call(
            body, tools=tools, error_prefix=f"tool_call[{idx}]"
        )
        if as_xml:
            calls += as_xml
            errors += xml_errors
            parsers.add("qwen_xml_tool_call")
        else:
            errors.append(f"tool_call[{idx}] is neither canonical JSON nor Qwen XML")
    if not calls and "<function=" in text:
        as_xml, xml_errors = try_parse_qwen_xml_tool_call(
            _THINK.sub("", text), tools=tools, error_prefix="tool_call"
        )
        if as_xml:
            calls += as_xml
            errors += xml_errors
            parsers.add("qwen_xml_tool_call_unwrapped")
    if expect_tool_calls and not calls:
        errors.append("no tool call found")
    extra = _FUNC.sub("", _CALL.sub("", _THINK.sub("", text))).strip()
    return ParsedCompletion(
        raw_text=text,
        think_text="\n\n".join(part for part in think if part),
        tool_calls=calls,
        answer_text=extra or text,
        parser_name="+".join(sorted(parsers)) if parsers else "qwen_tool_call",
        parse_errors=errors,
        extra_text=extra,
    )
