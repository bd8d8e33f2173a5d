"""Prompt rendering helpers that only need a tokenizer's public interface."""

from __future__ import annotations

import json
from typing import Any


def ensure_tokenizer_ready(tokenizer: Any) -> None:
    """Left padding, with EOS standing in for a missing pad token."""
    if tokenizer.pad_token_id is None:
        tokenizer.pad_token = tokenizer.eos_token
    if tokenizer.pad_token_id is None:
        raise ValueError("Tokenizer has no pad_token_id or eos_token_id")
    tokenizer.padding_side = "left"


def render_messages(
    tokenizer: Any,
    messages: list[dict[str, Any]],
    chat_template_kwargs: dict[str, Any] | None = None,
    *,
    tools: list[dict[str, Any]] | None = None,
) -> str:
    """Chat-template rendering with a generation prompt; plain text fallback.

    Without a chat template the prompt is ``role: content`` paragraphs followed
    by the tools as JSON (reference: transformer_adapter.py:255-291).
    """
    kwargs = dict(chat_template_kwargs or {})
    if tools is not None:
        kwargs["tools"] = tools
    if getattr(tokenizer, "chat_template", None):
        return tokenizer.apply_chat_template(
            messages, tokenize=False, add_generation_prompt=True, **kwargs
        )
    text = "\n\n".join(f"{m.get('role', 'user')}: {m.get('content', '')}" for m in messages)
    if tools is not None:
        text += "\n\ntools: " + json.dumps(tools, ensure_ascii=False)
    return text
