"""Rule-based structured reward for JSON-answer and tool-call completions.

Scoring (reference: src/graspo/core/reward.py:56-295; the numbers must match so
reward curves stay comparable across frameworks):

* The expected layout is a sequence of literal markers with one content slot:
  optional ``<think>`` .. ``</think>`` then, for a JSON target, ``` ```json ``` ..
  ```` ``` ```` around the answer (or the bare answer when fences are off).
  Markers are located left to right; each found marker earns
  ``marker_reward_weight``.  A missing marker stops the scan and discards any
  extracted content.
* Text outside the markers is "useless"; it earns
  ``anti_useless_str_reward_weight / 2**(len/anti_useless_str_half_reward_len)``.
* Valid JSON in the answer slot earns another marker weight; if the useless text
  is short enough and the JSON is an object, the best of the targets by
  ``dict_compare_score`` adds ``content_reward_weight * dcs`` and, when every
  non-numeric item matched, one more ``content_reward_weight``.
* The reward is ``raw / max`` where ``max`` counts markers and
  ``2*content + marker`` per slot; the anti-useless bonus is not in ``max``, so
  a perfect clean answer scores slightly above 1.0.
* Tool-call completions use parsed tool calls instead of the marker scan.
"""

from __future__ import annotations

import json
import math
from typing import Any

from pydantic import BaseModel, ConfigDict

from graspo_b200.core.compare import dict_compare_score
from graspo_b200.core.completion import ParsedCompletion, raw_parsed_completion


class RewardConfig(BaseModel):
    model_config = ConfigDict(extra="forbid")

    check_think: bool = False
    check_json_markdown: bool = True
    check_list_order: bool = False
    marker_reward_weight: float = 10.0
    content_reward_weight: float = 100.0
    anti_useless_str_reward_weight: float = 1.0
    anti_useless_str_half_reward_len: int = 100


class RewardResult(BaseModel):
    model_config = ConfigDict(extra="forbid", frozen=True)

    reward: float
    content_score: float
    base_content_score: float
    all_right: bool
    extracted: dict[str, Any]
    useless_text: str
    raw_score: float
    max_score: float
    matched_target_index: int | None = None
    matched_target_id: str | None = None
    target_scores: list[dict[str, Any]] | None = None


# --------------------------------------------------------------------------
# target normalisation
# --------------------------------------------------------------------------


def is_valid_json(text: str) -> bool:
    try:
        json.loads(text)
    except (TypeError, ValueError):
        return False
    return True


def normalize_tool_calls(value: Any, *, path: str = "tool_calls") -> list[dict[str, Any]]:
    """Validate a canonical ``[{"name": str, "arguments": {...}}, ...]`` list."""
    if not isinstance(value, list) or not value:
        raise ValueError(f"{path} must be a non-empty list")
    calls = []
    for i, call in enumerate(value):
        if not isinstance(call, dict):
            raise ValueError(f"{path}[{i}] must be a JSON object")
        name, args = call.get("name"), call.get("arguments")
        if not isinstance(name, str) or not name:
            raise ValueError(f"{path}[{i}].name must be a non-empty string")
        if not isinstance(args, dict):
            raise ValueError(f"{path}[{i}].arguments must be a JSON object")
        calls.append({"name": name, "arguments": dict(args)})
    return calls


def normalize_targets(value: Any) -> list[dict[str, Any]]:
    """Validate ``targets`` and return ``[{"id", "output": {content?, tool_calls?}}]``."""
    if not isinstance(value, list) or not value:
        raise ValueError("targets must be a non-empty list")
    out = []
    for i, target in enumerate(value):
        if not isinstance(target, dict):
            raise ValueError(f"targets[{i}] must be a JSON object")
        target_id = target.get("id")
        if target_id is not None and not isinstance(target_id, str):
            raise ValueError(f"targets[{i}].id must be a string when provided")
        output = target.get("output")
        if not isinstance(output, dict):
            raise ValueError(f"targets[{i}].output must be a JSON object")
        norm: dict[str, Any] = {}
        if "content" in output:
            if not isinstance(output["content"], dict):
                raise ValueError(f"targets[{i}].output.content must be a JSON object")
            norm["content"] = dict(output["content"])
        if "tool_calls" in output:
            norm["tool_calls"] = normalize_tool_calls(
                output["tool_calls"], path=f"targets[{i}].output.tool_calls"
            )
        if not norm:
            raise ValueError(f"targets[{i}].output must contain content and/or non-empty tool_calls")
        out.append({"id": target_id, "output": norm})
    return out


def empty_target_score(target: dict[str, Any], index: int) -> dict[str, Any]:
    return {
        "target_index": index,
        "target_id": target.get("id"),
        "content_score": 0.0,
        "base_content_score": 0.0,
        "all_right": False,
    }


# --------------------------------------------------------------------------
# scorer
# --------------------------------------------------------------------------

_SLOT = ("slot", "answer")  # a content slot in the layout
_GAP = None  # free text between two marker groups


class GraspoReward:
    def __init__(self, config: RewardConfig | None = None) -> None:
        self.config = config or RewardConfig()

    # -- layout ----------------------------------------------------------
    def _layout(self, has_answer: bool) -> list[Any]:
        items: list[Any] = []
        if self.config.check_think:
            items += ["<think>", _GAP, "</think>"]
        if has_answer:
            if items:
                items.append(_GAP)
            if self.config.check_json_markdown:
                items += ["```json", _SLOT, "```"]
            else:
                items.append(_SLOT)
        return items

    def _max_reward(self, layout: list[Any]) -> float:
        cfg = self.config
        total = 0.0
        for item in layout:
            if isinstance(item, str):
                total += cfg.marker_reward_weight
            elif item is not None:
                total += 2 * cfg.content_reward_weight + cfg.marker_reward_weight
        return total

    def _useless_text_score(self, text: str) -> float:
        cfg = self.config
        return cfg.anti_useless_str_reward_weight / math.pow(
            2, len(text) / cfg.anti_useless_str_half_reward_len
        )

    @staticmethod
    def _best_of(scores: list[dict[str, Any]]) -> dict[str, Any] | None:
        best = None
        for entry in scores:
            if "_scored" not in entry:
                continue
            if best is None or entry["content_score"] > best["content_score"]:
                best = entry
        return best

    def _result(
        self,
        *,
        raw: float,
        max_score: float,
        best: dict[str, Any] | None,
        content: float,
        base: float,
        all_right: bool,
        extracted: dict[str, Any],
        useless: str,
        scores: list[dict[str, Any]],
    ) -> RewardResult:
        matched = best is not None and content > 0
        for entry in scores:
            entry.pop("_scored", None)
        return RewardResult(
            reward=raw / max_score if max_score else 0.0,
            content_score=content,
            base_content_score=base,
            all_right=all_right,
            extracted=extracted,
            useless_text=useless,
            raw_score=raw,
            max_score=max_score,
            matched_target_index=int(best["target_index"]) if matched else None,
            matched_target_id=(
                str(best["target_id"]) if matched and best.get("target_id") is not None else None
            ),
            target_scores=scores,
        )

    # -- JSON answer path -------------------------------------------------
    def score(self, completion: str, targets: Any) -> RewardResult:
        cfg = self.config
        normalized = normalize_targets(targets)
        has_answer = any("content" in t["output"] for t in normalized)
        layout = self._layout(has_answer)
        max_score = self._max_reward(layout)

        raw = 0.0
        extracted: dict[str, str] = {}
        useless = ""
        cursor = 0
        open_slot: str | None = None
        for item in layout:
            if isinstance(item, str):
                hit = completion.find(item, cursor)
                if hit < 0:
                    extracted.clear()
                    break
                raw += cfg.marker_reward_weight
                if open_slot is None:
                    useless += completion[cursor:hit]
                else:
                    extracted[open_slot] = completion[cursor:hit]
                cursor = hit + len(item)
                open_slot = None
            else:
                open_slot = None if item is None else item[1]
        if open_slot is None:
            useless += completion[cursor:]
        else:
            extracted[open_slot] = completion[cursor:]

        scores = [empty_target_score(t, i) for i, t in enumerate(normalized)]
        content = base = 0.0
        all_right = False
        best = None
        answer = extracted.get("answer") if has_answer else None
        if answer is not None:
            text = answer.strip()
            if is_valid_json(text):
                raw += cfg.marker_reward_weight
                parsed = json.loads(text)
                if len(useless) <= cfg.anti_useless_str_half_reward_len and isinstance(parsed, dict):
                    for entry in scores:
                        want = normalized[entry["target_index"]]["output"].get("content")
                        if not isinstance(want, dict):
                            continue
                        res = dict_compare_score(parsed, want, cfg.check_list_order)
                        entry.update(
                            content_score=res.dcs,
                            base_content_score=res.base_dcs,
                            all_right=res.all_right,
                            _scored=True,
                        )
                    best = self._best_of(scores)
                    if best is not None:
                        content = float(best["content_score"])
                        base = float(best["base_content_score"])
                        raw += content * cfg.content_reward_weight
                        if best["all_right"]:
                            raw += cfg.content_reward_weight
                            all_right = True
        raw += self._useless_text_score(useless)
        return self._result(
            raw=raw,
            max_score=max_score,
            best=best,
            content=content,
            base=base,
            all_right=all_right,
            extracted=dict(extracted),
            useless=useless,
            scores=scores,
        )

    # -- tool-call path ---------------------------------------------------
    def _think_marker_score(self, text: str) -> tuple[float, bool]:
        if not self.config.check_think:
            return 0.0, True
        start = text.find("<think>")
        if start >= 0 and text.find("</think>", start + len("<think>")) >= 0:
            return 2 * self.config.marker_reward_weight, True
        return 0.0, False

    def _tool_call_max_reward(self) -> float:
        cfg = self.config
        total = 2 * cfg.content_reward_weight + cfg.marker_reward_weight
        if cfg.check_think:
            total += 2 * cfg.marker_reward_weight
        return total

    def score_parsed(
        self,
        parsed: ParsedCompletion | str,
        targets: Any,
        *,
        is_tool_call: bool = False,
    ) -> RewardResult:
        if isinstance(parsed, str):
            parsed = raw_parsed_completion(parsed)
        if not is_tool_call:
            return self.score(parsed.raw_text, targets)
        cfg = self.config
        normalized = normalize_targets(targets)
        raw, think_ok = self._think_marker_score(parsed.raw_text)
        scores = [empty_target_score(t, i) for i, t in enumerate(normalized)]
        content = base = 0.0
        all_right = False
        best = None
        if parsed.tool_calls and think_ok:
            raw += cfg.marker_reward_weight
            if len(parsed.extra_text) <= cfg.anti_useless_str_half_reward_len:
                got = {"tool_calls": parsed.tool_calls}
                for entry in scores:
                    calls = normalized[entry["target_index"]]["output"].get("tool_calls")
                    if not isinstance(calls, list):
                        continue
                    res = dict_compare_score(got, {"tool_calls": calls}, True)
                    entry.update(
                        content_score=res.dcs,
                        base_content_score=res.base_dcs,
                        all_right=res.all_right and not parsed.parse_errors,
                        _scored=True,
                    )
                best = self._best_of(scores)
                if best is not None:
                    content = float(best["content_score"])
                    base = float(best["base_content_score"])
                raw += content * cfg.content_reward_weight
                all_right = bool(best and best["all_right"])
                if all_right:
                    raw += cfg.content_reward_weight
        raw += self._useless_text_score(parsed.extra_text)
        return self._result(
            raw=raw,
            max_score=self._tool_call_max_reward(),
            best=best,
            content=content,
            base=base,
            all_right=all_right,
            extracted={
                "tool_calls": parsed.tool_calls,
                "think": parsed.think_text,
                "answer": parsed.answer_text,
                "parser": parsed.parser_name,
                "parse_errors": parsed.parse_errors,
                "extra_text": parsed.extra_text,
            },
            useless=parsed.extra_text,
            scores=scores,
        )
