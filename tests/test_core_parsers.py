"""Tool-call parser, parsed completions, replay buffer, LoRA target resolution,
prompt rendering, advantages and reward helpers (pure CPU).

Behaviour follows the reference: tool_parser.py:14-180, core/completion.py,
core/buffer.py:5-36, core/lora.py:10-85, core/graspo_parity.py (advantages),
core/reward.py (target / tool-call normalisation).
"""

from __future__ import annotations

import dataclasses
import math

import pytest

from graspo_b200.core.buffer import Experience, ReplayBuffer
from graspo_b200.core.chat_template import ensure_tokenizer_ready, render_messages
from graspo_b200.core.completion import ParsedCompletion, raw_parsed_completion
from graspo_b200.core.decisions import group_advantages, has_reward_variance, lower_median
from graspo_b200.core.lora_targets import (
    LORA_TARGET_PRESETS,
    lora_target_enabled,
    resolve_lora_target_modules,
)
from graspo_b200.core.reward import is_valid_json, normalize_targets, normalize_tool_calls
from graspo_b200.core.tool_parser import parse_qwen_tool_completion

TOOLS = [{"type": "function", "function": {"name": "book", "parameters": {"type": "object", "properties": {
    "seats": {"type": "integer"}, "price": {"type": "number"}, "vip": {"type": "boolean"},
    "note": {"type": ["null", "string"]}}}}}]


# ---------------------------------------------------------------- tool parser


def test_json_tool_calls_single_and_list():
    p = parse_qwen_tool_completion('<tool_call>{"name": "f", "arguments": {"a": 1}}</tool_call>')
    assert p.tool_calls == [{"name": "f", "arguments": {"a": 1}}] and p.parse_errors == []
    assert p.parser_name == "qwen_json_tool_call"
    text = ('<tool_call>[{"name": "f", "arguments": {}}, {"name": "g", "arguments": {"b": 2}}]</tool_call>\n'
            '<tool_call>{"name": "h", "arguments": {}}</tool_call>')
    assert [c["name"] for c in parse_qwen_tool_completion(text).tool_calls] == ["f", "g", "h"]


def test_no_tool_call():
    p = parse_qwen_tool_completion("plain answer")
    assert p.tool_calls == [] and p.parse_errors == [] and p.extra_text == "plain answer"
    missing = parse_qwen_tool_completion("plain answer", expect_tool_calls=True)
    assert missing.parse_errors == ["no tool call found"]


def test_think_blocks():
    p = parse_qwen_tool_completion("<think>step one</think>answer")
    assert p.think_text == "step one" and p.extra_text == "answer"
    multi = parse_qwen_tool_completion("<think>\nline 1\nline 2\n</think>\n<think>more</think>x")
    assert multi.think_text == "line 1\nline 2\n\nmore"


def test_extra_text_is_what_remains_outside_markers():
    p = parse_qwen_tool_completion('before <tool_call>{"name": "f", "arguments": {}}</tool_call> after')
    assert p.extra_text == "before  after"
    only_call = parse_qwen_tool_completion('  <tool_call>{"name": "f", "arguments": {}}</tool_call>\n ')
    assert only_call.extra_text == ""


def test_xml_tool_call_with_typed_parameters():
    text = ("<tool_call>\n<function=book>\n<parameter=seats>3</parameter>\n<parameter=price>9.5</parameter>\n"
            "<parameter=vip>TRUE</parameter>\n<parameter=note>window</parameter>\n</function>\n</tool_call>")
    p = parse_qwen_tool_completion(text, tools=TOOLS)
    assert p.tool_calls == [{"name": "book", "arguments": {"seats": 3, "price": 9.5, "vip": True, "note": "window"}}]
    assert p.parse_errors == [] and p.parser_name == "qwen_xml_tool_call"
    # without a schema every value stays text
    assert parse_qwen_tool_completion(text).tool_calls[0]["arguments"]["seats"] == "3"


@pytest.mark.parametrize("param, value, err", [("seats", "three", "expected integer"),
                                               ("price", "inf", "expected finite number"),
                                               ("price", "abc", "expected number"),
                                               ("vip", "yes", "expected boolean")])
def test_xml_values_that_break_their_type_are_kept_and_reported(param, value, err):
    text = f"<tool_call><function=book><parameter={param}>{value}</parameter></function></tool_call>"
    p = parse_qwen_tool_completion(text, tools=TOOLS)
    assert p.tool_calls[0]["arguments"][param] == value
    assert p.parse_errors == [f"tool_call[0].arguments.{param} {err}"]


def test_unwrapped_xml_function():
    p = parse_qwen_tool_completion("<think><function=no>x</function></think><function=book><parameter=seats>2"
                                   "</parameter></function>", tools=TOOLS)
    assert p.tool_calls == [{"name": "book", "arguments": {"seats": 2}}]
    assert p.parser_name == "qwen_xml_tool_call_unwrapped"


def test_empty_and_invalid_bodies():
    empty = parse_qwen_tool_completion("")
    assert empty.tool_calls == [] and empty.raw_text == ""
    bad = parse_qwen_tool_completion("<tool_call>{not json</tool_call>")
    assert bad.tool_calls == [] and bad.parse_errors == ["tool_call[0] is neither canonical JSON nor Qwen XML"]


# ---------------------------------------------------------------- parsed completion


def test_raw_parsed_completion():
    p = raw_parsed_completion("héllo ✓")
    assert (p.raw_text, p.answer_text, p.parser_name) == ("héllo ✓", "héllo ✓", "raw")
    assert p.tool_calls == [] and p.think_text == "" and p.extra_text == "" and p.parse_errors == []
    assert raw_parsed_completion("x", parser_name="custom").parser_name == "custom"
    assert raw_parsed_completion("").answer_text == ""


def test_parsed_completion_fields_and_slots():
    p = ParsedCompletion(raw_text="r", think_text="t", tool_calls=[{"name": "f", "arguments": {}}],
                         answer_text="a", parser_name="p", parse_errors=["e"], extra_text="x")
    assert set(p.to_dict()) == {f.name for f in dataclasses.fields(ParsedCompletion)}
    assert p.to_dict()["parse_errors"] == ["e"]
    with pytest.raises((AttributeError, TypeError)):
        p.new_attribute = 1
    d1, d2 = ParsedCompletion(raw_text="a"), ParsedCompletion(raw_text="b")
    d1.tool_calls.append({})
    assert d2.tool_calls == []  # no shared mutable defaults


# ---------------------------------------------------------------- replay buffer


def _exp(i):
    return Experience(sequences=i, old_log_probs=None, advantages=None, attention_mask=None, action_mask=None,
                      rewards=None)


def test_replay_buffer_basics():
    buf = ReplayBuffer()
    assert len(buf) == 0 and buf.take(3) == []
    buf.append_many([_exp(i) for i in range(3)])
    buf.append_many([])
    buf.append_many([_exp(3)])
    assert len(buf) == 4 and buf[0].sequences == 0 and buf[-1].sequences == 3
    assert [e.sequences for e in buf.take(2)] == [0, 1] and len(buf) == 4  # take does not remove
    assert len(buf.take(10)) == 4
    buf.clear()
    assert len(buf) == 0
    buf.append_many([_exp(7)])
    assert buf[0].sequences == 7


def test_replay_buffer_limit_keeps_the_newest():
    unlimited = ReplayBuffer(limit=0)
    unlimited.append_many([_exp(i) for i in range(100)])
    assert len(unlimited) == 100
    buf = ReplayBuffer(limit=3)
    buf.append_many([_exp(0), _exp(1)])
    buf.append_many([_exp(2)])
    assert [e.sequences for e in buf.items] == [0, 1, 2]
    buf.append_many([_exp(3), _exp(4)])
    assert [e.sequences for e in buf.items] == [2, 3, 4]


# ---------------------------------------------------------------- LoRA targets

AVAILABLE = [f"language.self_attn.{p}" for p in ("q_proj", "k_proj", "v_proj", "o_proj")] + \
            [f"language.mlp.{p}" for p in ("gate_proj", "up_proj", "down_proj")] + \
            ["visual.merger.linear_fc1", "visual.merger.linear_fc2", "visual.blocks.0.attn.qkv"]


def test_lora_presets_globs_and_canonical_names():
    safe = resolve_lora_target_modules(None, available=AVAILABLE)
    assert safe.resolved == ("language.self_attn.q_proj", "language.self_attn.v_proj")
    assert safe.requested == ("language_safe",)
    full = resolve_lora_target_modules(["language_all_linear"], available=AVAILABLE)
    assert len(full.resolved) == 7  # in_proj_z / out_proj are skipped on a dense model
    globbed = resolve_lora_target_modules(["language.mlp.*", "visual.merger.linear_fc1"], available=AVAILABLE)
    assert globbed.resolved == ("language.mlp.down_proj", "language.mlp.gate_proj", "language.mlp.up_proj",
                                "visual.merger.linear_fc1")
    assert globbed.signature == {"requested": ["language.mlp.*", "visual.merger.linear_fc1"],
                                 "resolved": list(globbed.resolved)}
    assert set(LORA_TARGET_PRESETS) >= {"language_safe", "language_all_linear", "vision_merger", "vision_common"}


def test_lora_targets_fail_closed():
    with pytest.raises(ValueError, match="Unsupported LoRA target"):
        resolve_lora_target_modules(["q_proj"], available=AVAILABLE)  # leaf aliases are not names
    with pytest.raises(ValueError, match="nonexistent"):
        resolve_lora_target_modules(["language.self_attn.q_proj", "nonexistent"], available=AVAILABLE)
    with pytest.raises(ValueError):
        resolve_lora_target_modules(["vision_merger"], available=AVAILABLE[:7])


def test_lora_target_enabled_by_canonical_or_leaf():
    assert lora_target_enabled({"language.self_attn.q_proj"}, "language.self_attn.q_proj")
    assert lora_target_enabled({"q_proj"}, "language.self_attn.q_proj")
    assert not lora_target_enabled({"k_proj"}, "language.self_attn.q_proj")


# ---------------------------------------------------------------- prompt rendering


class _Tok:
    def __init__(self, template=True):
        self.chat_template = "tpl" if template else None
        self.pad_token_id = None
        self.eos_token = "<eos>"
        self.pad_token = None
        self.padding_side = "right"
        self.calls = []

    def __setattr__(self, key, value):
        object.__setattr__(self, key, value)
        if key == "pad_token" and value == "<eos>":
            object.__setattr__(self, "pad_token_id", 2)

    def apply_chat_template(self, messages, **kw):
        self.calls.append((messages, kw))
        return "|".join(m["content"] for m in messages) + "|<gen>"


def test_render_messages_passes_turns_and_template_kwargs():
    tok = _Tok()
    msgs = [{"role": "system", "content": "s"}, {"role": "user", "content": "u1"},
            {"role": "assistant", "content": "a1"}, {"role": "user", "content": "u2"}]
    out = render_messages(tok, msgs, {"enable_thinking": False}, tools=[{"type": "function"}])
    assert out == "s|u1|a1|u2|<gen>"
    (passed, kw), = tok.calls
    assert passed == msgs
    assert kw == {"tokenize": False, "add_generation_prompt": True, "enable_thinking": False,
                  "tools": [{"type": "function"}]}


def test_render_without_template_and_tokenizer_padding():
    tok = _Tok(template=False)
    text = render_messages(tok, [{"role": "user", "content": "hi"}], tools=[{"n": 1}])
    assert text == 'user: hi\n\ntools: [{"n": 1}]'
    ensure_tokenizer_ready(tok)
    assert tok.pad_token == "<eos>" and tok.padding_side == "left"


# ---------------------------------------------------------------- advantages


def test_group_advantages():
    adv = group_advantages([1.0, 2.0, 3.0, 4.0])
    std = math.sqrt(sum((x - 2.5) ** 2 for x in (1, 2, 3, 4)) / 3)  # sample std (n - 1)
    assert adv == pytest.approx([(x - 2.5) / (std + 1e-8) for x in (1, 2, 3, 4)])
    assert sum(adv) == pytest.approx(0.0, abs=1e-9)
    assert group_advantages([0.7] * 5) == [0.0] * 5
    neg = group_advantages([-3.0, -1.0])
    assert neg[0] < 0 < neg[1]
    assert group_advantages([5.0]) == [0.0]
    assert group_advantages([]) == []
    wide = group_advantages([0.0, 1000.0])
    assert wide == pytest.approx([-1 / math.sqrt(2), 1 / math.sqrt(2)], rel=1e-6)
    custom = group_advantages([0.0, 1.0], eps=1.0)
    assert custom[1] == pytest.approx(0.5 / (math.sqrt(0.5) + 1.0))


def test_reward_variance_and_lower_median():
    assert has_reward_variance([0.1, 0.2])
    assert not has_reward_variance([0.3, 0.3])
    assert not has_reward_variance([0.3]) and not has_reward_variance([])
    assert not has_reward_variance([0.0, 1e-13])
    assert has_reward_variance([0.0, 1e-11])
    assert lower_median([4.0, 1.0, 3.0, 2.0]) == 2.0  # even groups take the lower middle
    assert lower_median([3.0, 1.0, 2.0]) == 2.0
    assert lower_median([]) == 0.0


# ---------------------------------------------------------------- reward helpers


def test_is_valid_json():
    assert is_valid_json('{"a": 1}') and is_valid_json("[1, 2]")
    for bad in ("", "plain text", '{"a": 1', None):
        assert not is_valid_json(bad)


def test_normalize_targets():
    (t,) = normalize_targets([{"output": {"content": {"a": 1}}}])
    assert t["output"] == {"content": {"a": 1}}
    (tc,) = normalize_targets([{"id": "x", "output": {"tool_calls": [{"name": "f", "arguments": {"k": 1}}]}}])
    assert tc["output"]["tool_calls"] == [{"name": "f", "arguments": {"k": 1}}] and tc["id"] == "x"
    assert len(normalize_targets([{"output": {"content": {"a": 1}}}, {"output": {"content": {"a": 2}}}])) == 2
    for bad in ([], {"output": {}}, ["x"], [{"id": "a"}], [{"output": "s"}], [{"output": {}}],
                [{"id": 1, "output": {"content": {"a": 1}}}]):
        with pytest.raises(ValueError):
            normalize_targets(bad)


def test_normalize_tool_calls():
    assert normalize_tool_calls([{"name": "f", "arguments": {"a": 1}}]) == [{"name": "f", "arguments": {"a": 1}}]
    assert len(normalize_tool_calls([{"name": "f", "arguments": {}}, {"name": "g", "arguments": {}}])) == 2
    for bad in ([], {"name": "f"}, ["f"], [{"name": "", "arguments": {}}], [{"arguments": {}}],
                [{"name": "f", "arguments": [1]}]):
        with pytest.raises(ValueError):
            normalize_tool_calls(bad)
