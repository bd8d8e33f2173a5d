"""JSONL record validation and the strict config schema (pure CPU).

Behaviour follows the reference's data layer (src/graspo/core/data.py:13-413)
and schema (src/graspo/core/schema.py:14-268).
"""

from __future__ import annotations

import json
import warnings

import pytest
from pydantic import ValidationError

from graspo_b200.core.data import (
    build_sft_target_text,
    content_to_text_and_media,
    load_jsonl,
    sample_from_record,
    write_jsonl,
)
from graspo_b200.core.schema import GraspoConfig, Sample, TrainingConfig

WEATHER_TOOL = {
    "type": "function",
    "function": {
        "name": "get_weather",
        "parameters": {
            "type": "object",
            "properties": {"city": {"type": "string"}, "unit": {"type": "string", "enum": ["c", "f"]}},
            "required": ["city"],
        },
    },
}


def _content_record(**extra):
    rec = {"messages": [{"role": "user", "content": "extract"}],
           "targets": [{"id": "a", "output": {"content": {"x": 1}}}]}
    rec.update(extra)
    return rec


def _tool_record(calls, tools=(WEATHER_TOOL,)):
    return {"messages": [{"role": "user", "content": "weather?"}], "tools": list(tools),
            "targets": [{"output": {"tool_calls": calls}}]}


def _write(tmp_path, records, name="d.jsonl"):
    p = tmp_path / name
    p.write_text("\n".join(json.dumps(r) for r in records) + "\n", encoding="utf-8")
    return p


# ---------------------------------------------------------------- data


def test_content_record_and_metadata():
    s = sample_from_record(_content_record(source="unit", difficulty=3))
    assert s.targets[0]["output"]["content"] == {"x": 1}
    assert s.metadata == {"source": "unit", "difficulty": 3}
    assert not s.expects_tool_calls and s.tools is None and s.media == []


def test_write_and_load_round_trip(tmp_path):
    samples = [sample_from_record(_content_record(k=i)) for i in range(3)]
    path = tmp_path / "sub" / "out.jsonl"
    write_jsonl(samples, path)
    loaded = load_jsonl(path)
    assert [s.model_dump() for s in loaded] == [s.model_dump() for s in samples]


def test_multi_turn_messages_are_kept(tmp_path):
    rec = {"messages": [{"role": "system", "content": "be terse"}, {"role": "user", "content": "q1"},
                        {"role": "assistant", "content": "a1"}, {"role": "user", "content": "q2"}],
           "targets": [{"output": {"content": {"y": 2}}}]}
    (s,) = load_jsonl(_write(tmp_path, [rec]))
    assert [m["role"] for m in s.messages] == ["system", "user", "assistant", "user"]


def test_tool_targets_alternatives_and_ordered_calls():
    alt = _tool_record([{"name": "get_weather", "arguments": {"city": "Paris"}}])
    alt["targets"].append({"output": {"tool_calls": [{"name": "get_weather", "arguments": {"city": "Lyon", "unit": "c"}}]}})
    s = sample_from_record(alt)
    assert s.expects_tool_calls and len(s.targets) == 2
    multi = _tool_record([{"name": "get_weather", "arguments": {"city": "A"}},
                          {"name": "get_weather", "arguments": {"city": "B"}}])
    calls = sample_from_record(multi).targets[0]["output"]["tool_calls"]
    assert [c["arguments"]["city"] for c in calls] == ["A", "B"]


@pytest.mark.parametrize("calls, needle", [
    ([{"name": "get_time", "arguments": {"city": "A"}}], "not declared"),
    ([{"name": "get_weather", "arguments": {"city": "A", "unit": "k"}}], "enum"),
    ([{"name": "get_weather", "arguments": {"unit": "c"}}], "required"),
])
def test_tool_targets_must_fit_the_declared_schema(calls, needle):
    with pytest.raises(ValueError, match=needle):
        sample_from_record(_tool_record(calls))


def test_tools_must_be_a_list():
    rec = _tool_record([{"name": "get_weather", "arguments": {"city": "A"}}])
    rec["tools"] = {"get_weather": WEATHER_TOOL}
    with pytest.raises(ValueError, match="list"):
        sample_from_record(rec)


def test_json_array_file_is_not_a_training_format(tmp_path):
    p = tmp_path / "d.json"
    p.write_text(json.dumps([_content_record(), _content_record()]), encoding="utf-8")
    with pytest.raises(ValueError, match=r"d\.json:1"):
        load_jsonl(p)


def test_multimodal_messages_collect_media_once():
    content = [{"type": "image", "image": "a.png"}, {"type": "text", "text": "what is it?"},
               {"type": "image_url", "image_url": {"url": "b.png"}}]
    rec = {"messages": [{"role": "user", "content": content}, {"role": "user", "content": [{"type": "image", "path": "a.png"}]}],
           "targets": [{"output": {"content": {"label": "cat"}}}]}
    s = sample_from_record(rec)
    assert s.media == [{"type": "image", "path": "a.png"}, {"type": "image", "path": "b.png"}]
    text, media = content_to_text_and_media(content)
    assert text == "<image>\nwhat is it?\n<image>" and len(media) == 2
    with pytest.raises(ValueError, match="unsupported"):
        content_to_text_and_media([{"type": "audio", "path": "x.wav"}])


def test_prompt_only_record_is_rejected():
    with pytest.raises(ValueError, match="targets"):
        sample_from_record({"messages": [{"role": "user", "content": "hi"}]})


@pytest.mark.parametrize("field", ["prompt", "image", "images", "video", "videos"])
def test_removed_top_level_fields_are_rejected(field):
    with pytest.raises(ValueError, match="removed input field"):
        sample_from_record(_content_record(**{field: "x"}))


def test_ground_truth_is_rejected():
    with pytest.raises(ValueError, match="ground_truth"):
        sample_from_record(_content_record(ground_truth={"x": 1}))


@pytest.mark.parametrize("targets", [[], "x", [{"output": {}}], [{"id": 3, "output": {"content": {"a": 1}}}],
                                     [{"no_output": 1}], [{"output": "text"}]])
def test_invalid_targets_are_rejected(targets):
    with pytest.raises(ValueError):
        sample_from_record({"messages": [{"role": "user", "content": "q"}], "targets": targets})


def test_final_assistant_message_is_rejected():
    rec = _content_record()
    rec["messages"].append({"role": "assistant", "content": '{"x": 1}'})
    with pytest.raises(ValueError, match="leak"):
        sample_from_record(rec)


def _with_assistant(msg):
    return {"messages": [{"role": "user", "content": "q"}, msg, {"role": "user", "content": "again"}],
            "targets": [{"output": {"content": {"x": 1}}}]}


def test_assistant_history_with_structured_tool_calls_is_accepted():
    msg = {"role": "assistant", "content": "", "tool_calls": [{"name": "f", "arguments": {"a": 1}}]}
    assert len(sample_from_record(_with_assistant(msg)).messages) == 3
    plain = {"role": "assistant", "content": "just text"}
    assert len(sample_from_record(_with_assistant(plain)).messages) == 3


@pytest.mark.parametrize("msg, needle", [
    ({"role": "assistant", "content": "<tool_call>{}</tool_call>"}, "raw tool-call"),
    ({"role": "assistant", "content": "<function=f><parameter=a>1</parameter></function>"}, "raw tool-call"),
    ({"role": "assistant", "content": [{"type": "text", "text": "<tool_call>"}]}, "raw tool-call"),
    ({"role": "assistant", "content": "", "tool_calls": {"name": "f"}}, "non-empty list"),
    ({"role": "assistant", "content": "", "tool_calls": []}, "non-empty list"),
    ({"role": "assistant", "content": "", "tool_calls": [{"arguments": {}}]}, "name"),
    ({"role": "assistant", "content": "", "tool_calls": [{"name": "f"}]}, "arguments"),
    ({"role": "assistant", "content": "", "tool_calls": [{"name": "f", "arguments": {"a": "<parameter=x>"}}]},
     "raw tool-call markers"),
])
def test_assistant_history_with_raw_or_malformed_calls_is_rejected(msg, needle):
    with pytest.raises(ValueError, match=needle):
        sample_from_record(_with_assistant(msg))


def test_message_shape_errors():
    with pytest.raises(ValueError, match="non-empty 'messages'"):
        sample_from_record({"messages": [], "targets": [{"output": {"content": {"a": 1}}}]})
    with pytest.raises(ValueError, match="role"):
        sample_from_record({"messages": [{"content": "x"}], "targets": [{"output": {"content": {"a": 1}}}]})
    with pytest.raises(ValueError, match="content"):
        sample_from_record({"messages": [{"role": "user"}], "targets": [{"output": {"content": {"a": 1}}}]})


def test_sft_target_text_forms():
    text = build_sft_target_text({"content": {"a": 1}})
    assert text.startswith("```json\n") and json.loads(text[8:-4]) == {"a": 1}
    xml = build_sft_target_text({"tool_calls": [{"name": "f", "arguments": {"n": 2.0, "ok": True, "s": "x"}}]})
    assert xml == ("<tool_call>\n<function=f>\n<parameter=n>2</parameter><parameter=ok>true</parameter>"
                   "<parameter=s>x</parameter>\n</function>\n</tool_call>")
    assert build_sft_target_text({}) == ""


# ---------------------------------------------------------------- schema


def test_unknown_fields_are_rejected_at_every_level():
    with pytest.raises(ValidationError):
        TrainingConfig(not_a_field=1)
    with pytest.raises(ValidationError):
        GraspoConfig.from_dict({"training": {"kl_coef": 0.1}})
    with pytest.raises(ValidationError):
        GraspoConfig.from_dict({"lora": {"dropout_p": 0.1}})
    with pytest.raises(ValueError, match="unknown top-level"):
        GraspoConfig.from_dict({"trainer": {}})


def test_output_dir_and_run_name_resolution():
    auto = GraspoConfig.from_dict({})
    assert auto.training.output_dir.startswith("outputs") and auto.training.run_name.startswith("graspo_")
    assert auto.training.output_dir.endswith(auto.training.run_name)
    only_dir = GraspoConfig.from_dict({"training": {"output_dir": "runs/exp7"}})
    assert only_dir.training.run_name == "exp7"
    only_name = GraspoConfig.from_dict({"training": {"run_name": "mine"}})
    assert only_name.training.output_dir.replace("\\", "/") == "outputs/mine"
    both = GraspoConfig.from_dict({"training": {"output_dir": "x/y", "run_name": "z"}})
    assert (both.training.output_dir, both.training.run_name) == ("x/y", "z")
    # the generated name is fixed for the life of the process
    assert GraspoConfig.from_dict({}).training.run_name == auto.training.run_name


def test_training_defaults_and_derived_threshold():
    t = TrainingConfig()
    assert t.seed == 42 and t.rollout_group_size == 8
    t = TrainingConfig(optimize_prompt_batch_size=3, rollout_group_size=5)
    assert t.replay_buffer_optimize_threshold == 15


def test_sample_model():
    tool_sample = Sample(messages=[{"role": "user", "content": "q"}],
                         targets=[{"output": {"tool_calls": [{"name": "f", "arguments": {}}]}}])
    assert tool_sample.expects_tool_calls
    content_sample = Sample(messages=[{"role": "user", "content": "q"}], targets=[{"output": {"content": {"a": 1}}}])
    assert not content_sample.expects_tool_calls
    assert content_sample.metadata == {} and content_sample.media == []
    with pytest.raises(ValidationError):
        content_sample.messages = []
    with pytest.raises(ValidationError):
        Sample(messages=[], targets=[], extra_key=1)


def test_legacy_backend_config_section():
    legacy = {"backend_config": {"graspoflow": {"tp_size": 2}}}
    with warnings.catch_warnings(record=True) as caught:
        warnings.simplefilter("always")
        cfg = GraspoConfig.from_dict(legacy)
    assert cfg.graspoflow.tp_size == 2
    assert any("deprecated" in str(w.message) for w in caught)
    both = GraspoConfig.from_dict({"graspoflow": {"tp_size": 4}, "backend_config": {"graspoflow": {"tp_size": 2}}})
    assert both.graspoflow.tp_size == 4
