"""Post-run tools: profile analyzer, GPU-memory recorder (fake query),
checkpoint evaluation (fake runtime), dataset split and synthetic images."""

import json
from pathlib import Path

import pytest
import torch

from graspo_b200.analysis.datasets import split_jsonl, synth_image_records
from graspo_b200.analysis.evaluate import evaluate_samples
from graspo_b200.analysis.gpu_memory import parse_query_csv, record, summarize_samples
from graspo_b200.analysis.profile import main as profile_main
from graspo_b200.analysis.profile import summarize_run
from graspo_b200.core.data import load_jsonl
from graspo_b200.core.schema import GraspoConfig, Sample


def _step(step, rollout, decode_tokens, trainable, total):
    return {"event": "train_step", "step": step,
            "timing": {"rollout_sec": rollout, "decode_tokens": decode_tokens, "total_observed_sec": total,
                       "optimize_sec": 1.0},
            "batch": {"decisions": {"trainable": {"total": trainable}, "terminal": {"invalid": 1}},
                      "reward": {"mean": 0.5}, "content": {"mean": 0.25}},
            "epoch": {"epoch": 0}}


def test_profile_summary_definitions(tmp_path, capsys):
    logs = tmp_path / "logs"
    logs.mkdir()
    events = [_step(1, 10.0, 100, 1, 20.0), _step(2, 4.0, 400, 2, 10.0), _step(3, 6.0, 600, 4, 30.0),
              {"event": "checkpoint_saved"}]
    (logs / "events.jsonl").write_text("".join(json.dumps(e) + "\n" for e in events) + "not json\n")
    s = summarize_run(tmp_path, skip_warmup_steps=1)
    assert s["step_count"] == 3 and s["measured_step_count"] == 2
    assert s["decode_tokens_per_sec"] == pytest.approx(1000 / 10.0)   # sum tokens / sum rollout seconds
    assert s["trainable_groups_per_hour"] == pytest.approx(6 * 3600 / (20.0 * 2))
    assert s["timing_mean"]["rollout_sec"] == 5.0 and s["latest_reward_mean"] == 0.5
    assert s["latest_trainable_groups"] == 4 and s["latest_invalid"] == 1
    assert profile_main([str(tmp_path), "--json"]) == 0
    assert json.loads(capsys.readouterr().out)[0]["name"] == tmp_path.name


def test_gpu_memory_recorder_with_fake_query(tmp_path):
    csv = "0, GPU-a, 1000, 180000, 183359, 50, 40, 300.5\n1, GPU-b, 3000, 178000, 183359, 90, 45, 700\nbad line\n"
    rows = parse_query_csv(csv)
    assert [r["gpu_index"] for r in rows] == ["0", "1"] and rows[1]["memory_used_mib"] == 3000.0
    calls = {"n": 0}

    def fake(gpus):
        calls["n"] += 1
        return [dict(r, memory_used_mib=r["memory_used_mib"] + calls["n"]) for r in parse_query_csv(csv)
                if r["gpu_index"] in gpus]

    summary = record(tmp_path / "mem", gpus=["0", "1"], interval_sec=0.0, query=fake,
                     stop=lambda: calls["n"] >= 3)
    assert summary["sample_count"] == 6
    assert summary["per_gpu"]["1"]["memory_used_mib_peak"] == 3003.0
    assert summary["per_gpu"]["0"]["utilization_gpu_pct_mean"] == 50.0
    assert len((tmp_path / "mem" / "gpu_memory.jsonl").read_text().splitlines()) == 6
    assert json.loads((tmp_path / "mem" / "gpu_memory_summary.json").read_text())["sample_count"] == 6
    assert summarize_samples([])["per_gpu"] == {}


class _Gen:
    def __init__(self, completions):
        self.completions = completions


class _EvalRuntime:
    def __init__(self, completions):
        self.completions = completions
        self.seen = []

    def is_primary(self):
        return True

    def generate_sample_groups(self, **kw):
        assert len(kw["samples"]) == 1
        self.seen.append(kw["rollout_group_size"])
        return [_Gen(self.completions)]


def test_evaluate_scores_groups_and_scrubs_media(tmp_path):
    cfg = GraspoConfig.from_dict({"training": {"rollout_group_size": 2, "output_dir": str(tmp_path)}})
    sample = Sample(messages=[{"role": "user", "content": "read"}],
                    targets=[{"id": "ok", "output": {"content": {"status": "ok"}}}],
                    metadata={"source": "synthetic"}, media=[{"type": "image", "path": "/private/p.png"}])
    good, bad = '```json\n{"status": "ok"}\n```', '```json\n{"status": "fail"}\n```'
    rt = _EvalRuntime([good, bad])
    summary = evaluate_samples(rt, cfg, [sample], tmp_path / "eval", checkpoint="/ckpt/final")
    assert rt.seen == [2]
    assert summary["count"] == 1 and summary["completion_count"] == 2 and summary["checkpoint"] == "/ckpt/final"
    assert summary["reward_range_mean"] > 0 and summary["all_right_rate"] == 0.5
    text = (tmp_path / "eval" / "completions.jsonl").read_text()
    rows = [json.loads(x) for x in text.splitlines()]
    assert rows[0]["matched_target_id"] == "ok" and rows[0]["metadata"]["media"] == [{"type": "image"}]
    assert "/private/p.png" not in text
    assert json.loads((tmp_path / "eval" / "summary.json").read_text())["completion_count"] == 2


def test_split_and_synthetic_images(tmp_path):
    info = synth_image_records(tmp_path / "synth", train_count=6, eval_count=2, seed=3)
    train = load_jsonl(info["train"])
    assert len(train) == 6 and len(load_jsonl(info["eval"])) == 2
    assert train[0].media and Path(train[0].media[0]["path"]).exists()
    assert set(train[0].targets[0]["output"]["content"]) == {"ticket", "status", "priority", "count"}
    again = synth_image_records(tmp_path / "synth2", train_count=6, eval_count=2, seed=3)
    assert Path(again["train"]).read_text().replace("synth2", "synth") == Path(info["train"]).read_text()
    src = tmp_path / "all.jsonl"
    src.write_text("".join(json.dumps({"i": i}) + "\n" for i in range(10)))
    res = split_jsonl(src, tmp_path / "t.jsonl", tmp_path / "e.jsonl", eval_count=3, seed=5,
                      manifest=tmp_path / "m.json")
    t = [json.loads(x)["i"] for x in (tmp_path / "t.jsonl").read_text().splitlines()]
    e = [json.loads(x)["i"] for x in (tmp_path / "e.jsonl").read_text().splitlines()]
    assert len(e) == 3 and sorted(t + e) == list(range(10)) and res["eval_indices"] == e
    assert split_jsonl(src, tmp_path / "t2.jsonl", tmp_path / "e2.jsonl", eval_count=3, seed=5)["eval_indices"] == e
    with pytest.raises(ValueError):
        split_jsonl(src, tmp_path / "a", tmp_path / "b", eval_count=10)


def test_endpoint_eval_against_a_local_server(tmp_path):
    """The OpenAI-compatible endpoint evaluator: wire format (image parts as data
    URLs, tools, per-completion seeds), structured tool-call replies and text
    replies both scored with the reward."""
    import threading
    from http.server import BaseHTTPRequestHandler, HTTPServer

    from graspo_b200.analysis.endpoint_eval import EndpointClient, evaluate_endpoint

    seen = []

    class Handler(BaseHTTPRequestHandler):
        def log_message(self, *a):
            pass

        def do_POST(self):
            body = json.loads(self.rfile.read(int(self.headers["Content-Length"])))
            seen.append((self.path, body))
            if body.get("tools"):
                msg = {"role": "assistant", "content": "",
                       "tool_calls": [{"type": "function", "function": {"name": "set_status",
                                                                         "arguments": json.dumps({"status": "ok"})}}]}
            else:
                status = "ok" if body["seed"] % 2 == 0 else "fail"
                msg = {"role": "assistant", "content": '```json\n{"status": "%s"}\n```' % status}
            data = json.dumps({"choices": [{"index": 0, "message": msg}]}).encode()
            self.send_response(200)
            self.send_header("Content-Type", "application/json")
            self.send_header("Content-Length", str(len(data)))
            self.end_headers()
            self.wfile.write(data)

    server = HTTPServer(("127.0.0.1", 0), Handler)
    threading.Thread(target=server.serve_forever, daemon=True).start()
    try:
        (tmp_path / "img.png").write_bytes(b"\x89PNG fake")
        tools = [{"type": "function", "function": {"name": "set_status", "parameters": {
            "type": "object", "properties": {"status": {"type": "string"}}, "required": ["status"]}}}]
        plain = Sample(messages=[{"role": "user", "content": [{"type": "image", "image": "img.png"},
                                                              {"type": "text", "text": "status?"}]}],
                       targets=[{"id": "t", "output": {"content": {"status": "ok"}}}])
        tool = Sample(messages=[{"role": "user", "content": "set it"}], tools=tools,
                      targets=[{"id": "c", "output": {"tool_calls": [{"name": "set_status",
                                                                      "arguments": {"status": "ok"}}]}}])
        cfg = GraspoConfig.from_dict({"training": {"output_dir": str(tmp_path), "max_new_tokens": 64}})
        client = EndpointClient(f"http://127.0.0.1:{server.server_port}/v1", "m", timeout=10)
        summary = evaluate_endpoint(cfg, [plain, tool], client, tmp_path / "ep", base_dir=tmp_path,
                                    samples_per_prompt=2, seed=10, chat_template_kwargs={"enable_thinking": False})
    finally:
        server.shutdown()
    assert [p for p, _ in seen] == ["/v1/chat/completions"] * 4
    first = seen[0][1]
    part = first["messages"][0]["content"][0]
    assert part["type"] == "image_url" and part["image_url"]["url"].startswith("data:image/png;base64,")
    assert [b["seed"] for _, b in seen] == [10, 11, 10, 11]
    assert first["max_tokens"] == 64 and first["chat_template_kwargs"] == {"enable_thinking": False}
    rows = [json.loads(x) for x in (tmp_path / "ep" / "completions.jsonl").read_text().splitlines()]
    assert [r["all_right"] for r in rows] == [True, False, True, True]
    assert rows[2]["parser_name"] == "endpoint_tool_calls" and rows[2]["tool_calls"][0]["name"] == "set_status"
    assert summary["completion_count"] == 4 and summary["all_right_rate"] == 0.75


def test_hf_baseline_generates_and_scores(tmp_path):
    """The transformers baseline on a tiny checkpoint: prompts through the chat
    template, sampled completions scored, EOS / length bookkeeping."""
    from graspo_b200.analysis.hf_baseline import HFGenerator, run_baseline
    from graspo_b200.utils.synth import TINY, write_qwen3_checkpoint

    path = write_qwen3_checkpoint(tmp_path / "m", TINY, seed=1, device="cpu", dtype=torch.float32)
    gen = HFGenerator(str(path), device="cpu", dtype=torch.float32)
    sample = Sample(messages=[{"role": "user", "content": "read"}],
                    targets=[{"id": "ok", "output": {"content": {"status": "ok"}}}])
    cfg = GraspoConfig.from_dict({"training": {"output_dir": str(tmp_path), "max_new_tokens": 6,
                                               "temperature": 1.0, "top_p": 1.0}})
    summary = run_baseline(cfg, [sample, sample], gen, tmp_path / "hf", base_dir=tmp_path, samples_per_prompt=2,
                           seed=3)
    rows = [json.loads(x) for x in (tmp_path / "hf" / "completions.jsonl").read_text().splitlines()]
    assert len(rows) == 4 and summary["completion_count"] == 4
    for r in rows:
        assert r["prompt_len"] > 0 and 0 <= r["completion_len"] <= 6
        assert r["truncated"] == (not r["hit_eos"] and r["completion_len"] == 6)
    assert "eos_rate" in summary and "truncated_rate" in summary
    # the same seeds give the same completions
    again = run_baseline(cfg, [sample, sample], gen, tmp_path / "hf2", base_dir=tmp_path, samples_per_prompt=2,
                         seed=3)
    assert again["reward_mean"] == summary["reward_mean"]
    assert (tmp_path / "hf2" / "completions.jsonl").read_text() == (tmp_path / "hf" / "completions.jsonl").read_text()
