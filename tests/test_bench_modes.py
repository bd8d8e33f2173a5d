"""Kernel-benchmark modes that also run on the CPU: the hybrid-family training
micro-batch at the test shape prints one JSON line with its timings."""

import json


def test_hybrid_training_benchmark_runs(tmp_path, capsys):
    from graspo_b200.bench.kernels import main

    main(["hybrid", "--tiny", "--layers", "4", "--rows", "2", "--seq", "64", "--iters", "1",
          "--ckpt", str(tmp_path)])
    line = [x for x in capsys.readouterr().out.splitlines() if x.startswith("{")][-1]
    out = json.loads(line)
    assert out["kernel"] == "hybrid_train_microbatch" and out["layers"] == 4
    assert out["fwd_ms"] > 0 and out["bwd_ms"] > 0 and out["tokens_per_s"] > 0
