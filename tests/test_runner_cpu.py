"""TrainRunner end to end on CPU: synthetic and token-shard data, logs, resume, export;
callbacks, telemetry, cluster planning and run-config handling."""
import json

import numpy as np
import pytest
import torch

from complexity_framework_b200 import ComplexityModel, ModelConfig
from complexity_framework_b200.data import write_token_shard
from complexity_framework_b200.training.callbacks import EarlyStoppingCallback, MetricsTracker
from complexity_framework_b200.training.cluster_plan import (ClusterRunPlan, ParallelPlan,
                                                             parse_tokens)
from complexity_framework_b200.training.run_config import compare_run_configs
from complexity_framework_b200.training.runner import TrainRunner
from complexity_framework_b200.training.telemetry import global_tr_diagnostics

TINY = dict(hidden_size=64, num_hidden_layers=1, num_attention_heads=4, num_key_value_heads=2,
            vocab_size=256, intermediate_size=64, shared_intermediate_size=128,
            num_experts=4, top_k=2, routing_strategy="modulo_cyclic",
            max_position_embeddings=64)


def _runner():
    return TrainRunner(make_config=lambda a: ModelConfig(**TINY))


def test_runner_synthetic_logs_resume_export(tmp_path):
    ck = tmp_path / "ck"
    args = ["--synthetic", "--max-steps", "4", "--batch-size", "2", "--seq-len", "16",
            "--checkpoint-dir", str(ck), "--log-steps", "1", "--save-steps", "2",
            "--precision", "fp32", "--no-progress"]
    s = _runner().main(args)
    assert s["steps"] == 4
    rows = (ck / "logs" / "training_log.csv").read_text().strip().splitlines()
    assert rows[0].startswith("step,loss") and len(rows) == 5
    recs = [json.loads(l) for l in (ck / "logs" / "metrics.jsonl").read_text().splitlines()]
    assert recs[-1]["step"] == 4
    assert (ck / "final" / "config.json").exists()
    assert (ck / "run_config.json").exists()
    s2 = _runner().main(args[:2] + ["6"] + args[3:] + ["--resume", "auto"])
    assert s2["steps"] == 6


def test_runner_token_shard(tmp_path):
    write_token_shard(tmp_path / "d", np.random.default_rng(0).integers(0, 256, 20000),
                      vocab_size=256)
    s = _runner().main(["--data", str(tmp_path / "d"), "--max-steps", "3", "--batch-size", "2",
                        "--seq-len", "16", "--checkpoint-dir", str(tmp_path / "ck"),
                        "--precision", "fp32", "--no-progress", "--optimizer", "lion"])
    assert s["steps"] == 3


def test_runner_token_mixture_resume_skips_trained_rows(tmp_path, monkeypatch):
    from complexity_framework_b200.data import corpus_mixture as cm

    rng = np.random.default_rng(1)
    cm.write_token_mixture(tmp_path / "mix", {"a": (0.5, rng.integers(0, 256, 16 * 40 + 1)),
                                              "b": (0.5, rng.integers(0, 256, 16 * 40 + 1))},
                           16, 16)
    seen = []
    orig = cm.PretokenizedCorpusMixtureDataset.__iter__

    def spy(self):
        for item in orig(self):
            seen.append(tuple(item["input_ids"].tolist()))
            yield item

    monkeypatch.setattr(cm.PretokenizedCorpusMixtureDataset, "__iter__", spy)
    ck = tmp_path / "ck"
    base = ["--token-mixture", str(tmp_path / "mix"), "--batch-size", "2", "--seq-len", "16",
            "--checkpoint-dir", str(ck), "--save-steps", "3", "--precision", "fp32",
            "--no-progress"]
    assert _runner().main(base + ["--max-steps", "3"])["steps"] == 3
    first = list(seen[:6])
    seen.clear()
    assert _runner().main(base + ["--max-steps", "5", "--resume", "auto"])["steps"] == 5
    full = list(cm.PretokenizedCorpusMixtureDataset(tmp_path / "mix"))
    rows = [tuple(x["input_ids"].tolist()) for x in full]
    assert first == rows[:6] and seen[:4] == rows[6:10]  # resumed on the next unseen rows


def test_cluster_plan_and_tokens():
    assert parse_tokens("200B") == 200 * 10 ** 9 and parse_tokens("1.5m") == 1_500_000
    p = ClusterRunPlan("x", parse_tokens("70b"), 1024, 201_194_368, ParallelPlan(1, 1, 8, 8, 8))
    assert p.tokens_per_step == 8 * 64 * 1024
    assert p.steps * p.tokens_per_step >= p.target_tokens
    assert "chinchilla_multiple" in "\n".join(p.summary_lines())


def test_run_config_diff_and_metrics(tmp_path):
    assert compare_run_configs({"lr": 1, "resume": None}, {"lr": 2, "resume": "auto"}) == [("lr", 1, 2)]
    m = MetricsTracker()
    for i in range(5):
        m.update(i, loss=10 - i)
    m.save(tmp_path / "m.json")
    assert MetricsTracker.load(tmp_path / "m.json").latest("loss") == 6


def test_early_stopping_and_telemetry():
    class T:
        should_stop = False
    cb = EarlyStoppingCallback(patience=2)
    t = T()
    for v in (1.0, 0.9, 0.95, 0.96):
        cb.on_evaluate(t, 0, v)
    assert t.should_stop
    model = ComplexityModel(ModelConfig(**TINY))
    d = global_tr_diagnostics(model, torch.arange(256))
    assert abs(d["max_min_ratio"] - 1.0) < 1e-6  # modulo-cyclic routing is exactly balanced
