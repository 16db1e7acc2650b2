"""Evaluation metrics and benchmark runners on CPU."""
import json
import math

import torch

from complexity_framework_b200 import ComplexityModel, ModelConfig
from complexity_framework_b200.data import ByteTokenizer
from complexity_framework_b200.evaluation import (BenchmarkRunner, bleu, build_induction_batch,
                                                  compute_f1, compute_perplexity,
                                                  expected_calibration_error, rouge,
                                                  score_target_logits, token_f1)


def test_text_metrics():
    assert abs(bleu(["the cat sat on the mat"], [["the cat sat on the mat"]]) - 1.0) < 1e-9
    assert bleu(["a b c d"], [["w x y z"]]) == 0.0
    r = rouge("the cat sat", "the cat sat on the mat")
    assert r["rouge1"] > 0.5 and 0 < r["rougeL"] <= 1
    assert token_f1("The Cat", "cat") > 0.6
    f = compute_f1([0, 1, 1, 0], [0, 1, 0, 0])
    assert 0 < f["f1"] < 1
    assert expected_calibration_error([1.0, 1.0], [True, True]) == 0.0


def _model(vocab):
    torch.manual_seed(0)
    return ComplexityModel(ModelConfig(hidden_size=64, num_hidden_layers=1, num_attention_heads=4,
                                       num_key_value_heads=2, vocab_size=vocab,
                                       intermediate_size=64, shared_intermediate_size=128,
                                       num_experts=4, top_k=2, routing_strategy="modulo_cyclic",
                                       max_position_embeddings=256)).eval()


def test_perplexity_matches_loss():
    m = _model(256)
    ids = torch.randint(0, 256, (2, 32))
    out = compute_perplexity(m, [ids])
    assert abs(out["loss"] - float(m.loss(ids))) < 1e-4
    assert abs(out["perplexity"] - math.exp(out["loss"])) < 1e-3
    b = build_induction_batch(4, 8, 256)
    met = score_target_logits(m(b.input_ids)["logits"], b.target_ids)
    assert 0 <= met.accuracy <= 1


def test_benchmark_runner(tmp_path):
    rows = [{"ctx": "The sky is", "endings": ["blue", "loud", "fast", "sad"], "label": 0}] * 3
    (tmp_path / "hellaswag.jsonl").write_text("\n".join(json.dumps(r) for r in rows))
    mm = [{"question": "2+2?", "choices": ["3", "4", "5", "6"], "answer": 1}] * 2
    (tmp_path / "mmlu.jsonl").write_text("\n".join(json.dumps(r) for r in mm))
    tok = ByteTokenizer()
    res = BenchmarkRunner(_model(tok.vocab_size), tok, str(tmp_path)).run_all()
    assert set(res) == {"hellaswag", "mmlu"} and res["hellaswag"].num_samples == 3
    assert "acc=" in BenchmarkRunner.summarize(res)
