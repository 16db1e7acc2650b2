"""Reference-named scorers and the Evaluator; ROUGE/BLEU parity with the reference."""
import os
import sys

import pytest
import torch

from complexity_framework_b200.evaluation.evaluator import (BleuScorer, CoherenceMetrics,
                                                            DiversityMetrics, Evaluator,
                                                            RougeScorer, evaluate_on_dataset)

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
REF = os.path.join(ROOT, "baseline", "_ref")
PRED = "the cat sat on the mat today"
REFS = ["the cat is on the mat", "a cat sat on a mat today"]


def test_scorers_against_reference():
    if not os.path.isdir(os.path.join(REF, "complexity")):
        pytest.skip("reference install not present")
    sys.path.insert(0, REF)
    try:
        from complexity.evaluation import metrics as R
    finally:
        sys.path.remove(REF)
    a, b = RougeScorer().score(PRED, REFS[0]), R.RougeScorer().score(PRED, REFS[0])
    for m in ("rouge1", "rouge2", "rougeL"):
        for k in ("precision", "recall", "f1"):
            assert a[m][k] == pytest.approx(b[m][k]), (m, k)
    x, y = BleuScorer().score(PRED, REFS), R.BleuScorer().score(PRED, REFS)
    assert x["bleu"] == pytest.approx(y["bleu"], rel=1e-9)
    d1 = DiversityMetrics().entropy([PRED, REFS[0]])
    d2 = R.DiversityMetrics().entropy([PRED, REFS[0]])
    assert d1 == pytest.approx(d2)
    assert CoherenceMetrics().repetition_rate("a b c a b c a b c") == pytest.approx(
        R.CoherenceMetrics().repetition_rate("a b c a b c a b c"))


def test_scorers_basic():
    assert RougeScorer().score("a b c", "a b c")["rougeL"]["f1"] == 1.0
    assert BleuScorer().score("", ["x"])["bleu"] == 0.0
    assert DiversityMetrics().compute_all(["a b", "c d"])["distinct_1"] == 1.0
    assert CoherenceMetrics().sentence_coherence("one sentence") == 1.0


def test_evaluator_model_side():
    from complexity_framework_b200 import ComplexityModel, ModelConfig
    from complexity_framework_b200.data.tokenization import get_tokenizer

    torch.manual_seed(0)
    m = ComplexityModel(ModelConfig(hidden_size=32, num_hidden_layers=1, num_attention_heads=4,
                                    num_key_value_heads=2, vocab_size=260, intermediate_size=32,
                                    shared_intermediate_size=64, num_experts=2, top_k=2,
                                    max_position_embeddings=64))
    tok = get_tokenizer("byte")
    batches = [torch.randint(0, 260, (2, 12)) for _ in range(2)]
    r = evaluate_on_dataset(m, batches, metrics=("perplexity", "accuracy", "ece"))
    assert r["perplexity"] > 1 and 0 <= r["accuracy"] <= 1 and 0 <= r["ece"] <= 1
    ev = Evaluator(m, tok)
    acc = ev.multiple_choice_accuracy([{"context": "ab", "choices": ["c", "d"], "answer": 0}])
    assert acc in (0.0, 1.0)
    g = ev.generate_and_evaluate(["hi"], ["there"], max_new_tokens=3,
                                 metrics=("f1", "exact_match", "rouge", "bleu"))
    assert set(g) >= {"f1", "exact_match", "rouge1", "bleu"}
