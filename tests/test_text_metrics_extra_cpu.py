"""BERTScore, distinct-n and self-BLEU (CPU)."""
import pytest
import torch

from complexity_framework_b200 import ComplexityModel, ModelConfig
from complexity_framework_b200.data.tokenization import ByteTokenizer
from complexity_framework_b200.evaluation import BertScoreEvaluator, distinct_n, self_bleu


class _OneHot(torch.nn.Module):
    """Hidden state = one-hot of the token id: BERTScore becomes token overlap."""

    def __init__(self):
        super().__init__()
        self.w = torch.nn.Parameter(torch.zeros(1))

    def forward(self, x):
        return torch.nn.functional.one_hot(x, 300).float()


def test_bertscore_greedy_matching_on_one_hot_encoder():
    ev = BertScoreEvaluator(_OneHot(), lambda s: [ord(c) for c in s])
    r = ev.score(["abc"], ["abcd"])
    assert r["precision"] == pytest.approx(1.0)
    assert r["recall"] == pytest.approx(0.75)
    assert r["f1"] == pytest.approx(2 * 0.75 / 1.75)
    assert ev.score(["xy"], ["ab"])["f1"] == pytest.approx(0.0)
    mean = BertScoreEvaluator(_OneHot(), lambda s: [ord(c) for c in s], pooling="mean")
    assert mean.score(["ab"], ["ab"])["f1"] == pytest.approx(1.0)


def test_bertscore_with_complexity_model():
    torch.manual_seed(0)
    m = ComplexityModel(ModelConfig(hidden_size=64, num_hidden_layers=2, num_attention_heads=4,
                                    num_key_value_heads=2, vocab_size=300, intermediate_size=64,
                                    shared_intermediate_size=128, num_experts=4, top_k=2,
                                    routing_strategy="modulo_cyclic"))
    ev = BertScoreEvaluator(m, ByteTokenizer())
    same = ev.score(["the cat sat"], ["the cat sat"])
    assert same["f1"] == pytest.approx(1.0, abs=1e-5)
    diff = ev.score(["the cat sat"], ["zz qq"])
    assert diff["f1"] < same["f1"]


def test_diversity():
    d = distinct_n(["a b a b", "a b c"], max_n=2)
    assert d["distinct_1"] == pytest.approx(3 / 7)
    assert d["distinct_2"] == pytest.approx(3 / 5)
    assert self_bleu(["a b c d e", "a b c d e"]) > self_bleu(["a b c d e", "v w x y z"])
