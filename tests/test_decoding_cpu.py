"""Beam search, speculative decoding (greedy equivalence, self-speculative), sliding cache."""
import torch

from complexity_framework_b200 import ComplexityModel, ModelConfig
from complexity_framework_b200.inference import GenerationConfig, InferenceEngine
from complexity_framework_b200.inference.decoding import (LayerSkipDraft, SlidingWindowCache,
                                                          SpeculativeDecoder, beam_search)

CFG = dict(hidden_size=64, num_hidden_layers=3, num_attention_heads=4, num_key_value_heads=2,
           vocab_size=128, intermediate_size=64, shared_intermediate_size=128, num_experts=4,
           top_k=2, routing_strategy="modulo_cyclic", max_position_embeddings=128)


def _model(seed=0):
    torch.manual_seed(seed)
    return ComplexityModel(ModelConfig(**CFG)).eval()


def _greedy(model, prompt, n):
    eng = InferenceEngine(model)
    return eng.generate_tokens([prompt], GenerationConfig(max_new_tokens=n))[0]


def test_beam_width_one_is_greedy():
    m = _model()
    prompt = [3, 17, 42, 9]
    g = _greedy(m, prompt, 6)
    b = beam_search(m, prompt, num_beams=1, max_new_tokens=6)
    assert b["tokens"] == g


def test_beam_search_scores_sorted():
    m = _model()
    out = beam_search(m, [1, 2, 3], num_beams=3, max_new_tokens=5)
    scores = [s for _, s in out["hypotheses"]]
    assert scores == sorted(scores, reverse=True) and len(out["tokens"]) == 5


def test_speculative_greedy_matches_target():
    target = _model(0)
    draft = _model(1)  # unrelated weights: low acceptance, output must still match
    prompt = [5, 6, 7, 8, 9]
    ref = _greedy(target, prompt, 12)
    sd = SpeculativeDecoder(target, draft, num_draft_tokens=3)
    assert sd.generate(prompt, max_new_tokens=12) == ref
    self_sd = SpeculativeDecoder(target, LayerSkipDraft(target, 2), num_draft_tokens=4)
    assert self_sd.generate(prompt, max_new_tokens=12) == ref
    assert self_sd.stats.target_forwards <= 12


def test_speculative_sampling_runs():
    target = _model(0)
    sd = SpeculativeDecoder(target, LayerSkipDraft(target, 1), num_draft_tokens=3)
    out = sd.generate([1, 2, 3], max_new_tokens=10, temperature=1.0, seed=0)
    assert len(out) == 10 and 0 <= sd.stats.acceptance_rate <= 1


def test_sliding_window_cache():
    c = SlidingWindowCache(1, 1, 2, 4, window=5)
    for i in range(4):
        k, v = c.update(0, torch.full((1, 2, 2, 4), float(i)), torch.zeros(1, 2, 2, 4))
    assert k.shape[2] == 5 and float(k[0, 0, -1, 0]) == 3.0 and float(k[0, 0, 0, 0]) == 1.0
