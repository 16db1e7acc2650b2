"""Paged-KV engine against full-recompute greedy decoding (CPU, fp32)."""
import torch

from complexity_framework_b200 import ComplexityModel, ModelConfig
from complexity_framework_b200.inference import (BatchConfig, ContinuousBatcher,
                                                  GenerationConfig, InferenceConfig,
                                                  InferenceEngine, Request)

TINY = dict(hidden_size=128, num_hidden_layers=2, num_attention_heads=4, num_key_value_heads=2,
            vocab_size=1024, intermediate_size=128, shared_intermediate_size=384, num_experts=4,
            top_k=2, routing_strategy="modulo_cyclic", max_position_embeddings=256)


def greedy_recompute(model, prompt, n):
    ids = list(prompt)
    with torch.no_grad():
        for _ in range(n):
            logits = model(torch.tensor([ids]))["logits"][0, -1]
            ids.append(int(logits.argmax()))
    return ids[len(prompt):]


def _model():
    torch.manual_seed(0)
    return ComplexityModel(ModelConfig(**TINY)).eval()


def test_paged_engine_matches_recompute_ragged_batch():
    m = _model()
    g = torch.Generator().manual_seed(3)
    prompts = [torch.randint(0, 1024, (n,), generator=g).tolist() for n in (5, 37, 16, 1)]
    eng = InferenceEngine(m, InferenceConfig(page_size=16, num_pages=64, max_tokens_per_step=40,
                                             prefill_chunk_size=24))
    out = eng.generate(prompts, GenerationConfig(max_new_tokens=16))["new_tokens"]
    for p, o in zip(prompts, out):
        assert o == greedy_recompute(m, p, 16)
    assert len(eng.pool.free) == 64  # every page returned


def test_model_generate_and_batcher():
    m = _model()
    prompt = torch.randint(0, 1024, (1, 9), generator=torch.Generator().manual_seed(5))
    seq = m.generate(prompt, max_new_tokens=8)[0]
    assert seq[9:] == greedy_recompute(m, prompt[0].tolist(), 8)
    b = ContinuousBatcher(m, BatchConfig(max_batch_size=4, max_sequence_length=128))
    ids = [b.add_request(Request(input_ids=prompt[0], max_tokens=6, temperature=0.0))
           for _ in range(3)]
    done = b.run_until_complete()
    assert len(done) == 3 and all(r.output_ids == seq[9:15] for r in done)
    assert b.get_statistics()["completed"] == 3


def test_tiny_config_cpu_workload():
    """forward, CE backward, AdamW step, 16-token greedy decode (paged)."""
    from complexity_framework_b200.training import FusedAdamW

    cfg = dict(TINY, hidden_size=128, num_attention_heads=4, num_key_value_heads=2,
               shared_intermediate_size=384, intermediate_size=128)
    torch.manual_seed(0)
    m = ComplexityModel(ModelConfig(**cfg))
    ids = torch.randint(0, 1024, (2, 64), generator=torch.Generator().manual_seed(0))
    opt = FusedAdamW(m.parameters(), lr=3e-4)
    loss = m.loss(ids)
    loss.backward()
    opt.step()
    assert torch.isfinite(loss)
    m.eval()
    out = InferenceEngine(m).generate(ids[:, :8].tolist(),
                                      GenerationConfig(max_new_tokens=16))["new_tokens"]
    assert out[0] == greedy_recompute(m, ids[0, :8].tolist(), 16)
