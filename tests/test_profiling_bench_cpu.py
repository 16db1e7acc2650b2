"""Reference-named profiling entry points on a tiny model (CPU)."""
import torch

from complexity_framework_b200 import ComplexityModel, ModelConfig
from complexity_framework_b200 import profiling as P


def _m():
    torch.manual_seed(0)
    return ComplexityModel(ModelConfig(hidden_size=64, num_hidden_layers=2, num_attention_heads=4,
                                       num_key_value_heads=2, vocab_size=128,
                                       intermediate_size=64, shared_intermediate_size=128,
                                       num_experts=2, top_k=2, max_position_embeddings=32))


def test_flops_latency_training_memory():
    m = _m()
    c = P.get_model_complexity(m, (2, 16))
    assert c.flops > 0 and c.params == sum(p.numel() for p in m.parameters())
    assert P.count_flops(m, (2, 16)) == c.flops and P.estimate_macs(m, (2, 16)) == c.flops // 2
    r = P.benchmark_inference(m, (2, 16), num_runs=3, warmup_runs=1)
    assert r.num_runs == 3 and r.p50_latency_ms > 0 and r.throughput > 0 and "p99" in str(r)
    t = P.benchmark_training(_m(), batch_size=2, seq_length=16, num_steps=2, warmup_steps=1)
    assert t["tokens_per_s"] > 0
    est = P.estimate_model_memory(m, shards=2)
    assert est["parameters"] > 0 and est["optimizer_gb"] > 0
    a = P.ActivationMemoryProfiler(m)
    out = a.profile(torch.randint(0, 128, (2, 16)))
    assert out["module_outputs_gb"] > 0 and a.top(3)
    if not torch.cuda.is_available():
        assert P.find_optimal_batch_size(m, 16, start_batch=3) == 3
    with P.MemoryTracker() as tr:
        pass
    assert tr.peak_memory >= 0 and isinstance(P.get_memory_stats(), dict)
