"""Routed-Q/O GQA, lexical attention channels and the conv + state mixer (CPU)."""
import pytest
import torch

from complexity_framework_b200 import ComplexityModel, ModelConfig
from complexity_framework_b200.core.attention import AttentionConfig, GroupedQueryAttention
from complexity_framework_b200.core.attention_variants import (
    CausalStateConvMixer, LexicalBiasGQA, LexicalKeyGQA, ProjectedLexicalKeyGQA, RoutedGQA,
    diagonal_decay_scan, routed_projection)

BASE = dict(hidden_size=64, num_hidden_layers=2, num_attention_heads=4, num_key_value_heads=2,
            vocab_size=128, intermediate_size=64, shared_intermediate_size=128, num_experts=4,
            top_k=2, routing_strategy="modulo_cyclic", max_position_embeddings=128)
ACFG = dict(hidden_size=64, num_attention_heads=4, num_key_value_heads=2, vocab_size=128,
            max_position_embeddings=64)


@pytest.mark.parametrize("attn", ["routed_gqa", "lexical_gqa", "lexical_key_gqa",
                                  "projected_lexical_key_gqa", "causal_state_conv"])
def test_model_train_step_and_causality(attn):
    torch.manual_seed(0)
    m = ComplexityModel(ModelConfig(**dict(BASE, attention_type=attn)))
    ids = torch.randint(0, 128, (2, 24))
    loss = m.loss(ids)
    loss.backward()
    assert torch.isfinite(loss)
    assert all(p.grad is not None for n, p in m.named_parameters()
               if "self_attn" in n and p.requires_grad and "lexical_objects" not in n), attn
    ids2 = ids.clone()
    ids2[:, 12:] = (ids2[:, 12:] + 1) % 128
    assert torch.allclose(m(ids)["logits"][:, :12], m(ids2)["logits"][:, :12], atol=1e-5), attn


def test_routed_projection_matches_per_chunk_matmul():
    torch.manual_seed(0)
    x, w = torch.randn(2, 8, 16), torch.randn(4, 16, 8)
    order = torch.randperm(16)
    y = routed_projection(x, w, order).reshape(16, 8)
    flat = x.reshape(16, 16)
    for e in range(4):
        rows = order[e * 4:(e + 1) * 4]
        torch.testing.assert_close(y[rows], flat[rows] @ w[e])


def test_routed_gqa_experts_by_token_id_and_sort_idx():
    torch.manual_seed(0)
    a = RoutedGQA(AttentionConfig(**ACFG))
    torch.nn.init.normal_(a.o_proj_w)
    x = torch.randn(1, 8, 64)
    ids = torch.tensor([[0, 1, 2, 3, 4, 5, 6, 7]])
    a.set_token_ids(ids)
    out, _ = a(x)
    # the same tokens in a different routing: moving every token to expert 0 changes it
    a.set_token_ids(ids * 4)
    out0, _ = a(x)
    assert not torch.allclose(out, out0)
    # an explicit sort_idx with experts in id order reproduces the id-modulo routing
    # of ids 0,4 | 1,5 | 2,6 | 3,7
    order = torch.tensor([0, 4, 1, 5, 2, 6, 3, 7])
    a.set_token_ids(ids)
    out_s, _ = a(x, sort_idx=order)
    torch.testing.assert_close(out_s, out)


def _copy_base(dst, src):
    for n in ("q_proj", "k_proj", "v_proj", "o_proj", "q_norm", "k_norm"):
        getattr(dst, n).load_state_dict(getattr(src, n).state_dict())


@pytest.mark.parametrize("cls", [LexicalBiasGQA, LexicalKeyGQA, ProjectedLexicalKeyGQA])
def test_lexical_zero_gate_equals_gqa(cls):
    torch.manual_seed(0)
    extra = dict(lexical_gqa_gate_init=0.0, lexical_key_gate_init=0.0, lexical_object_rank=8)
    lex = cls(AttentionConfig(**ACFG, extra=extra))
    base = GroupedQueryAttention(AttentionConfig(**ACFG))
    _copy_base(lex, base)
    x = torch.randn(2, 10, 64)
    ids = torch.randint(0, 128, (2, 10))
    torch.nn.init.normal_(lex.lexical_objects.weight)
    lex.set_token_ids(ids)
    torch.testing.assert_close(lex(x)[0], base(x)[0], atol=1e-5, rtol=1e-5)
    with torch.no_grad():
        lex.lexical_gate.fill_(1.0)
    assert not torch.allclose(lex(x)[0], base(x)[0], atol=1e-4)


def test_lexical_gqa_explicit_scale_and_token_code():
    torch.manual_seed(0)
    a = LexicalBiasGQA(AttentionConfig(**ACFG, extra=dict(lexical_gqa_gate_init=0.5,
                                                         lexical_object_rank=8)))
    x = torch.randn(1, 6, 64)
    ids = torch.arange(6)[None]
    scale = torch.randn(1, 6, 8)
    o1, _ = a(x, lexical_scale=scale, token_ids=ids)
    o2, _ = a(x, lexical_scale=scale, token_ids=ids + 1)  # token code differs
    assert not torch.allclose(o1, o2)
    code = a.token_code(torch.tensor([0]))[0]
    d = torch.arange(1, 9, dtype=torch.float64)
    ph = torch.pi * d.sqrt()
    ref = torch.where(d.long() % 2 == 0, ph.sin(), ph.cos()).float()
    torch.testing.assert_close(code, ref)
    with pytest.raises(ValueError):
        a(x, lexical_scale=torch.randn(1, 6, 4), token_ids=ids)


def test_diagonal_decay_scan_matches_loop():
    torch.manual_seed(0)
    u, d, s0 = torch.randn(2, 150, 8), torch.rand(8) * 0.05 + 0.95, torch.randn(2, 8)
    states, last = diagonal_decay_scan(u, d, s0, chunk=32)
    s = s0.clone()
    for t in range(150):
        s = d * s + u[:, t]
        torch.testing.assert_close(states[:, t], s, atol=1e-4, rtol=1e-4)
    torch.testing.assert_close(last, s, atol=1e-4, rtol=1e-4)


def test_state_conv_cached_decode_equals_full():
    torch.manual_seed(0)
    m = CausalStateConvMixer(AttentionConfig(**ACFG, extra=dict(causal_conv_kernel_size=4)))
    x = torch.randn(2, 12, 64)
    full, _ = m(x)
    out, cache = m(x[:, :5], use_cache=True)
    outs = [out]
    for t in range(5, 12):
        o, cache = m(x[:, t:t + 1], past_key_value=cache, use_cache=True)
        outs.append(o)
    torch.testing.assert_close(torch.cat(outs, 1), full, atol=1e-5, rtol=1e-4)


@pytest.mark.parametrize("delta", [False, True])
def test_associative_scan_matches_recurrence(delta):
    from complexity_framework_b200.core.associative import associative_scan

    torch.manual_seed(0)
    B, S, r = 2, 70, 8
    q = torch.nn.functional.normalize(torch.randn(B, S, r), dim=-1)
    k = torch.nn.functional.normalize(torch.randn(B, S, r), dim=-1)
    v, S0 = torch.randn(B, S, r), torch.randn(B, r, r) * 0.1
    d, w = torch.tensor(0.97), torch.tensor(0.8)
    reads, last = associative_scan(q, k, v, S0, d, w, delta, chunk=16)
    st = S0.clone()
    for t in range(S):
        torch.testing.assert_close(reads[:, t], torch.einsum("br,brc->bc", q[:, t], st),
                                   atol=1e-4, rtol=1e-4)
        e = v[:, t] - torch.einsum("br,brc->bc", k[:, t], st) if delta else v[:, t]
        st = d * st + w * k[:, t, :, None] * e[:, None, :]
    torch.testing.assert_close(last, st, atol=1e-4, rtol=1e-4)


@pytest.mark.parametrize("delta", [False, True])
def test_fast_weight_conv_model_and_cached_decode(delta):
    from complexity_framework_b200.core.attention_variants import CausalFastWeightConvMixer

    torch.manual_seed(0)
    m = ComplexityModel(ModelConfig(**dict(BASE, attention_type="causal_fast_weight_conv",
                                           causal_stable_delta=delta,
                                           causal_contextual_mix_init=0.1)))
    ids = torch.randint(0, 128, (2, 24))
    loss = m.loss(ids)
    loss.backward()
    assert torch.isfinite(loss)
    ids2 = ids.clone()
    ids2[:, 12:] = (ids2[:, 12:] + 1) % 128
    assert torch.allclose(m(ids)["logits"][:, :12], m(ids2)["logits"][:, :12], atol=1e-5)
    mix = CausalFastWeightConvMixer(AttentionConfig(**ACFG, extra=dict(
        causal_stable_delta=delta, causal_contextual_mix_init=0.2, causal_delta_chunk_size=4)))
    x, tid = torch.randn(2, 11, 64), torch.randint(0, 128, (2, 11))
    full, _ = mix(x, token_ids=tid)
    out, cache = mix(x[:, :6], token_ids=tid[:, :6], use_cache=True)
    outs = [out]
    for t in range(6, 11):
        o, cache = mix(x[:, t:t + 1], token_ids=tid[:, t:t + 1], past_key_value=cache,
                       use_cache=True)
        outs.append(o)
    torch.testing.assert_close(torch.cat(outs, 1), full, atol=1e-4, rtol=1e-4)
