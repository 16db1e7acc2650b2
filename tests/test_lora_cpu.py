"""LoRA adapters keep parameter names/shapes, train only adapters, merge exactly."""
import torch

from complexity_framework_b200 import ComplexityModel, ModelConfig
from complexity_framework_b200.training.lora import (LoRAConfig, LoRALinear, apply_lora,
                                                     count_trainable, load_lora_state_dict,
                                                     lora_parameters, lora_state_dict, merge_lora,
                                                     set_lora_enabled)

TINY = dict(hidden_size=64, num_hidden_layers=2, num_attention_heads=4, num_key_value_heads=2,
            vocab_size=256, intermediate_size=64, shared_intermediate_size=128,
            num_experts=4, top_k=2, routing_strategy="modulo_cyclic",
            max_position_embeddings=64)


def _model():
    torch.manual_seed(0)
    return ComplexityModel(ModelConfig(**TINY))


def test_apply_train_merge_roundtrip():
    m = _model()
    ids = torch.randint(0, 256, (2, 16))
    base_logits = m(ids)["logits"].detach()
    names = apply_lora(m, LoRAConfig(r=4, alpha=8, include_experts=True))
    assert any("expert_gate" in n for n in names) and any("q_proj" in n for n in names)
    # B = 0 at init: the adapted model is the base model
    assert torch.allclose(m(ids)["logits"], base_logits, atol=1e-6)
    ct = count_trainable(m)
    assert 0 < ct["trainable"] < ct["total"] // 5
    opt = torch.optim.AdamW(lora_parameters(m), lr=1e-2)
    for _ in range(5):
        opt.zero_grad()
        m.loss(ids).backward()
        opt.step()
    tuned = m(ids)["logits"].detach()
    assert not torch.allclose(tuned, base_logits)
    set_lora_enabled(m, False)
    assert torch.allclose(m(ids)["logits"], base_logits, atol=1e-6)
    set_lora_enabled(m, True)
    sd = lora_state_dict(m)
    m2 = _model()
    apply_lora(m2, LoRAConfig(r=4, alpha=8, include_experts=True))
    load_lora_state_dict(m2, sd)
    assert torch.allclose(m2(ids)["logits"], tuned, atol=1e-5)
    n = merge_lora(m)
    assert n == len(names)
    keys = set(m.state_dict())
    assert keys == set(_model().state_dict())
    assert torch.allclose(m(ids)["logits"], tuned, atol=1e-5)


def test_lora_linear_merge_unmerge():
    torch.manual_seed(0)
    lin = torch.nn.Linear(16, 8)
    l = LoRALinear(lin, r=2, alpha=4)
    with torch.no_grad():
        l.lora_B.normal_()
    x = torch.randn(3, 16)
    y = l(x)
    l.merge()
    assert torch.allclose(l(x), y, atol=1e-5)
    l.unmerge()
    assert torch.allclose(l(x), y, atol=1e-5)


def test_reference_adapter_helpers():
    import torch

    from complexity_framework_b200 import ComplexityModel, ModelConfig
    from complexity_framework_b200.training.lora import (LoRAConfig, adapter_state_dict,
                                                         apply_lora, expert_lora_modules,
                                                         load_adapter_state_dict, lora_modules,
                                                         merged_model_state_dict,
                                                         unmerge_adapter_from_base)

    torch.manual_seed(0)
    cfg = ModelConfig(hidden_size=32, num_hidden_layers=1, num_attention_heads=4,
                      num_key_value_heads=2, vocab_size=64, intermediate_size=32,
                      shared_intermediate_size=64, num_experts=2, top_k=2,
                      max_position_embeddings=32)
    base = ComplexityModel(cfg)
    m = ComplexityModel(cfg)
    m.load_state_dict(base.state_dict())
    apply_lora(m, LoRAConfig(r=2, include_experts=True))
    with torch.no_grad():  # non-zero B so the adapters change the output
        for name, mod in {**lora_modules(m), **{k: v[2] for k, v in expert_lora_modules(m).items()}}.items():
            mod.lora_B.normal_(std=0.1)
    assert lora_modules(m) and expert_lora_modules(m)
    sd = adapter_state_dict(m)
    assert all(k.endswith((".lora_A", ".lora_B")) for k in sd)
    ids = torch.randint(0, 64, (1, 8))
    want = m(ids)["logits"]
    merged = merged_model_state_dict(m)
    assert set(merged) == set(base.state_dict())
    plain = ComplexityModel(cfg)
    plain.load_state_dict(merged)
    assert torch.allclose(plain(ids)["logits"], want, atol=1e-5)
    # a merged checkpoint + its adapter: unmerge restores the original base
    m2 = ComplexityModel(cfg)
    m2.load_state_dict(merged)
    apply_lora(m2, LoRAConfig(r=2, include_experts=True))
    load_adapter_state_dict(m2, sd)
    unmerge_adapter_from_base(m2)
    assert torch.allclose(m2(ids)["logits"], want, atol=1e-5)
    import pytest

    with pytest.raises(ValueError, match="does not match"):
        load_adapter_state_dict(m2, {k: v for k, v in list(sd.items())[1:]})
