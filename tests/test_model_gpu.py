"""Fused sm_100a model path against the fp32 PyTorch reference path on the same weights."""
import copy

import pytest
import torch

pytestmark = pytest.mark.gpu

CFG = dict(hidden_size=256, num_hidden_layers=2, num_attention_heads=4, num_key_value_heads=2,
           vocab_size=2048, intermediate_size=256, shared_intermediate_size=512, num_experts=4,
           top_k=2, top_k_primary_weight=0.5, routed_output_scale=2.0,
           routing_strategy="token_id_multi_hash", max_position_embeddings=256)


def _models():
    from complexity_framework_b200 import ComplexityModel, ModelConfig

    torch.manual_seed(0)
    ref = ComplexityModel(ModelConfig(**CFG)).cuda().float()
    fused = copy.deepcopy(ref).to(torch.bfloat16)
    return ref, fused


def _rel(a, b):
    return ((a.float() - b.float()).norm() / (b.float().norm() + 1e-12)).item()


def test_forward_logits_close():
    ref, fused = _models()
    ids = torch.randint(0, CFG["vocab_size"], (2, 128), device="cuda")
    with torch.no_grad():
        lr = ref(ids)["logits"]
        lf = fused(ids)["logits"]
    assert fused.layers[0].mlp.engine.last_backend.selected.value == "fused_cuda"
    assert _rel(lf, lr) < 3e-2


def test_loss_and_grads_close():
    ref, fused = _models()
    ids = torch.randint(0, CFG["vocab_size"], (2, 128), device="cuda")
    l_ref = ref.loss(ids)
    l_fused = fused.loss(ids)
    l_ref.backward()
    l_fused.backward()
    assert abs(l_ref.item() - l_fused.item()) < 2e-2 * abs(l_ref.item())
    gr = dict(ref.named_parameters())
    worst = []
    for name, p in fused.named_parameters():
        g_ref = gr[name].grad
        assert p.grad is not None, name
        worst.append((_rel(p.grad, g_ref), name))
    worst.sort(reverse=True)
    assert worst[0][0] < 6e-2, worst[:5]


def test_kernels_report_no_errors():
    from complexity_framework_b200.ops import check_errors

    torch.cuda.synchronize()
    check_errors(0)
