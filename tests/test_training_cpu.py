"""CPU checks of the flat-buffer optimizer, scheduler and trainer."""
import math

import pytest
import torch

from complexity_framework_b200 import ComplexityModel, ModelConfig
from complexity_framework_b200.training import (FusedAdamW, Trainer, TrainingConfig,
                                                 lr_multiplier)

TINY = dict(hidden_size=128, num_hidden_layers=2, num_attention_heads=4, num_key_value_heads=2,
            vocab_size=1024, intermediate_size=128, shared_intermediate_size=384,
            num_experts=4, top_k=2, routing_strategy="modulo_cyclic",
            max_position_embeddings=128)


def test_fused_adamw_matches_torch_adamw():
    torch.manual_seed(0)
    a = torch.nn.Linear(16, 8)
    b = torch.nn.Linear(16, 8)
    b.load_state_dict(a.state_dict())
    oa = FusedAdamW(a.parameters(), lr=1e-2, betas=(0.9, 0.95), weight_decay=0.1)
    ob = torch.optim.AdamW(b.parameters(), lr=1e-2, betas=(0.9, 0.95), weight_decay=0.1,
                           eps=1e-8)
    for _ in range(5):
        x = torch.randn(4, 16)
        for m, o in ((a, oa), (b, ob)):
            o.zero_grad()
            m(x).pow(2).sum().backward()
            o.step()
    for pa, pb in zip(a.parameters(), b.parameters()):
        assert torch.allclose(pa, pb, atol=1e-6, rtol=1e-5)


def test_clip_matches_torch():
    torch.manual_seed(0)
    m = torch.nn.Linear(8, 8)
    o = FusedAdamW(m.parameters(), lr=1e-3)
    m(torch.randn(3, 8)).pow(2).sum().mul(100).backward()
    ref = torch.sqrt(sum((p.grad ** 2).sum() for p in m.parameters()))
    n = o.clip_grad_norm_(1.0)
    assert math.isclose(float(n), float(ref), rel_tol=1e-5)
    assert math.isclose(float(o._clip), min(1.0, 1.0 / (float(ref) + 1e-6)), rel_tol=1e-5)


def test_scheduler_shapes():
    assert lr_multiplier(0, kind="cosine", warmup=10, total=100, min_ratio=0.1) == 0.1
    assert lr_multiplier(9, kind="cosine", warmup=10, total=100, min_ratio=0.1) == 1.0
    assert math.isclose(lr_multiplier(100, kind="cosine", warmup=10, total=100, min_ratio=0.1), 0.1)
    assert lr_multiplier(50, kind="wsd", warmup=10, total=100, min_ratio=0.1) == 1.0
    assert lr_multiplier(50, kind="constant", warmup=10, total=100, min_ratio=0.1) == 1.0


def test_trainer_reduces_loss_and_resumes(tmp_path):
    torch.manual_seed(0)
    model = ComplexityModel(ModelConfig(**TINY))
    cfg = TrainingConfig(learning_rate=3e-3, warmup_steps=0, max_steps=50, lr_scheduler="constant",
                         checkpoint_dir=str(tmp_path), save_steps=1000, precision="fp32")
    tr = Trainer(model, cfg, device="cpu")
    ids = torch.randint(0, 1024, (2, 32), generator=torch.Generator().manual_seed(1))
    first = tr.train_step(ids)
    for _ in range(8):
        last = tr.train_step(ids)
    assert last < first
    tr.save_checkpoint()
    model2 = ComplexityModel(ModelConfig(**TINY))
    tr2 = Trainer(model2, cfg, device="cpu")
    assert tr2.resume("auto")
    assert tr2.global_step == tr.global_step
    a = tr.train_step(ids)
    b = tr2.train_step(ids)
    assert abs(a - b) < 1e-5
