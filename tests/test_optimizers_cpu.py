"""Optimizer family: Newton-Schulz, each optimizer lowers a loss, Trainer factory."""
import pytest
import torch

from complexity_framework_b200 import ComplexityModel, ModelConfig
from complexity_framework_b200.training import Trainer, TrainingConfig
from complexity_framework_b200.training import optimizers as O

TINY = dict(hidden_size=64, num_hidden_layers=1, num_attention_heads=4, num_key_value_heads=2,
            vocab_size=256, intermediate_size=64, shared_intermediate_size=128,
            num_experts=4, top_k=2, routing_strategy="modulo_cyclic",
            max_position_embeddings=64)


def test_newton_schulz_orthogonalises():
    torch.manual_seed(0)
    M = torch.randn(3, 32, 48)
    X = O.newton_schulz(M, steps=10)
    s = torch.linalg.svdvals(X)
    # quintic NS drives singular values into a band around 1 (not exactly 1)
    assert s.min() > 0.5 and s.max() < 1.3
    Xa, n = O.newton_schulz_adaptive(M[0], min_steps=3, max_steps=12, tol=1e-2)
    assert 3 <= n <= 12 and Xa.shape == M[0].shape


def _quadratic_problem():
    torch.manual_seed(0)
    model = torch.nn.Sequential(torch.nn.Linear(16, 32), torch.nn.Linear(32, 8))
    x = torch.randn(64, 16)
    y = torch.randn(64, 8)
    return model, lambda: torch.nn.functional.mse_loss(model(x), y)


@pytest.mark.parametrize("kind", ["adamw", "lion", "sophia", "adam8bit", "came", "adalomo",
                                  "muon", "musgd", "adam", "sgd"])
def test_each_optimizer_reduces_loss(kind):
    model, loss_fn = _quadratic_problem()
    opt = O.get_optimizer(model, kind, lr=1e-2, weight_decay=0.0,
                          **({"min_8bit_size": 16} if kind == "adam8bit" else {}))
    first = float(loss_fn())
    for i in range(60):
        opt.zero_grad()
        loss = loss_fn()
        loss.backward()
        if kind == "sophia" and i % 5 == 0:
            opt.update_hessian(batch_size=64)
        opt.step()
    assert float(loss_fn()) < first


def test_adam8bit_tracks_fp32_adam():
    torch.manual_seed(0)
    a = torch.nn.Linear(64, 64, bias=False)
    b = torch.nn.Linear(64, 64, bias=False)
    b.load_state_dict(a.state_dict())
    oa = O.Adam8bit(a.parameters(), lr=1e-3, min_8bit_size=1)
    ob = torch.optim.Adam(b.parameters(), lr=1e-3)
    for _ in range(10):
        x = torch.randn(8, 64)
        for m, o in ((a, oa), (b, ob)):
            o.zero_grad()
            m(x).pow(2).mean().backward()
            o.step()
    rel = (a.weight - b.weight).norm() / (b.weight - b.weight.detach()).norm().clamp_min(1)
    assert float((a.weight - b.weight).abs().max()) < 5e-3, rel


def test_tr_groups_and_muon_tr_per_expert():
    model = ComplexityModel(ModelConfig(**TINY))
    groups = O.tr_param_groups(model, 4)
    kinds = {g["param_type"] for g in groups}
    assert "expert" in kinds and "norm" in kinds
    opt = O.MuonTR(groups, lr=0.01, num_experts=4, token_counts=torch.tensor([10., 20, 30, 40]),
                   lr_warmup_steps=1)
    ids = torch.randint(0, 256, (2, 16))
    before = {n: p.detach().clone() for n, p in model.named_parameters()}
    model.loss(ids).backward()
    opt.step()
    moved = [n for n, p in model.named_parameters() if not torch.equal(p, before[n])]
    assert any("expert" in n for n in moved)


def test_adam_tr_spectral_runs():
    model = ComplexityModel(ModelConfig(**TINY))
    opt = O.AdamTR(O.adamtr_param_groups(model, 4), lr=1e-3, spectral_warmup_steps=0)
    ids = torch.randint(0, 256, (2, 16))
    for _ in range(3):
        opt.zero_grad()
        model.loss(ids).backward()
        opt.step()


@pytest.mark.parametrize("kind", ["muon", "lion", "adam_tr"])
def test_trainer_with_optimizer_type(kind, tmp_path):
    torch.manual_seed(0)
    model = ComplexityModel(ModelConfig(**TINY))
    cfg = TrainingConfig(optimizer_type=kind, learning_rate=3e-3, warmup_steps=0, max_steps=10,
                         lr_scheduler="constant", precision="fp32",
                         checkpoint_dir=str(tmp_path))
    tr = Trainer(model, cfg, device="cpu")
    ids = torch.randint(0, 256, (2, 16), generator=torch.Generator().manual_seed(1))
    l0 = tr.train_step(ids)
    for _ in range(8):
        l1 = tr.train_step(ids)
    assert l1 < l0
    tr.save_checkpoint()


def test_zeroth_power_newton_schulz():
    import pytest

    from complexity_framework_b200.training.optimizers import zeroth_power_newton_schulz

    torch.manual_seed(0)
    m = torch.randn(32, 16)
    o = zeroth_power_newton_schulz(m)
    assert o.shape == m.shape
    # singular values pushed into the quintic's band around 1
    s = torch.linalg.svdvals(o)
    assert s.min() > 0.5 and s.max() < 1.3
    with pytest.raises(ValueError):
        zeroth_power_newton_schulz(torch.randn(2, 3, 4))
