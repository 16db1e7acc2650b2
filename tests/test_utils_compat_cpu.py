"""Reference-named utility entry points: schedulers, local checkpoints,
training state, activation checkpointing, Hugging Face directory conversion."""
import pytest
import torch

from complexity_framework_b200 import ComplexityModel, ModelConfig


def _m(**kw):
    torch.manual_seed(0)
    base = dict(hidden_size=32, num_hidden_layers=2, num_attention_heads=4,
                num_key_value_heads=2, vocab_size=64, intermediate_size=32,
                shared_intermediate_size=64, num_experts=2, top_k=2, max_position_embeddings=32)
    base.update(kw)
    return ComplexityModel(ModelConfig(**base))


def test_scheduler_names():
    from complexity_framework_b200.training import TrainingConfig
    from complexity_framework_b200.training.scheduler import get_lr_scheduler, resolve_scheduler_name

    cfg = TrainingConfig(lr_scheduler="auto", warmup_steps=2, max_steps=10)
    assert resolve_scheduler_name(cfg) == "cosine"
    opt = torch.optim.SGD([torch.nn.Parameter(torch.zeros(1))], lr=1.0)
    s = get_lr_scheduler(opt, cfg)
    lrs = []
    for _ in range(10):
        lrs.append(opt.param_groups[0]["lr"])
        opt.step()
        s.step()
    assert lrs[0] < lrs[2] and lrs[-1] < lrs[2]
    with pytest.raises(ValueError):
        get_lr_scheduler(opt)


def test_local_checkpoints(tmp_path):
    from complexity_framework_b200.utils.local_checkpoint import (load_local_checkpoint,
                                                                  save_local_checkpoint)

    for s in (1, 2, 3, 4):
        save_local_checkpoint(tmp_path, step=s, state={"step": s}, total_limit=2)
    assert sorted(p.name for p in tmp_path.glob("step_*")) == ["step_000003", "step_000004"]
    d, st = load_local_checkpoint(tmp_path / "latest")
    assert d.name == "step_000004" and st["step"] == 4


def test_training_state_and_activation_checkpointing():
    from complexity_framework_b200.utils.checkpointing import (TrainingState,
                                                               checkpoint_sequential,
                                                               enable_activation_checkpointing)

    st = TrainingState(step=3, best_loss=1.5)
    assert TrainingState.from_dict({**st.to_dict(), "unknown": 1}) == st
    m = _m()
    ids = torch.randint(0, 64, (1, 8))
    want = m.loss(ids)
    enable_activation_checkpointing(m)
    got = m.loss(ids)
    got.backward()
    assert torch.allclose(got, want)
    seq = [torch.nn.Linear(4, 4), torch.nn.Tanh(), torch.nn.Linear(4, 4)]
    x = torch.randn(2, 4, requires_grad=True)
    y = checkpoint_sequential(seq, x, segments=2)
    assert torch.allclose(y, seq[2](seq[1](seq[0](x))))


def test_huggingface_directory_roundtrip(tmp_path):
    from complexity_framework_b200.utils.conversion import (load_from_huggingface, push_to_hub,
                                                            save_to_huggingface)

    src = _m()
    save_to_huggingface(src, tmp_path / "hf")
    dst = _m()
    torch.manual_seed(5)
    for p in dst.parameters():
        p.data.normal_()
    load_from_huggingface(str(tmp_path / "hf"), dst)
    a, b = src.state_dict(), dst.state_dict()
    assert torch.equal(a["layers.0.self_attn.q_proj.weight"], b["layers.0.self_attn.q_proj.weight"])
    with pytest.raises(FileNotFoundError):
        load_from_huggingface("org/model-on-hub", dst)
    with pytest.raises(RuntimeError, match="network"):
        push_to_hub(src, "x")
