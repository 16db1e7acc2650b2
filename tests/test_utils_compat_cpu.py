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


def _ref_ckpt(base, name, step, *, complete=True, has_state=True, marker="checkpoint.pt"):
    import json
    d = base / name
    d.mkdir(parents=True)
    if complete:
        (d / marker).write_bytes(b"x")
    if has_state:
        (d / "training_state.json").write_text(json.dumps({"step": step}))
    return d


def test_peek_reads_reference_layout_checkpoints(tmp_path):
    from complexity_framework_b200.utils.checkpointing import peek_latest_checkpoint_step

    assert peek_latest_checkpoint_step(tmp_path / "missing") is None
    assert peek_latest_checkpoint_step(tmp_path) is None
    _ref_ckpt(tmp_path, "token_pack_001_4133", 4133)
    (tmp_path / "token_pack_002_9999").mkdir()                # crashed mid-save
    assert peek_latest_checkpoint_step(tmp_path) == 4133
    _ref_ckpt(tmp_path, "token_pack_002_8265", 8265, has_state=False)   # step from the name
    _ref_ckpt(tmp_path, "interrupted_5000", 5000)
    assert peek_latest_checkpoint_step(tmp_path) == 8265
    other = tmp_path / "meta"
    _ref_ckpt(other, "step_500", 500, marker=".metadata")
    assert peek_latest_checkpoint_step(other) == 500


def test_peek_mixes_both_layouts(tmp_path):
    import torch

    from complexity_framework_b200.utils.checkpointing import (CheckpointManager,
                                                               peek_latest_checkpoint_step)

    m = torch.nn.Linear(2, 2)
    CheckpointManager(str(tmp_path)).save(m, None, step=9000, tag="step")
    _ref_ckpt(tmp_path, "token_pack_001_4133", 4133)
    assert peek_latest_checkpoint_step(tmp_path) == 9000
    (tmp_path / "step-12000").mkdir()      # ours, incomplete (no training state)
    assert peek_latest_checkpoint_step(tmp_path) == 9000
