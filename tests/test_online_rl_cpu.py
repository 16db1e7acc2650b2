"""Shared online RL loop: monitoring, batched update, checkpoint rotation (CPU)."""
import json

import torch

from complexity_framework_b200 import ComplexityModel, ModelConfig
from complexity_framework_b200.data.tokenization import ByteTokenizer
from complexity_framework_b200.rl import SharedOnlineRLConfig, SharedOnlineRLLoop


def _model():
    torch.manual_seed(0)
    return ComplexityModel(ModelConfig(hidden_size=64, num_hidden_layers=2, num_attention_heads=4,
                                       num_key_value_heads=2, vocab_size=300,
                                       intermediate_size=64, shared_intermediate_size=128,
                                       num_experts=4, top_k=2, routing_strategy="modulo_cyclic"))


def test_loop_monitors_updates_and_rotates(tmp_path):
    m = _model()
    cfg = SharedOnlineRLConfig(output_dir=str(tmp_path), min_events_before_update=3,
                               max_new_tokens=4, learning_rate=1e-3, keep_last_n_checkpoints=2,
                               entropy_trigger=1e9, confidence_trigger=-1.0)
    loop = SharedOnlineRLLoop(m, ByteTokenizer(), config=cfg)
    before = [p.detach().clone() for p in m.parameters()]
    # plain request without feedback: served, not monitored
    _, stats, ck = loop.infer("hello")
    assert stats is None and ck is None and not loop.pending_events
    loop.infer("hi", user_feedback="that is wrong")
    assert loop.pending_events[-1].reward == cfg.negative_reward
    loop.infer("Q: calculate 6*7")   # verified calculator episode, reward 1
    ev = loop.pending_events[-1]
    assert ev.reward == 1.0 and ev.target_response.endswith("Assistant:\n42")
    _, stats, ck = loop.infer("yo", user_feedback="incorrect")
    assert stats["num_events"] == 3.0 and ck is not None and (ck / "model.pt").exists()
    assert not loop.pending_events
    assert any(not torch.equal(a, b) for a, b in zip(before, m.parameters()))
    assert (tmp_path / cfg.current_pointer_name).read_text() == str(ck)
    lines = (tmp_path / cfg.monitor_log_name).read_text().splitlines()
    assert len(lines) == 3 and json.loads(lines[0])["feedback"] == "that is wrong"
    for i in range(2):
        loop.infer("again", force_monitor=True, force_update=True)
    names = sorted(p.name for p in tmp_path.iterdir() if p.is_dir())
    assert names == ["checkpoint_online_rl_000002", "checkpoint_online_rl_000003"]
    # a new loop on the same directory continues the numbering
    assert SharedOnlineRLLoop(m, ByteTokenizer(), config=cfg).rl_step == 4


def test_reward_rules():
    loop = SharedOnlineRLLoop.__new__(SharedOnlineRLLoop)
    loop.config = SharedOnlineRLConfig()
    assert loop.compute_reward("Correct!", None, None) == 1.0
    assert loop.compute_reward("incorrect", None, None) == -1.0
    assert loop.compute_reward(None, 9.0, 0.9) == loop.config.uncertainty_reward
    assert loop.compute_reward(None, 1.0, 0.9) == 0.0
