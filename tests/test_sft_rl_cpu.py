"""SFT entry (full and LoRA) and GRPO/DAPO on CPU."""
import json

import torch

from complexity_framework_b200 import ComplexityModel, ModelConfig
from complexity_framework_b200.data import ByteTokenizer
from complexity_framework_b200.rl import (GRPOConfig, GRPOTrainer, dapo_loss, group_advantages,
                                          mcq_exact_match_reward)
from complexity_framework_b200.training import sft


def _model(vocab):
    torch.manual_seed(0)
    return ComplexityModel(ModelConfig(hidden_size=64, num_hidden_layers=1, num_attention_heads=4,
                                       num_key_value_heads=2, vocab_size=vocab,
                                       intermediate_size=64, shared_intermediate_size=128,
                                       num_experts=4, top_k=2, routing_strategy="modulo_cyclic",
                                       max_position_embeddings=512))


def test_sft_full_and_lora(tmp_path):
    tok = ByteTokenizer()
    _model(tok.vocab_size).save_pretrained(tmp_path / "m")
    rows = [{"messages": [{"role": "user", "content": f"q{i}"},
                          {"role": "assistant", "content": f"answer {i}"}]} for i in range(8)]
    (tmp_path / "d.jsonl").write_text("\n".join(json.dumps(r) for r in rows))
    s = sft.main(["--model", str(tmp_path / "m"), "--data", str(tmp_path / "d.jsonl"),
                  "--output", str(tmp_path / "o"), "--batch-size", "4", "--epochs", "2",
                  "--precision", "fp32", "--lr", "1e-3", "--eval-data", str(tmp_path / "d.jsonl")])
    assert s["steps"] == 4 and "eval_loss" in s
    assert (tmp_path / "o" / "final" / "config.json").exists()
    s2 = sft.main(["--model", str(tmp_path / "m"), "--data", str(tmp_path / "d.jsonl"),
                   "--output", str(tmp_path / "o2"), "--batch-size", "4", "--lora-rank", "4",
                   "--precision", "fp32", "--pack", "--seq-len", "128"])
    assert (tmp_path / "o2" / "adapter.pt").exists() and s2["steps"] >= 1


def test_advantages_and_dapo():
    r = torch.tensor([1.0, 0.0, 0.0, 1.0, 2.0, 2.0, 2.0, 2.0])
    a = group_advantages(r, 4)
    assert abs(float(a[:4].mean())) < 1e-6 and torch.allclose(a[4:], torch.zeros(4))
    lp = torch.zeros(2, 3, requires_grad=True)
    loss = dapo_loss(lp, torch.zeros(2, 3), torch.tensor([1.0, -1.0]), torch.ones(2, 3), 0.2, 0.28)
    loss.backward()
    assert float(loss) == 0.0 and lp.grad is not None


def test_grpo_step_runs():
    tok = ByteTokenizer()
    m = _model(tok.vocab_size)
    tr = GRPOTrainer(m, tok, GRPOConfig(group_size=4, max_new_tokens=4, lr=1e-3, kl_coef=0.01),
                     reward_fn=lambda comps, ans: [float(len(c) % 2) for c in comps])
    st = tr.step(["2+2?", "B or C?"], answers=["A", "B"])
    assert "reward_mean" in st and st["groups_kept"] >= 0
    assert mcq_exact_match_reward(["The answer is B.", "C"], "B") == [1.0, 0.0]
