"""GRPO script helpers: MMLU / FineWeb-Edu loading, prompt encoding, group
sampling, completion log-probabilities and the training driver on CPU."""
import json

import torch

from complexity_framework_b200 import ComplexityModel, ModelConfig
from complexity_framework_b200.data import ByteTokenizer
from complexity_framework_b200.rl import train_grpo as tg


def _model(vocab):
    torch.manual_seed(0)
    return ComplexityModel(ModelConfig(hidden_size=64, num_hidden_layers=1, num_attention_heads=4,
                                       num_key_value_heads=2, vocab_size=vocab,
                                       intermediate_size=64, shared_intermediate_size=128,
                                       num_experts=4, top_k=2, routing_strategy="modulo_cyclic",
                                       max_position_embeddings=512))


def _mmlu(tmp_path):
    p = tmp_path / "mmlu.jsonl"
    rows = [{"question": "2+2?", "choices": ["3", "4", "5", "6"], "answer": 1, "subject": "math"},
            {"question": "Sky colour?", "choices": ["red", "blue", "green", "black"],
             "answer": "B", "subject": "nature"}]
    p.write_text("\n".join(json.dumps(r) for r in rows))
    return p


def test_loaders_and_prompt(tmp_path):
    data = tg.load_mmlu_dataset(_mmlu(tmp_path))
    assert [d["answer"] for d in data] == ["B", "B"]
    assert "Question (math):\n2+2?" in data[0]["prompt"]
    assert "B. 4" in data[0]["prompt"] and data[0]["prompt"].endswith("Answer:")
    assert len(tg.load_mmlu_dataset(_mmlu(tmp_path), subset="nature")) == 1
    fw = tmp_path / "fw.jsonl"
    fw.write_text(json.dumps({"text": " ".join(f"w{i}" for i in range(100))}) + "\n"
                  + json.dumps({"text": "too short"}))
    d = tg.load_fineweb_edu_dataset(fw, prompt_words=10)
    assert len(d) == 1 and d[0]["prompt"].split() == [f"w{i}" for i in range(10)]


def test_encode_decode_and_rewards():
    tok = ByteTokenizer()
    ids = tg.encode_prompt(tok, "hello world", max_len=5)
    assert ids.shape == (5,)
    assert tg.decode_tokens(tok, ids) == tok.decode(tok.encode("hello world")[-5:])
    assert tg.mmlu_reward([" B. 4", "A", "nothing"], "B") == [1.0, 0.0, 0.0]


def test_group_and_log_probs():
    tok = ByteTokenizer()
    m = _model(tok.vocab_size)
    prompt = tg.encode_prompt(tok, "Q: x", max_len=32)
    ids = tg.generate_group(m, prompt, group_size=3, max_new_tokens=4, seed=1)
    assert ids.shape[0] == 3 and ids.shape[1] <= prompt.numel() + 4
    assert torch.equal(ids[:, :prompt.numel()], prompt.expand(3, -1))
    lp = tg.compute_log_probs(m, ids, prompt.numel())
    assert lp.shape == (3,) and not lp.requires_grad
    # matches an fp32 full-sequence reference
    with torch.no_grad():
        logits = m(ids)["logits"].float().log_softmax(-1)
    P = prompt.numel()
    for i in range(3):
        c = ids[i, P:]
        n = int((c != 0).sum())
        ref = logits[i, torch.arange(P - 1, P - 1 + n), c[:n]].sum()
        torch.testing.assert_close(lp[i], ref, rtol=1e-4, atol=1e-4)
    lpt = tg.compute_log_probs_trainable(m, ids, P)
    lpt.sum().backward()
    assert any(p.grad is not None for p in m.parameters())


def test_train_grpo_driver(tmp_path):
    tok = ByteTokenizer()
    m = _model(tok.vocab_size)
    data = tg.load_mmlu_dataset(_mmlu(tmp_path))
    cfg = tg.GRPOConfig(group_size=4, max_new_tokens=3, lr=1e-3, drop_uniform_groups=False)
    hist = tg.train_grpo(m, tok, data, steps=2, batch_prompts=2, config=cfg,
                         output=str(tmp_path / "out"))
    assert [h["step"] for h in hist] == [1, 2]
    assert (tmp_path / "out" / "final").is_dir()
    assert json.loads((tmp_path / "out" / "history.json").read_text())[1]["step"] == 2
