"""SFT depth on CPU: curriculum selection and task weights, early stopping with
best-checkpoint selection, per-epoch resume with RNG states, and data-parallel
SFT over two gloo ranks."""
import json
import os
import socket

import pytest
import torch
import torch.multiprocessing as mp

from complexity_framework_b200 import ComplexityModel, ModelConfig
from complexity_framework_b200.data import ByteTokenizer
from complexity_framework_b200.training import sft
from complexity_framework_b200.training.sft_curriculum import (CurriculumStage, load_curriculum,
                                                               select_examples)


def _setup(tmp_path, n=12):
    tok = ByteTokenizer()
    torch.manual_seed(0)
    ComplexityModel(ModelConfig(hidden_size=64, num_hidden_layers=1, num_attention_heads=4,
                                num_key_value_heads=2, vocab_size=tok.vocab_size,
                                intermediate_size=64, shared_intermediate_size=128,
                                num_experts=4, top_k=2, routing_strategy="modulo_cyclic",
                                max_position_embeddings=256)).save_pretrained(tmp_path / "m")
    rows = [{"task": ("math" if i % 3 == 0 else "chat"),
             "difficulty": ("hard" if i % 4 == 0 else "easy"),
             "messages": [{"role": "user", "content": f"question {i}"},
                          {"role": "assistant", "content": f"answer {i % 5}"}]}
            for i in range(n)]
    (tmp_path / "d.jsonl").write_text("\n".join(json.dumps(r) for r in rows))
    return rows


def _args(tmp_path, out, *extra):
    return ["--model", str(tmp_path / "m"), "--data", str(tmp_path / "d.jsonl"),
            "--output", str(tmp_path / out), "--batch-size", "2", "--precision", "fp32",
            "--lr", "1e-3", *extra]


def test_curriculum_selection_is_deterministic(tmp_path):
    rows = _setup(tmp_path, 30)
    (tmp_path / "c.yaml").write_text(
        "seed: 3\nstages:\n"
        "  - name: easy_chat\n    tasks: [chat]\n    difficulties: [easy]\n"
        "    max_repeats_per_response: 2\n"
        "  - name: sample\n    exclude_tasks: [math]\n    max_examples: 5\n"
        "    task_weights: {chat: 2.5}\n")
    cur = load_curriculum(str(tmp_path / "c.yaml"))
    easy = select_examples(rows, cur.stage("easy_chat"), seed=cur.seed)
    assert all(rows[i]["task"] == "chat" and rows[i]["difficulty"] == "easy" for i in easy)
    answers = [rows[i]["messages"][1]["content"] for i in easy]
    assert max(answers.count(a) for a in answers) <= 2          # response cap
    s1 = select_examples(rows, cur.stage("sample"), seed=cur.seed)
    assert len(s1) == 5 and s1 == select_examples(rows, cur.stage("sample"), seed=cur.seed)
    assert cur.stage("sample").task_weight("chat") == 2.5
    assert cur.stage("sample").task_weight("other") == 1.0
    with pytest.raises(ValueError, match="unknown keys"):
        CurriculumStage.from_dict({"name": "x", "bogus": 1})
    lens = [(10 + i, 5 + i) for i in range(len(rows))]
    short = select_examples(rows, CurriculumStage(name="s", max_num_tokens=15), token_counts=lens)
    assert short == [0, 1, 2, 3, 4, 5]


def test_weighted_loss_matches_unweighted_when_weights_are_one():
    torch.manual_seed(0)
    m = ComplexityModel(ModelConfig(hidden_size=64, num_hidden_layers=1, num_attention_heads=4,
                                    num_key_value_heads=2, vocab_size=256, intermediate_size=64,
                                    shared_intermediate_size=128, num_experts=4, top_k=2,
                                    max_position_embeddings=64))
    ids = torch.randint(0, 256, (2, 16))
    labels = torch.roll(ids, -1, 1)
    labels[:, -1] = -100
    packed = torch.stack([labels.double(), torch.ones_like(labels, dtype=torch.float64)], -1)
    a = sft.weighted_sft_loss(m, ids, packed)
    assert torch.allclose(a, m.loss(ids, labels), atol=1e-5)
    packed[0, :, 1] = 3.0            # row 0 three times as heavy
    b = sft.weighted_sft_loss(m, ids, packed)
    assert not torch.allclose(a, b)


def test_curriculum_stage_training_with_task_weights(tmp_path):
    _setup(tmp_path)
    (tmp_path / "c.yaml").write_text(
        "stages:\n  - name: s1\n    tasks: [chat]\n    task_weights: {chat: 2.0}\n")
    s = sft.main(_args(tmp_path, "o", "--curriculum", str(tmp_path / "c.yaml"),
                       "--curriculum-stage", "s1"))
    assert s["curriculum_stage"] == "s1" and s["examples"] == 8 and s["steps"] == 4


def test_early_stopping_and_best_checkpoint(tmp_path):
    _setup(tmp_path)
    # a learning rate this high makes held-out loss stop improving quickly
    s = sft.main(_args(tmp_path, "o", "--epochs", "30", "--eval-steps", "1", "--lr", "0.5",
                       "--eval-data", str(tmp_path / "d.jsonl"), "--early-stopping-patience",
                       "2", "--early-stopping-min-epochs", "0", "--save-best"))
    assert s["stopped_early"] and s["steps"] < 30 * 6
    best = json.loads((tmp_path / "o" / "best.json").read_text())
    assert best["eval_loss"] == pytest.approx(min(h["eval_loss"] for h in s["eval_history"]))
    assert os.path.isdir(best["checkpoint"])


def test_resume_from_epoch_checkpoint_continues_exactly(tmp_path):
    import shutil

    _setup(tmp_path)
    full = sft.main(_args(tmp_path, "run", "--epochs", "3"))
    assert full["steps"] == 18
    want = torch.load(tmp_path / "run" / "epoch-18" / "checkpoint.pt", weights_only=False)["model"]
    st = json.loads((tmp_path / "run" / "epoch-6" / "sft_state.json").read_text())
    assert st["epoch"] == 1 and st["step_in_epoch"] == 0
    assert (tmp_path / "run" / "epoch-6" / "rng_states.pt").exists()
    # lose everything after the first epoch, then resume from its checkpoint
    shutil.rmtree(tmp_path / "run" / "epoch-12")
    shutil.rmtree(tmp_path / "run" / "epoch-18")
    resumed = sft.main(_args(tmp_path, "run", "--epochs", "3", "--resume",
                             str(tmp_path / "run" / "epoch-6")))
    assert resumed["steps"] == 18
    got = torch.load(tmp_path / "run" / "epoch-18" / "checkpoint.pt", weights_only=False)["model"]
    for k in want:
        assert torch.allclose(want[k], got[k], atol=1e-6), k


def _port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


def _ddp_rank(rank, world, port, tmp):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), RANK=str(rank),
                      WORLD_SIZE=str(world), LOCAL_RANK=str(rank), CUDA_VISIBLE_DEVICES="")
    from pathlib import Path

    s = sft.main(_args(Path(tmp), "ddp", "--epochs", "2"))
    torch.save({"steps": s["steps"]}, os.path.join(tmp, f"ddp_rank{rank}.pt"))


def test_data_parallel_sft_two_ranks(tmp_path):
    _setup(tmp_path)
    port = _port()
    ctx = mp.get_context("spawn")
    procs = [ctx.Process(target=_ddp_rank, args=(r, 2, port, str(tmp_path))) for r in range(2)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(240)
    assert [p.exitcode for p in procs] == [0, 0]
    steps = [torch.load(tmp_path / f"ddp_rank{r}.pt")["steps"] for r in range(2)]
    # 12 examples, 2 per rank per step over 2 ranks: 3 steps per epoch on both ranks
    assert steps == [6, 6]
    assert (tmp_path / "ddp" / "final" / "model.safetensors").exists()
