"""Stacked SFT: config validation, file-backed mix building (three record
formats, Unicode line separators, counts), and a two-stage chained LoRA run on
a tiny model (each stage merges its adapter and the next stage loads it)."""
import json
from pathlib import Path

import pytest
import torch

from complexity_framework_b200.training.stack_sft import (DatasetMix, SourceConfig,
                                                           StackSFTConfig,
                                                           StackSFTDatasetBuilder,
                                                           StackSFTRunner)


def _jsonl(path: Path, rows):
    path.write_text("".join(json.dumps(r, ensure_ascii=False) + "\n" for r in rows),
                    encoding="utf-8")
    return path


def test_config_validation():
    with pytest.raises(ValueError, match="hardcoded synthetic"):
        DatasetMix.from_dict({"records": 8, "sources": {"final": 1.0}})
    with pytest.raises(ValueError, match="missing weight"):
        SourceConfig.from_dict({"name": "a"})
    with pytest.raises(ValueError, match="at least one stage"):
        StackSFTConfig.from_dict({"name": "x", "base_checkpoint": "b", "stages": []})
    stage = {"name": "s1", "steps": 2, "lr": 1e-3,
             "mix": {"records": 4, "sources": [{"name": "a", "path": "a.jsonl", "weight": 1}]}}
    with pytest.raises(ValueError, match="positive LoRA rank"):
        StackSFTConfig.from_dict({"name": "x", "base_checkpoint": "b", "lora_rank": 0,
                                  "stages": [stage]})
    cfg = StackSFTConfig.from_dict({"name": "x", "base_checkpoint": "b", "stages": [stage]})
    assert cfg.lora_rank == 64 and cfg.stages[0].mix.sources[0].weight == 1.0


def test_builder_formats_counts_and_unicode(tmp_path):
    general = _jsonl(tmp_path / "g.jsonl", [
        {"prompt": "User:\nHello\n\nAssistant:\n", "completion": "Hello!"},
        {"instruction": "Explain gravity", "output": "Gravity pulls masses together."}])
    code = _jsonl(tmp_path / "c.jsonl", [
        {"instruction": "Write Python that adds two numbers.", "input": "Use a function.",
         "output": "def add(a, b):\n    return a + b"}])
    msgs = _jsonl(tmp_path / "m.jsonl", [
        {"messages": [{"role": "user", "content": "What is 2+2?"},
                      {"role": "assistant", "content": "4"}]},
        {"messages": [{"role": "user", "content": "no answer"}]}])
    uni = _jsonl(tmp_path / "u.jsonl", [{"prompt": "User:\nA B\n\nAssistant:\n",
                                         "completion": "C"}])
    mix = DatasetMix(records=13, seed=1, sources=[
        SourceConfig(name="g", path=str(general), weight=0.5),
        SourceConfig(name="c", path=str(code), weight=0.25),
        SourceConfig(name="m", path=str(msgs), weight=0.125),
        SourceConfig(name="u", path=str(uni), weight=0.125)])
    counts = [n for _, n in StackSFTDatasetBuilder.counts(mix)]
    assert sum(counts) == 13 and counts[1:] == [3, 1, 1]
    out = StackSFTDatasetBuilder().build(mix, tmp_path / "mix.jsonl")
    lines = [l for l in out.read_text(encoding="utf-8").split("\n") if l]
    assert len(lines) == 13
    rows = [json.loads(l) for l in lines]
    text = "\n".join(r["prompt"] + r["completion"] for r in rows)
    assert "def add(a, b):" in text and "User:\nWhat is 2+2?" in text
    assert any(r["completion"] == "C" for r in rows)
    with pytest.raises(ValueError, match="must define a JSONL/parquet path"):
        StackSFTDatasetBuilder().build(
            DatasetMix(records=1, sources=[SourceConfig(name="x", weight=1.0)]), tmp_path / "x")


def test_two_stage_chain(tmp_path):
    from complexity_framework_b200 import ComplexityModel, ModelConfig

    torch.manual_seed(0)
    base = ComplexityModel(ModelConfig(hidden_size=64, num_hidden_layers=2, num_attention_heads=4,
                                       num_key_value_heads=2, vocab_size=260,
                                       intermediate_size=64, shared_intermediate_size=128,
                                       num_experts=2, top_k=2, max_position_embeddings=64))
    base.save_pretrained(tmp_path / "base")
    src = _jsonl(tmp_path / "d.jsonl", [{"prompt": f"q{i}", "completion": f"a{i}"}
                                        for i in range(8)])
    recipe = {"name": "t", "base_checkpoint": str(tmp_path / "base"), "tokenizer": "byte",
              "output_dir": str(tmp_path / "out"), "data_dir": str(tmp_path / "data"),
              "batch_size": 4, "seq_len": 32, "lora_rank": 4, "lora_alpha": 8, "bf16": False,
              "stages": [{"name": f"s{k}", "steps": 2, "lr": 1e-2,
                          "mix": {"records": 8, "seed": k,
                                  "sources": [{"name": "d", "path": str(src), "weight": 1}]}}
                         for k in (1, 2)]}
    (tmp_path / "r.yaml").write_text(json.dumps(recipe))  # JSON is valid YAML
    runner = StackSFTRunner.from_yaml(tmp_path / "r.yaml")
    final = runner.run()
    assert final.endswith("t-s2/final")
    m1 = ComplexityModel.from_pretrained(tmp_path / "out" / "t-s1" / "final")
    m2 = ComplexityModel.from_pretrained(final)
    w0 = base.layers[0].self_attn.q_proj.weight
    w1, w2 = (m.layers[0].self_attn.q_proj.weight for m in (m1, m2))
    assert not torch.equal(w0, w1) and not torch.equal(w1, w2)  # each stage trained on
    assert set(m2.state_dict()) == set(base.state_dict())       # plain checkpoint format
    summary = json.loads((tmp_path / "out" / "t-s2" / "sft_summary.json").read_text())
    assert summary["steps"] == 2
