"""Grouped cfb commands (train / inference / tokenize / profile / info / quickstart)."""
import json

import numpy as np

from complexity_framework_b200.cli.app import main


def _json(capsys):
    return json.loads(capsys.readouterr().out)


def test_tokenize_group(tmp_path, capsys):
    main(["tokenize", "encode", "hello"])
    ids = _json(capsys)["ids"]
    main(["tokenize", "decode", *map(str, ids)])
    assert _json(capsys)["text"] == "hello"
    corpus = tmp_path / "c.jsonl"
    corpus.write_text("\n".join(json.dumps({"text": f"document number {i} " * 5})
                                for i in range(50)))
    main(["tokenize", "count", str(corpus)])
    c = _json(capsys)
    assert c["documents"] == 50 and c["tokens"] > 0
    main(["tokenize", "train", "--input", str(corpus), "--output", str(tmp_path / "bpe"),
          "--vocab-size", "300"])
    assert _json(capsys)["vocab_size"] <= 300
    main(["tokenize", "extend", str(tmp_path / "bpe" / "tokenizer.json"), "--tokens", "<|x|>",
          "--special"])
    e = _json(capsys)
    assert e["after"] == e["before"] + 1
    for d in ("s1", "s2"):
        main(["tokenize", "preprocess", "--input", str(corpus), "--output", str(tmp_path / d)])
        capsys.readouterr()
    main(["tokenize", "merge", str(tmp_path / "s1"), str(tmp_path / "s2"),
          "--output", str(tmp_path / "m")])
    merged = _json(capsys)
    main(["info", "tokens", str(tmp_path / "s1")])
    one = _json(capsys)
    assert merged["num_tokens"] == 2 * one["num_tokens"]


def test_info_train_inference_groups(tmp_path, capsys):
    main(["info", "version"])
    assert "torch" in _json(capsys)
    main(["info", "model", "tr-hash-200m"])
    assert _json(capsys)["parameters"] == 201_194_368
    main(["info", "benchmark-env"])
    assert "python" in _json(capsys)
    main(["train", "create-config", str(tmp_path / "run.yaml"), "--model", "tiny"])
    assert _json(capsys)["keys"] > 10
    main(["info", "config", "tr-hash-200m"])
    (tmp_path / "cfg.json").write_text(capsys.readouterr().out)
    main(["train", "validate", str(tmp_path / "cfg.json")])
    assert _json(capsys)["parameters"] == 201_194_368
    (tmp_path / "p.txt").write_text("hello\nworld\n")
    main(["inference", "batch", "--model", "tiny", "--input", str(tmp_path / "p.txt"),
          "--output", str(tmp_path / "o.jsonl"), "--max-new-tokens", "3", "--device", "cpu"])
    assert _json(capsys)["requests"] == 2
    rows = [json.loads(l) for l in (tmp_path / "o.jsonl").read_text().splitlines()]
    assert [r["prompt"] for r in rows] == ["hello", "world"]


def test_quickstart(capsys):
    main(["quickstart", "--steps", "3"])
    out = _json(capsys)
    assert out["trained_steps"] == 3 and isinstance(out["sample"], str)
