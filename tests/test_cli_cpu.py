"""CLI commands end to end on CPU (in-process)."""
import json

from complexity_framework_b200 import ComplexityModel, ModelConfig
from complexity_framework_b200.cli.app import main
from complexity_framework_b200.data import ByteTokenizer


def _ckpt(tmp_path):
    tok = ByteTokenizer()
    m = ComplexityModel(ModelConfig(hidden_size=64, num_hidden_layers=1, num_attention_heads=4,
                                    num_key_value_heads=2, vocab_size=tok.vocab_size,
                                    intermediate_size=64, shared_intermediate_size=128,
                                    num_experts=4, top_k=2, routing_strategy="modulo_cyclic",
                                    max_position_embeddings=256))
    m.save_pretrained(tmp_path / "m")
    return str(tmp_path / "m")


def test_cli_commands(tmp_path, capsys):
    ck = _ckpt(tmp_path)
    main(["info"])
    assert json.loads(capsys.readouterr().out)["framework"] == "complexity_framework_b200"
    main(["generate", "--model", ck, "--prompt", "hi", "--max-new-tokens", "3"])
    capsys.readouterr()
    main(["bench-infer", "--model", ck, "--batch", "2", "--prompt-len", "8", "--new-tokens", "3"])
    assert json.loads(capsys.readouterr().out.strip().splitlines()[-1])["batch"] == 2
    (tmp_path / "t.txt").write_text("hello world\nsecond line\n")
    main(["tokenize", "--input", str(tmp_path / "t.txt"), "--output", str(tmp_path / "shard")])
    assert json.loads(capsys.readouterr().out)["num_tokens"] > 20
    main(["convert", "to-gguf", ck, str(tmp_path / "m.gguf")])
    main(["convert", "to-hf", ck, str(tmp_path / "hf")])
    assert (tmp_path / "m.gguf").exists() and (tmp_path / "hf" / "config.json").exists()
    main(["profile", "model", "--model", ck, "--seq-len", "64"])
    assert "train_flops_per_token" in capsys.readouterr().out
    main(["plan", "--params", "200m", "--target-tokens", "70b", "--dp", "8"])
    assert "tokens_per_step" in capsys.readouterr().out
