"""Behaviour regression gate: response checks, sandboxed code cases, the
PIQA floor, chat-report generation and PIQA scoring on a tiny model."""
import json

import pytest

from complexity_framework_b200.evaluation.regression_gate import (audit_regression, check_response,
                                                                  generate_chat_report,
                                                                  run_python_cases)

PANEL = {
    "schema_version": 1, "id": "tiny-panel",
    "generation": {"max_tokens": 4, "temperature": 0.0, "top_p": 1.0, "top_k": 0},
    "piqa": {"baseline_acc_norm": 0.70, "maximum_absolute_drop": 0.01, "examples": 2},
    "prompts": [
        {"id": "hi", "capability": "conversation", "prompt": "Hi!",
         "checks": {"required_any": ["hello", "hi"], "max_words": 10}},
        {"id": "mul", "capability": "math", "prompt": "12 x 11?",
         "checks": {"required_numbers": ["132"]}},
        {"id": "sq", "capability": "code", "prompt": "Write square(x).",
         "checks": {"python_function": "square",
                    "cases": [{"args": [3], "expected": 9}, {"args": [-2], "expected": 4}]}},
        {"id": "mem", "capability": "multi_turn_memory",
         "messages": [{"role": "user", "content": "My cat is Tom."},
                      {"role": "assistant", "content": "Noted."},
                      {"role": "user", "content": "Cat's name?"}],
         "checks": {"required_all": ["tom"]}},
        {"id": "bul", "capability": "instruction_constraints", "prompt": "Two tips.",
         "checks": {"exact_bullets": 2, "max_words_per_bullet": 4}},
    ],
}
GOOD = {"hi": "Hello there", "mul": "It is 132.", "sq": "```python\ndef square(x):\n    return x * x\n```",
        "mem": "Your cat is Tom.", "bul": "- drink water\n- sleep well"}


def test_checks():
    items = {i["id"]: i for i in PANEL["prompts"]}
    assert all(check_response(items[k], v) == [] for k, v in GOOD.items())
    assert check_response(items["hi"], "") == ["empty_response"]
    assert check_response(items["hi"], "good day " * 8)[0].startswith("missing_any")
    assert any(f.startswith("too_many_words") for f in check_response(items["hi"], "hi " * 11))
    assert check_response(items["mul"], "It is 1320.") == ["missing_number:132"]
    assert check_response(items["bul"], "- a\n- b\n- c") == ["bullet_count:3"]
    assert check_response(items["bul"], "- one two three four five\n- ok") == ["long_bullets:0"]


def test_code_sandbox():
    cases = [{"args": [3], "expected": 9}]
    assert run_python_cases("def square(x):\n    return x * x", "square", cases) is None
    assert run_python_cases("def square(x):\n    return x + x", "square", cases).startswith(
        "case_0_expected_9_got_6")
    assert run_python_cases("import os\ndef square(x):\n    return x*x", "square", cases) == \
        "unsafe_python_import"
    assert run_python_cases("import math\ndef square(x):\n    return int(math.pow(x, 2))",
                            "square", cases) is None
    assert run_python_cases("def square(x):\n    return x.__class__", "square", cases) == \
        "unsafe_dunder_access"
    assert run_python_cases("def square(x):\n    while True:\n        pass", "square", cases,
                            timeout_s=1.0) == "python_timeout:TimeoutError"
    assert run_python_cases("def sq(x):\n    return x", "square", cases) == \
        "missing_function:square"
    assert run_python_cases("def square(x) return", "square", cases).startswith("invalid_python")
    assert run_python_cases("open('f', 'w')\ndef square(x):\n    return x*x", "square",
                            cases) == "python_exec_error:NameError"


def test_audit_combines_behaviour_template_and_piqa():
    report = {"chat_template_applied": True,
              "results": [{"id": k, "response": v} for k, v in GOOD.items()]}
    ok = audit_regression(PANEL, report, {"benchmarks": {"piqa": {"acc_norm": 0.695}}})
    assert ok["passed"] and ok["piqa_threshold"] == pytest.approx(0.69)
    low = audit_regression(PANEL, report, {"benchmarks": {"piqa": {"acc_norm": 0.68}}})
    assert not low["passed"] and "piqa" in low["failures"]
    raw = audit_regression(PANEL, {**report, "chat_template_applied": False},
                           {"benchmarks": {"piqa": {"acc_norm": 0.9}}})
    assert raw["failures"] == {"chat_template": ["official_chat_template_not_applied"]}


def test_report_and_piqa_on_a_tiny_model(tmp_path):
    import torch

    from complexity_framework_b200 import ComplexityModel, ModelConfig
    from complexity_framework_b200.data import ByteTokenizer
    from complexity_framework_b200.evaluation import PIQABenchmark

    tok = ByteTokenizer()
    torch.manual_seed(0)
    m = ComplexityModel(ModelConfig(hidden_size=64, num_hidden_layers=1, num_attention_heads=4,
                                    num_key_value_heads=2, vocab_size=tok.vocab_size,
                                    intermediate_size=64, shared_intermediate_size=128,
                                    num_experts=4, top_k=2, routing_strategy="modulo_cyclic",
                                    max_position_embeddings=1024)).eval()
    rep = generate_chat_report(m, tok, PANEL)
    assert rep["chat_template_applied"] and [r["id"] for r in rep["results"]] == \
        [p["id"] for p in PANEL["prompts"]]
    p = tmp_path / "piqa.jsonl"
    p.write_text("\n".join(json.dumps(r) for r in [
        {"goal": "Dry wet hands", "sol1": "use a towel", "sol2": "use water", "label": 0},
        {"goal": "Open a jar", "sol1": "twist the lid", "sol2": "paint the lid", "label": 0}]))
    res = PIQABenchmark(str(p)).run(m, tok)
    assert res.num_samples == 2 and 0.0 <= res.accuracy <= 1.0
    assert set(res.details[-1]) == {"acc", "acc_norm"}


def _release_fixture(tmp_path, rows, ours=False):
    import csv
    ev, ck, mp = tmp_path / "eval", tmp_path / "ckpt", tmp_path / "metrics.csv"
    tmp_path.mkdir(parents=True, exist_ok=True)
    with mp.open("w", newline="") as fh:
        w = csv.DictWriter(fh, fieldnames=("step", "matched_eval_loss", "matched_eval_ppl"))
        w.writeheader()
        for step, _a, _n, loss, _p in rows:
            w.writerow({"step": step, "matched_eval_loss": loss, "matched_eval_ppl": 3.0})
    for e, (step, acc, accn, _l, passed) in enumerate(rows, start=1):
        d = ev / f"epoch_{e:02d}_step_{step:06d}"
        d.mkdir(parents=True)
        (d / "piqa.json").write_text(json.dumps({"checkpoint_step": step, "benchmarks": {
            "piqa": {"acc": acc, "acc_norm": accn, "correct": 1, "correct_norm": 1}}}))
        (d / "promotion.json").write_text(json.dumps({"passed": passed, "failures": {}}))
        c = ck / (f"step-{step}" if ours else f"step_{step:06d}")
        c.mkdir(parents=True)
        (c / ("training_state.json" if ours else "checkpoint.pt")).write_text("{}")
    return ev, mp, ck


def test_release_selection(tmp_path):
    from complexity_framework_b200.evaluation.release import select_release_checkpoint

    s = select_release_checkpoint(*_release_fixture(tmp_path / "a", [
        (100, 0.70, 0.70, 1.3, True), (200, 0.75, 0.75, 1.2, False),
        (300, 0.71, 0.72, 1.4, True)]), expected_epochs=3)
    assert s["release_ready"] and s["selected"]["step"] == 300
    assert s["candidates"][1]["promotion_passed"] is False
    s = select_release_checkpoint(*_release_fixture(tmp_path / "b", [
        (100, 0.70, 0.71, 1.3, True), (200, 0.70, 0.71, 1.1, True),
        (300, 0.69, 0.70, 1.0, True)], ours=True))
    assert s["selected"]["step"] == 200          # eval loss breaks the PIQA tie
    s = select_release_checkpoint(*_release_fixture(tmp_path / "c", [
        (100, 0.7, 0.7, 1.0, False), (200, 0.7, 0.7, 1.0, False)]))
    assert not s["release_ready"] and s["selected"] is None
    with pytest.raises(ValueError):
        select_release_checkpoint(*_release_fixture(tmp_path / "d", [(1, .5, .5, 1., True)]),
                                  expected_epochs=3)


@pytest.mark.parametrize("layout,dtype", [("ours", None), ("reference", "bfloat16")])
def test_export_release(tmp_path, layout, dtype):
    import torch
    from safetensors import safe_open

    from complexity_framework_b200 import ComplexityModel, ModelConfig
    from complexity_framework_b200.evaluation.release import export_release
    from complexity_framework_b200.utils.checkpointing import CheckpointManager

    cfg = ModelConfig(hidden_size=32, num_hidden_layers=1, num_attention_heads=2,
                      num_key_value_heads=1, vocab_size=64, intermediate_size=32,
                      shared_intermediate_size=64, num_experts=4, top_k=2,
                      routing_strategy="modulo_cyclic", max_position_embeddings=64)
    torch.manual_seed(0)
    m = ComplexityModel(cfg)
    if layout == "ours":
        ck = CheckpointManager(str(tmp_path / "ck")).save(m, None, step=200, tag="step")
    else:
        ck = tmp_path / "ck" / "step_000200"
        ck.mkdir(parents=True)
        torch.save({"step": 200, "model": m.state_dict(), "config": cfg.to_dict()},
                   ck / "checkpoint.pt")
    sel = {"epoch": 2, "step": 200, "checkpoint": str(ck), "promotion_passed": True,
           "piqa_acc": 0.69, "piqa_acc_norm": 0.70, "matched_eval_loss": 1.2,
           "matched_eval_ppl": 3.3}
    sp = tmp_path / "summary.json"
    sp.write_text(json.dumps({"release_ready": True, "selection_policy": "p", "selected": sel,
                              "candidates": [sel]}))
    tok = tmp_path / "tok"
    tok.mkdir()
    (tok / "tokenizer.json").write_text("{}")
    (tok / "tokenizer_config.json").write_text(json.dumps(
        {"eos_token": "</s>", "added_tokens_decoder": {"0": {"content": "</s>"}}}))
    out = tmp_path / "release"
    man = export_release(sp, out, tokenizer_dir=tok, weights_dtype=dtype)
    want = "bfloat16" if dtype else "float32"
    conf = json.loads((out / "config.json").read_text())
    assert conf["model_type"] == "tr_hash_moe" and conf["architectures"] == ["TRHashForCausalLM"]
    assert conf["num_experts_per_tok"] == 2 and conf["eos_token_id"] == 0
    assert conf["torch_dtype"] == want and man["weights_dtype"] == want
    assert man["selected_epoch"] == 2 and man["behavior_gate_passed"] and man["weights_sha256"]
    assert (out / "tokenizer.json").is_file() and "Apache-2.0" in (out / "README.md").read_text()
    with safe_open(str(out / "model.safetensors"), "pt") as f:
        assert f.metadata()["format"] == "pt"
        assert f.get_tensor("embed_tokens.weight").dtype == getattr(torch, want)
    # the release directory loads back as a model with the same config
    back = ComplexityModel.from_pretrained(str(out))
    assert back.config.num_experts == 4
    with pytest.raises(FileExistsError):
        export_release(sp, out)
