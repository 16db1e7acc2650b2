"""Chat-template contract: validation, rendering, Jinja export (CPU)."""
import json

import pytest

from complexity_framework_b200.inference import chat_template as ct


def test_default_renders_and_validates(tmp_path):
    t = ct.default_chat_template()
    assert ct.validate_chat_template(t) == t
    assert ct.render_inference_prompt(" hi ", t) == "User:\nhi\n\nAssistant:\n"
    assert ct.render_thinking_inference_prompt("hi", t).endswith("Assistant:\n<think>\n")
    assert ct.render_assistant_envelope(" r ", " f ", t) == \
        "<think>\nr\n</think>\n<final>\nf\n</final>"
    p = ct.save_chat_template(t, tmp_path)
    assert p.name == "chat_template.json"
    assert ct.load_chat_template(tmp_path) == t
    assert ct.load_chat_template(tmp_path / "nothing") == ct.default_chat_template()


@pytest.mark.parametrize("bad", [dict(id="other"), dict(assistant_only_loss=False),
                                 dict(user_format="User:"), dict(training_projection="x"),
                                 dict(assistant_envelope=None)])
def test_validation_rejects(bad):
    t = dict(ct.default_chat_template(), **bad)
    with pytest.raises(ValueError):
        ct.validate_chat_template(t)
    with pytest.raises(ValueError):
        ct.validate_chat_template({k: v for k, v in t.items() if k != "eos_token"})


def test_messages_system_rules():
    v2 = dict(ct.default_chat_template(), system_prompt="Be brief.")
    msgs = [{"role": "system", "content": "Custom"}, {"role": "user", "content": "a"},
            {"role": "assistant", "content": "b"}, {"role": "user", "content": "c"}]
    out = ct.render_messages_before_assistant(msgs, v2)
    assert out == ("System:\nCustom\n\nUser:\na\n\nAssistant:\nb<|endoftext|>"
                   "User:\nc\n\nAssistant:\n")
    v1 = dict(v2, id=ct.LEGACY_CHAT_TEMPLATE_ID)
    assert ct.render_messages_before_assistant(msgs, v1).startswith("System:\nBe brief.\n\nUser:")
    with pytest.raises(ValueError):
        ct.render_messages_before_assistant([{"role": "tool", "content": "x"}], v2)


@pytest.mark.parametrize("template_id", [ct.CHAT_TEMPLATE_ID, ct.LEGACY_CHAT_TEMPLATE_ID])
def test_jinja_export_matches_python_renderer(template_id, tmp_path):
    t = dict(ct.default_chat_template(), id=template_id, system_prompt="Sys")
    src = ct.huggingface_chat_template(t)
    msgs = [{"role": "user", "content": " q1 "}, {"role": "assistant", "content": "a1"},
            {"role": "user", "content": "q2"}]
    got = ct.render_jinja_messages(msgs, src, eos_token=t["eos_token"],
                                   add_generation_prompt=True)
    assert got == ct.render_messages_before_assistant(msgs, t)
    (tmp_path / "chat_template.jinja").write_text(src)
    assert ct.load_chat_template_jinja(tmp_path) == src
    assert ct.render_jinja_inference_prompt("x", src, eos_token="</s>") == \
        ct.render_inference_prompt("x", t)
    think = ct.huggingface_chat_template(t, force_thinking=True)
    assert ct.render_jinja_inference_prompt("x", think, eos_token="</s>").endswith("<think>\n")
    aligned = ct.align_chat_template_eos(t, eos_token="</s>")
    assert aligned["eos_token"] == "</s>" and json.dumps(aligned)
