"""Portable chat-template contract shared by SFT, export and inference.

Counterpart: complexity/inference/chat_template.py:1-332.  A template is a
JSON-able dict (``chat_template.json`` beside a model bundle); the field names,
the two template ids, the think/final envelope strings and the rendered text
are a format other tools read, so they match the counterpart exactly.  The
code is independent: rendering goes through one ``_turns`` generator that both
the Python renderer and the exported Jinja source follow, and the Jinja source
is produced by a small builder rather than string splicing per branch.
"""
from __future__ import annotations

import json
from pathlib import Path
from typing import Any, Dict, Iterable, Iterator, List, Optional

CHAT_TEMPLATE_ID = "complexity-chat-v2"
LEGACY_CHAT_TEMPLATE_ID = "complexity-chat-v1"
SUPPORTED_CHAT_TEMPLATE_IDS = frozenset({LEGACY_CHAT_TEMPLATE_ID, CHAT_TEMPLATE_ID})
SUPPORTED_TRAINING_PROJECTIONS = frozenset({
    "naturalize_card_hand_preserve_assistant_turns",
    "naturalize_card_hand_target_final_assistant",
    "naturalize_card_hand_supervise_all_assistant_turns",
    "card_corpus_v2_direct",
})
THINK_FINAL_ENVELOPE: Dict[str, str] = {
    "type": "optional_think_final",
    "think_start": "<think>\n",
    "think_end": "\n</think>",
    "final_start": "\n<final>\n",
    "final_end": "\n</final>",
    "scope": "reasoning_tasks",
}
REQUIRED_FIELDS = ("id", "version", "system_prompt", "system_format", "user_format",
                   "assistant_prefix", "turn_separator", "eos_token", "assistant_only_loss",
                   "training_projection")


def default_chat_template() -> Dict[str, Any]:
    return dict(id=CHAT_TEMPLATE_ID, version=2, system_prompt="",
                system_format="System:\n{content}\n\n", user_format="User:\n{content}\n\n",
                assistant_prefix="Assistant:\n", turn_separator="\n\n",
                eos_token="<|endoftext|>", assistant_only_loss=True,
                training_projection="naturalize_card_hand_supervise_all_assistant_turns",
                assistant_envelope=dict(THINK_FINAL_ENVELOPE))


def validate_chat_template(template: Dict[str, Any]) -> Dict[str, Any]:
    missing = [f for f in REQUIRED_FIELDS if f not in template]
    if missing:
        raise ValueError(f"Chat template is missing fields: {', '.join(missing)}")
    if template["id"] not in SUPPORTED_CHAT_TEMPLATE_IDS:
        raise ValueError(f"Unsupported chat template: {template['id']}")
    if template["id"] == CHAT_TEMPLATE_ID and template.get("assistant_envelope") != THINK_FINAL_ENVELOPE:
        raise ValueError("complexity-chat-v2 requires the canonical think/final protocol")
    if not template["assistant_only_loss"]:
        raise ValueError("SFT requires assistant_only_loss=true")
    if template["training_projection"] not in SUPPORTED_TRAINING_PROJECTIONS:
        raise ValueError(f"Unsupported SFT training projection: {template['training_projection']}")
    for f in ("system_format", "user_format"):
        if "{content}" not in template[f]:
            raise ValueError(f"Chat template {f} must contain {{content}}")
    return dict(template)


def align_chat_template_eos(template: Dict[str, Any], *, eos_token: str) -> Dict[str, Any]:
    """Use the loaded tokenizer's spelling of EOS (the contract is the EOS id)."""
    if not isinstance(eos_token, str) or not eos_token:
        raise ValueError("chat-template EOS alignment requires a non-empty token")
    out = validate_chat_template(template)
    out["eos_token"] = eos_token
    return out


def _bundle_file(path, name: str) -> Path:
    p = Path(path)
    return p / name if p.is_dir() else p


def load_chat_template(path=None) -> Dict[str, Any]:
    """The template of a bundle directory / JSON file; the default when absent."""
    if path is None:
        return default_chat_template()
    p = _bundle_file(path, "chat_template.json")
    if not p.exists():
        return default_chat_template()
    return validate_chat_template(json.loads(p.read_text(encoding="utf-8")))


def save_chat_template(template: Dict[str, Any], path) -> Path:
    p = _bundle_file(path, "chat_template.json")
    p.write_text(json.dumps(validate_chat_template(template), indent=2), encoding="utf-8")
    return p


def load_chat_template_jinja(path) -> str:
    p = _bundle_file(path, "chat_template.jinja")
    if not p.is_file():
        raise FileNotFoundError(f"Model bundle has no standalone Jinja chat template: {p}")
    src = p.read_text(encoding="utf-8")
    if not src.strip():
        raise ValueError(f"Jinja chat template is empty: {p}")
    return src


# ------------------------------------------------------------------ rendering
def _fmt(fmt: str, content: str) -> str:
    return fmt.format(content=content)


def render_system_prefix(template: Dict[str, Any]) -> str:
    s = str(template["system_prompt"]).strip()
    return _fmt(template["system_format"], s) if s else ""


def render_system_turn(content: str, template: Dict[str, Any]) -> str:
    c = content.strip()
    return _fmt(template["system_format"], c) if c else ""


def render_user_turn(content: str, template: Dict[str, Any]) -> str:
    return _fmt(template["user_format"], content.strip())


def render_inference_prompt(user_content: str, template: Dict[str, Any]) -> str:
    return (render_system_prefix(template) + render_user_turn(user_content, template)
            + template["assistant_prefix"])


def render_thinking_inference_prompt(user_content: str, template: Dict[str, Any]) -> str:
    """Inference prompt with the thinking envelope's opening prefilled."""
    env = validate_chat_template(template).get("assistant_envelope")
    if not env:
        raise ValueError("Chat template has no assistant envelope")
    return render_inference_prompt(user_content, template) + env["think_start"]


def _turns(messages: List[Dict[str, Any]], template: Dict[str, Any]) -> Iterator[str]:
    v2 = template["id"] == CHAT_TEMPLATE_ID
    norm = [(str(m.get("role", "")).strip().lower(), str(m.get("content", "")).strip())
            for m in messages]
    has_system = any(r == "system" and c for r, c in norm)
    # v1 always prints the template's system prompt; v2 prints it only when the
    # conversation brings no system turn of its own
    if not v2 or not has_system:
        yield render_system_prefix(template)
    for role, content in norm:
        if not content:
            continue
        if role == "system":
            if v2:
                yield render_system_turn(content, template)
        elif role == "user":
            yield render_user_turn(content, template)
        elif role == "assistant":
            yield template["assistant_prefix"] + content + template["eos_token"]
        else:
            raise ValueError(f"Unsupported chat role: {role}")


def render_messages_before_assistant(messages: Iterable[Dict[str, Any]],
                                     template: Dict[str, Any]) -> str:
    """Prior turns, ending at the next assistant prefix."""
    return "".join(_turns(list(messages), template)) + template["assistant_prefix"]


def render_assistant_envelope(reasoning: str, final: str, template: Dict[str, Any]) -> str:
    env = validate_chat_template(template).get("assistant_envelope")
    if not env:
        raise ValueError("Chat template has no assistant envelope")
    return (env["think_start"] + reasoning.strip() + env["think_end"] + env["final_start"]
            + final.strip() + env["final_end"])


# ---------------------------------------------------------------------- Jinja
def render_jinja_messages(messages: Iterable[Dict[str, Any]], jinja_source: str, *,
                          eos_token: str, add_generation_prompt: bool) -> str:
    """Render a standalone Jinja template the way HF tokenizers and vLLM do."""
    if not isinstance(eos_token, str) or not eos_token:
        raise ValueError("A non-empty tokenizer EOS token is required for Jinja rendering")
    from jinja2 import Environment, StrictUndefined

    env = Environment(autoescape=False, undefined=StrictUndefined, keep_trailing_newline=True)
    return env.from_string(jinja_source).render(messages=list(messages), eos_token=eos_token,
                                                add_generation_prompt=add_generation_prompt)


def render_jinja_inference_prompt(user_content: str, jinja_source: str, *,
                                  eos_token: str) -> str:
    return render_jinja_messages([{"role": "user", "content": user_content}], jinja_source,
                                 eos_token=eos_token, add_generation_prompt=True)


def huggingface_chat_template(template: Dict[str, Any], *, force_thinking: bool = False) -> str:
    """Jinja source equivalent to ``render_messages_before_assistant`` for HF /
    vLLM export.  EOS is Jinja's ``eos_token`` so the exported tokenizer's
    spelling of the EOS id is used."""
    t = validate_chat_template(template)
    q = json.dumps

    def wrap(fmt: str) -> str:
        pre, post = fmt.split("{content}", 1)
        return f"{{{{- {q(pre)} + (message['content'] | trim) + {q(post)} -}}}}"

    branches = []
    if t["id"] == CHAT_TEMPLATE_ID:
        branches.append(("system", wrap(t["system_format"])))
    branches.append(("user", wrap(t["user_format"])))
    branches.append(("assistant",
                     f"{{{{- {q(t['assistant_prefix'])} + (message['content'] | trim) + eos_token -}}}}"))
    body = "".join(("{%- if " if i == 0 else "{%- elif ") + f"message['role'] == '{r}' -%}}" + b
                   for i, (r, b) in enumerate(branches)) + "{%- endif -%}"
    gen = t["assistant_prefix"] + (t["assistant_envelope"]["think_start"]
                                   if force_thinking and t.get("assistant_envelope") else "")
    return (f"{{{{- {q(render_system_prefix(t))} -}}}}"
            "{%- for message in messages -%}" + body + "{%- endfor -%}"
            "{%- if add_generation_prompt -%}" + f"{{{{- {q(gen)} -}}}}" + "{%- endif -%}")


__all__ = [n for n in dir() if not n.startswith("_") and n not in (
    "annotations", "json", "Path", "Any", "Dict", "Iterable", "Iterator", "List", "Optional")]
