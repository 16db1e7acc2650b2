"""Reflect-then-tool agent loop for a local SFT checkpoint, and its eval.

    python -m complexity_framework_b200.rl.agentic_demo "What is 17 + 25?" --checkpoint ckpt/
    python -m complexity_framework_b200.rl.agentic_demo --checkpoint ckpt/ --eval

Counterpart of complexity/scripts/agentic_calculator_demo.py:42-387.  The
model first answers with a ``reflect`` tool call that restates the question;
the host pulls an arithmetic expression or a date operation out of it and
returns which tool applies; the model then calls that tool (``calculator`` or
``datetime``), and the host runs it in the sandboxed evaluators of
``rl.tool_rewards`` (whitelisted AST arithmetic, ISO-date operations).  The
tool-call text is ``<tool_call>{"name": ..., "arguments": {...}}</tool_call>``,
the same transcript format SFT and RL data use.

``parse_tool_call`` here is the strict parser of that loop: a malformed block
raises ``ToolCallParseError`` (the loop reports it), whereas
``rl.tool_rewards.parse_tool_call`` returns None so a reward can score it 0.
"""
from __future__ import annotations

import argparse
import json
import re
from dataclasses import dataclass
from typing import Any, Callable, Dict, List, Optional, Tuple

from .tool_rewards import (CalculatorError, DatetimeError, DatetimeHint,  # noqa: F401
                           extract_arithmetic_expression, extract_datetime_hint, safe_calculator,
                           safe_datetime)


class ToolCallParseError(ValueError):
    """A ``<tool_call>`` block that is not valid JSON or is not closed."""


@dataclass
class ToolCall:
    name: str
    arguments: Dict[str, Any]
    raw: str


_BLOCK = re.compile(r"<tool_call>\s*(.*?)\s*</tool_call>", re.S)


def parse_tool_call(text: str) -> Optional[ToolCall]:
    """The first tool call in ``text``; None when there is none."""
    m = _BLOCK.search(text)
    if m is None:
        if "<tool_call>" in text or "</tool_call>" in text:
            raise ToolCallParseError(f"unterminated tool call block in {text!r}")
        return None
    raw = m.group(1)
    try:
        obj = json.loads(raw)
    except json.JSONDecodeError as e:
        raise ToolCallParseError(f"tool call is not JSON: {raw!r}") from e
    if not isinstance(obj, dict):
        raise ToolCallParseError(f"tool call is not an object: {raw!r}")
    args = obj.get("arguments", {})
    return ToolCall(str(obj.get("name", "")), dict(args) if isinstance(args, dict) else {}, raw)


def engine_generator(model, tokenizer, max_new_tokens: int = 96, temperature: float = 0.2,
                     top_p: float = 0.9, seed: int = 0) -> Callable[[str], str]:
    """prompt -> completion text through the paged inference engine."""
    from ..inference.engine import GenerationConfig, InferenceEngine

    eng = InferenceEngine(model)
    gen = GenerationConfig(max_new_tokens=max_new_tokens, do_sample=temperature > 0,
                           temperature=max(temperature, 1e-5), top_p=top_p,
                           eos_token_id=getattr(tokenizer, "eos_token_id", None), seed=seed)

    def run(prompt: str) -> str:
        return tokenizer.decode(eng.generate_tokens([tokenizer.encode(prompt)], gen)[0])

    return run


def run_bootstrap_loop(generate: Callable[[str], str], question: str,
                       model_final: bool = False) -> Dict[str, Any]:
    """One question through reflect -> tool -> answer; the result records
    every turn and either ``final`` or an ``error`` string."""
    rec: Dict[str, Any] = {"question": question}
    prompt = f"User:\n{question}\n\nAssistant:\n"
    rec["first"] = first = generate(prompt)
    try:
        call = parse_tool_call(first)
    except ToolCallParseError as e:
        rec["error"] = f"invalid_tool_json: {e}"
        return rec
    if call is None:                       # plain chat answer
        rec.update(tool="chat", final=first.strip())
        return rec
    if call.name != "reflect":
        rec.update(tool_call=call.raw, error=f"expected_reflect_got_{call.name}")
        return rec
    restated = str(call.arguments.get("question", question))
    hint = extract_datetime_hint(restated)
    if hint is not None:
        suggestion = {"tool": "datetime", "arguments": {"op": hint.op, **hint.args}}
    else:
        expr = extract_arithmetic_expression(restated)
        if expr is None:
            rec.update(embedded=restated, error="reflect_extraction_failed")
            return rec
        suggestion = {"tool": "calculator", "arguments": {"expression": expr}}
    prompt2 = (f"{prompt}{first}\n\nTool result from reflect: "
               f"{json.dumps(suggestion, separators=(',', ':'))}\n\nAssistant:\n")
    rec["second"] = second = generate(prompt2)
    try:
        call2 = parse_tool_call(second)
    except ToolCallParseError as e:
        rec["error"] = f"invalid_2nd_tool: {e}"
        return rec
    if call2 is None or call2.name != suggestion["tool"]:
        rec["error"] = f"wrong_2nd_tool:{None if call2 is None else call2.name}"
        return rec
    rec.update(tool=call2.name, tool_call=call2.raw)
    try:
        if call2.name == "calculator":
            result = safe_calculator(str(call2.arguments.get("expression", "")).strip())
        else:
            a = {k: v for k, v in call2.arguments.items() if k != "op"}
            result = safe_datetime(str(call2.arguments.get("op", "")), **a)
    except (CalculatorError, DatetimeError, TypeError) as e:
        rec["error"] = str(e)
        return rec
    rec["tool_result"] = result
    if model_final:
        rec["final"] = generate(f"{prompt2}<tool_call>{call2.raw}</tool_call>\n\n"
                                f"Tool result from {call2.name}: {result}\n\nAssistant:\n")
    else:
        rec["final"] = f"The answer is {result}."
    return rec


# (question, expected tool, expected substring of the final answer)
EVAL_CASES: List[Tuple[str, str, str]] = [
    ("What is 17 + 25?", "calculator", "42"),
    ("How many days between 2026-01-01 and 2026-12-31?", "datetime", "364"),
    ("What is 12 * 12?", "calculator", "144"),
    ("What day of the week is 2027-01-01?", "datetime", "Friday"),
    ("Hello", "chat", ""),
    ("What is 100 - 58?", "calculator", "42"),
    ("What is 2026-05-20 plus 30 days?", "datetime", "2026-06-19"),
    ("Thanks for the help today.", "chat", ""),
]


def bootstrap_eval(generate: Callable[[str], str], max_cases: int = 8,
                   model_final: bool = False) -> Dict[str, Any]:
    """Tool choice and answer accuracy over ``EVAL_CASES``."""
    rows, tool_ok, ans_ok = [], 0, 0
    for q, tool, want in EVAL_CASES[:max_cases]:
        r = run_bootstrap_loop(generate, q, model_final)
        t = r.get("tool") == tool and "error" not in r
        a = t and want in str(r.get("final", ""))
        tool_ok += t
        ans_ok += a
        rows.append({**r, "expected_tool": tool, "tool_ok": t, "answer_ok": a})
    n = max(1, len(rows))
    return {"cases": rows, "tool_accuracy": tool_ok / n, "answer_accuracy": ans_ok / n}


def main(argv=None) -> Dict[str, Any]:
    from ..data.tokenization import get_tokenizer
    from ..models.builder import ComplexityModel

    ap = argparse.ArgumentParser(description="reflect-then-tool agent demo / eval")
    ap.add_argument("question", nargs="?", default="What is 17 + 25?")
    ap.add_argument("--checkpoint", required=True)
    ap.add_argument("--tokenizer", default="byte")
    ap.add_argument("--device", default="auto")
    ap.add_argument("--max-new-tokens", type=int, default=96)
    ap.add_argument("--temperature", type=float, default=0.2)
    ap.add_argument("--top-p", type=float, default=0.9)
    ap.add_argument("--eval", action="store_true")
    ap.add_argument("--max-cases", type=int, default=8)
    ap.add_argument("--model-final", action="store_true")
    a = ap.parse_args(argv)
    import torch

    dev = ("cuda" if torch.cuda.is_available() else "cpu") if a.device == "auto" else a.device
    tok = get_tokenizer("byte") if a.tokenizer == "byte" else get_tokenizer("huggingface", a.tokenizer)
    model = ComplexityModel.from_pretrained(a.checkpoint).to(dev)
    if dev.startswith("cuda"):
        model = model.to(torch.bfloat16)
    gen = engine_generator(model, tok, a.max_new_tokens, a.temperature, a.top_p)
    out = (bootstrap_eval(gen, a.max_cases, a.model_final) if a.eval
           else run_bootstrap_loop(gen, a.question, a.model_final))
    print(json.dumps(out, indent=2, default=str))
    return out


if __name__ == "__main__":
    main()
