"""Verified tool-use episodes and rewards for online RL.

Counterpart: complexity/inference/tool_rewards.py:1-215.  A question that a
deterministic tool can answer (arithmetic, ISO-date arithmetic) becomes a
``VerifiedToolEpisode`` whose target response is the tool-call transcript
``<tool_call>{json}</tool_call>`` / ``Tool result from <tool>: r`` /
``Assistant:\\nr`` (that text is a format the SFT/RL data share, so it is
kept identical).  ``tool_call_reward`` scores a model completion: it parses
the first tool call, re-runs the tool itself, and pays for a well-formed call,
a call whose result equals the verified answer, and a final answer equal to it.

The calculator evaluates a whitelisted arithmetic AST (no names, calls or
attributes; exponents bounded), so untrusted model text is never executed.
"""
from __future__ import annotations

import ast
import json
import operator
import re
from dataclasses import dataclass, field
from datetime import date, timedelta
from typing import Any, Callable, Dict, List, Optional


class CalculatorError(ValueError):
    pass


class DatetimeError(ValueError):
    pass


@dataclass
class VerifiedToolEpisode:
    prompt: str
    target_response: str
    reward: float
    tool_call: Dict[str, Any]
    tool_result: Dict[str, Any]
    metadata: Dict[str, Any] = field(default_factory=dict)


_DATE = re.compile(r"\d{4}-\d{2}-\d{2}")
_INT = re.compile(r"-?\d+")
_LEAD = re.compile(r"(?:what is|calculate|compute|tell me|how much is|combien fait|calcule)\s+(.+)$",
                   re.IGNORECASE)
_ARITH_CHARS = frozenset("0123456789+-*/().% ")
WEEKDAYS = ("Monday", "Tuesday", "Wednesday", "Thursday", "Friday", "Saturday", "Sunday")


# ------------------------------------------------------------------ calculator
def extract_arithmetic_expression(question: str) -> Optional[str]:
    """The arithmetic expression a question asks for (None for date questions
    or text without both a digit and an operator)."""
    if _DATE.search(question):
        return None
    text = question.strip().rstrip("?")
    m = _LEAD.search(text)
    if m:
        text = m.group(1)
    expr = "".join(c for c in text if c in _ARITH_CHARS).replace(" ", "")
    if any(c.isdigit() for c in expr) and any(op in expr for op in "+-*/%"):
        return expr
    return None


_BIN = {ast.Add: operator.add, ast.Sub: operator.sub, ast.Mult: operator.mul,
        ast.Div: operator.truediv, ast.FloorDiv: operator.floordiv, ast.Mod: operator.mod,
        ast.Pow: operator.pow}
_UN = {ast.USub: operator.neg, ast.UAdd: operator.pos}


def safe_calculator(expression: str) -> str:
    def ev(n):
        if isinstance(n, ast.Constant) and type(n.value) in (int, float):
            return n.value
        if isinstance(n, ast.UnaryOp) and type(n.op) in _UN:
            return _UN[type(n.op)](ev(n.operand))
        if isinstance(n, ast.BinOp) and type(n.op) in _BIN:
            a, b = ev(n.left), ev(n.right)
            if isinstance(n.op, ast.Pow) and abs(b) > 10:
                raise CalculatorError("power too large")
            return _BIN[type(n.op)](a, b)
        raise CalculatorError(f"unsupported expression: {expression!r}")

    try:
        value = ev(ast.parse(expression, mode="eval").body)
    except ZeroDivisionError as e:
        raise CalculatorError("division by zero") from e
    except SyntaxError as e:
        raise CalculatorError(f"invalid expression: {expression!r}") from e
    if isinstance(value, float) and value.is_integer():
        value = int(value)
    return str(value)


# -------------------------------------------------------------------- datetime
@dataclass
class DatetimeHint:
    op: str
    args: Dict[str, Any]


def extract_datetime_hint(question: str) -> Optional[DatetimeHint]:
    dates = _DATE.findall(question)
    if not dates:
        return None
    q = question.lower()
    if any(k in q for k in ("day of the week", "weekday", "jour de la semaine")):
        return DatetimeHint("weekday", {"date": dates[0]})
    if len(dates) >= 2 and any(k in q for k in ("between", "difference", "from ", "entre",
                                                "différence")):
        return DatetimeHint("diff", {"a": dates[0], "b": dates[1]})
    if "day" in q and any(k in q for k in ("plus", "add", "after", "après")):
        n = [int(x) for x in _INT.findall(_DATE.sub("", question))]
        if n:
            return DatetimeHint("add_days", {"date": dates[0], "days": n[0]})
    return None


def safe_datetime(op: str, **args: Any) -> str:
    try:
        if op == "diff":
            return str((date.fromisoformat(str(args["b"])) - date.fromisoformat(str(args["a"]))).days)
        if op == "add_days":
            return (date.fromisoformat(str(args["date"])) + timedelta(days=int(args["days"]))).isoformat()
        if op == "weekday":
            return WEEKDAYS[date.fromisoformat(str(args["date"])).weekday()]
    except (KeyError, ValueError, TypeError) as e:
        raise DatetimeError(f"invalid datetime args op={op} args={args}: {e}") from e
    raise DatetimeError(f"unknown datetime op: {op!r}")


TOOLS: Dict[str, Callable[..., str]] = {
    "calculator": lambda expression: safe_calculator(str(expression)),
    "datetime": lambda op, **a: safe_datetime(op, **a),
}


# -------------------------------------------------------------------- episodes
def _arg_json(args: Dict[str, Any]) -> str:
    # compact JSON with the argument order of the call (strings quoted, ints bare)
    return "{" + ",".join(f'"{k}":' + (f'"{v}"' if isinstance(v, str) else str(v))
                          for k, v in args.items()) + "}"


def _episode(prompt: str, name: str, args: Dict[str, Any], result: str,
             meta: Dict[str, Any]) -> VerifiedToolEpisode:
    text = (f'<tool_call>{{"name":"{name}","arguments":{_arg_json(args)}}}</tool_call>\n'
            f"Tool result from {name}: {result}\nAssistant:\n{result}")
    return VerifiedToolEpisode(prompt, text, 1.0, {"name": name, "arguments": dict(args)},
                               {"name": name, "result": result},
                               dict(meta, verified_tool=name, expected=result))


def build_calculator_episode(prompt: str, question: str) -> Optional[VerifiedToolEpisode]:
    expr = extract_arithmetic_expression(question)
    if expr is None:
        return None
    return _episode(prompt, "calculator", {"expression": expr}, safe_calculator(expr),
                    {"expression": expr})


def build_datetime_episode(prompt: str, question: str) -> Optional[VerifiedToolEpisode]:
    hint = extract_datetime_hint(question)
    if hint is None:
        return None
    return _episode(prompt, "datetime", {"op": hint.op, **hint.args},
                    safe_datetime(hint.op, **hint.args), {"op": hint.op, "arguments": hint.args})


def build_verified_tool_episode(prompt: str, question: str) -> Optional[VerifiedToolEpisode]:
    return build_datetime_episode(prompt, question) or build_calculator_episode(prompt, question)


# ---------------------------------------------------------------------- reward
_CALL = re.compile(r"<tool_call>(.*?)</tool_call>", re.DOTALL)


def parse_tool_call(text: str) -> Optional[Dict[str, Any]]:
    m = _CALL.search(text)
    if not m:
        return None
    try:
        call = json.loads(m.group(1))
    except json.JSONDecodeError:
        return None
    if not isinstance(call, dict) or not isinstance(call.get("arguments"), dict):
        return None
    return call if call.get("name") in TOOLS else None


def tool_call_reward(completion: str, episode: VerifiedToolEpisode,
                     weights=(0.2, 0.4, 0.4)) -> float:
    """w0 for a well-formed call of the episode's tool, w1 when running that
    call gives the verified result, w2 when the text after the last
    ``Assistant:`` marker (or the whole completion) equals the result."""
    expected = str(episode.tool_result["result"])
    r = 0.0
    call = parse_tool_call(completion)
    if call is not None and call["name"] == episode.tool_call["name"]:
        r += weights[0]
        try:
            if TOOLS[call["name"]](**call["arguments"]) == expected:
                r += weights[1]
        except (CalculatorError, DatetimeError, TypeError):
            pass
    final = completion.rsplit("Assistant:", 1)[-1].strip()
    if final == expected:
        r += weights[2]
    return r


def batch_tool_rewards(completions: List[str], episode: VerifiedToolEpisode) -> List[float]:
    """Batch form for a GRPO group sampled from one prompt."""
    return [tool_call_reward(c, episode) for c in completions]
