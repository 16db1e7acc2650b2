"""Behaviour regression gate for chat / SFT checkpoints.

    python -m complexity_framework_b200.evaluation.regression_gate panel.json \
        --model ckpt/ --piqa piqa.jsonl --out audit.json

Counterpart of complexity/scripts/check_sft_v2_regression.py:60-180 and its
panel file (configs/tr_hash_200m_sft_v2_regression.json).  A panel lists
prompts (a single ``prompt`` or a multi-turn ``messages`` history), each with
checks on the response; the gate passes when every response passes its
checks, the chat template was applied when the responses were generated, and
zero-shot PIQA acc_norm has not dropped more than ``maximum_absolute_drop``
below ``baseline_acc_norm``.  Panel and report layouts are the reference's,
so a panel or a generated report moves between frameworks.

Checks (case-insensitive substring tests unless noted):
``required_all``, ``required_any``, ``required_numbers`` (whole numbers, not
digits inside longer numbers), ``max_words``, ``exact_bullets`` with
``max_words_per_bullet``, and ``python_function`` + ``cases`` -- the
response's code (first fenced block, else the whole text) must define the
function and return ``expected`` for every ``args``.

Model-written code runs in a child interpreter (``python -I``) with a hard
wall-clock limit, builtins reduced to pure functions, and a static screen
first: no imports other than ``math``, no ``global`` / ``nonlocal`` /
``with``, no dunder attribute access.  The child runs under address-space
(1 GiB) and CPU-time limits, so an endless loop or a memory blow-up ends the
child, not the evaluator.
"""
from __future__ import annotations

import argparse
import ast
import json
import re
import subprocess
import sys
from pathlib import Path
from typing import Any, Dict, List, Mapping, Optional, Sequence

# builtins left to model-written code: pure functions and basic types only
_SAFE_BUILTINS = ("abs", "all", "any", "bool", "dict", "divmod", "enumerate", "filter",
                  "float", "int", "isinstance", "len", "list", "map", "max", "min", "pow",
                  "range", "reversed", "round", "set", "sorted", "str", "sum", "tuple", "zip",
                  "ValueError", "TypeError", "ZeroDivisionError", "Exception")

_CHILD = r"""
import builtins, json, sys
spec = json.loads(sys.stdin.read())
safe = {n: getattr(builtins, n) for n in spec["builtins"]}
def _imp(name, *a, **k):
    if name != "math":
        raise ImportError(name)
    return __import__(name)
safe["__import__"] = _imp
ns = {"__builtins__": safe}
try:
    exec(compile(spec["code"], "<response>", "exec"), ns, ns)
except Exception as e:
    print(json.dumps({"error": "python_exec_error:" + type(e).__name__})); sys.exit(0)
fn = ns.get(spec["function"])
if not callable(fn):
    print(json.dumps({"error": "missing_function:" + spec["function"]})); sys.exit(0)
for i, case in enumerate(spec["cases"]):
    try:
        got = fn(*case["args"])
    except Exception as e:
        print(json.dumps({"error": "case_%d_raised:%s" % (i, type(e).__name__)})); sys.exit(0)
    if got != case["expected"]:
        print(json.dumps({"error": "case_%d_expected_%r_got_%r" % (i, case["expected"], got)}))
        sys.exit(0)
print(json.dumps({"error": None}))
"""


def _limit_child(mem_bytes: int = 1 << 30, cpu_s: int = 5):
    """preexec hook: cap the child's address space and CPU time (POSIX)."""
    def apply():
        try:
            import resource

            resource.setrlimit(resource.RLIMIT_AS, (mem_bytes, mem_bytes))
            resource.setrlimit(resource.RLIMIT_CPU, (cpu_s, cpu_s))
        except (ImportError, ValueError, OSError):
            pass
    return apply


def _words(text: str) -> List[str]:
    return re.findall(r"[\w']+", text)


def extract_python(text: str) -> str:
    """The first fenced code block (```python / ```py / ```), else the text."""
    m = re.search(r"```(?:python|py)?[ \t]*\n(.*?)```", text, re.I | re.S)
    return (m.group(1) if m else text).strip()


def _screen(tree: ast.AST) -> Optional[str]:
    for node in ast.walk(tree):
        if isinstance(node, (ast.Global, ast.Nonlocal, ast.With, ast.AsyncWith)):
            return "unsafe_python_construct"
        if isinstance(node, ast.Import) and [a.name for a in node.names] != ["math"]:
            return "unsafe_python_import"
        if isinstance(node, ast.ImportFrom) and node.module != "math":
            return "unsafe_python_import"
        if isinstance(node, ast.Attribute) and node.attr.startswith("__"):
            return "unsafe_dunder_access"
    return None


def run_python_cases(text: str, function_name: str, cases: Sequence[Mapping[str, Any]],
                     timeout_s: float = 2.0) -> Optional[str]:
    """None when the response's ``function_name`` passes every case, else the
    first failure (syntax, screen, exec error, timeout, wrong value)."""
    code = extract_python(text)
    try:
        tree = ast.parse(code)
    except SyntaxError as e:
        return f"invalid_python:{e.msg}"
    bad = _screen(tree)
    if bad:
        return bad
    spec = json.dumps({"code": code, "function": function_name, "cases": list(cases),
                       "builtins": list(_SAFE_BUILTINS)})
    try:
        res = subprocess.run([sys.executable, "-I", "-c", _CHILD], input=spec, text=True,
                             capture_output=True, timeout=timeout_s,
                             preexec_fn=_limit_child() if sys.platform != "win32" else None)
    except subprocess.TimeoutExpired:
        return "python_timeout:TimeoutError"
    try:
        return json.loads(res.stdout.strip().splitlines()[-1])["error"]
    except (IndexError, ValueError, KeyError):
        return f"python_child_failed:{res.returncode}"


def check_response(item: Mapping[str, Any], response: str) -> List[str]:
    """Failed checks of one panel item (empty list = pass)."""
    if not response.strip():
        return ["empty_response"]
    c = item.get("checks", {})
    low = response.casefold()
    fails: List[str] = []
    if "required_all" in c:
        miss = [str(v) for v in c["required_all"] if str(v).casefold() not in low]
        if miss:
            fails.append("missing_all:" + ",".join(miss))
    if "required_any" in c and not any(str(v).casefold() in low for v in c["required_any"]):
        fails.append("missing_any:" + ",".join(map(str, c["required_any"])))
    for num in c.get("required_numbers", []):
        if not re.search(rf"(?<!\d){re.escape(str(num))}(?!\d)", response):
            fails.append(f"missing_number:{num}")
    if "max_words" in c and len(_words(response)) > int(c["max_words"]):
        fails.append(f"too_many_words:{len(_words(response))}")
    if "exact_bullets" in c:
        bullets = [ln for ln in response.splitlines() if re.match(r"^\s*[-*]\s+\S", ln)]
        if len(bullets) != int(c["exact_bullets"]):
            fails.append(f"bullet_count:{len(bullets)}")
        lim = int(c.get("max_words_per_bullet", 10 ** 9))
        long_ = [i for i, ln in enumerate(bullets)
                 if len(_words(re.sub(r"^\s*[-*]\s+", "", ln))) > lim]
        if long_:
            fails.append("long_bullets:" + ",".join(map(str, long_)))
    if "python_function" in c:
        f = run_python_cases(response, c["python_function"], c.get("cases", []))
        if f:
            fails.append(f)
    return fails


def audit_regression(panel: Mapping[str, Any], chat_report: Mapping[str, Any],
                     piqa_report: Mapping[str, Any]) -> Dict[str, Any]:
    """Combine the behaviour checks, the chat-template flag and the PIQA floor."""
    got = {str(r["id"]): str(r.get("response", "")) for r in chat_report.get("results", [])}
    failures: Dict[str, List[str]] = {}
    for item in panel["prompts"]:
        f = check_response(item, got.get(str(item["id"]), ""))
        if f:
            failures[str(item["id"])] = f
    p = panel["piqa"]
    score = float(piqa_report["benchmarks"]["piqa"]["acc_norm"])
    floor = float(p["baseline_acc_norm"]) - float(p["maximum_absolute_drop"])
    if score < floor:
        failures["piqa"] = [f"acc_norm:{score:.6f}<threshold:{floor:.6f}"]
    if chat_report.get("chat_template_applied") is not True:
        failures["chat_template"] = ["official_chat_template_not_applied"]
    return {"passed": not failures, "panel_id": panel.get("id"), "piqa_acc_norm": score,
            "piqa_threshold": floor, "failures": failures}


def generate_chat_report(model, tokenizer, panel: Mapping[str, Any],
                         chat_format: str = "complexity") -> Dict[str, Any]:
    """Responses to every panel prompt through the chat template and the
    paged engine, with the panel's generation settings (greedy at
    temperature 0)."""
    from ..data.tokenization import ChatTemplate
    from ..inference.engine import GenerationConfig, InferenceEngine

    g = panel.get("generation", {})
    temp = float(g.get("temperature", 0.0))
    gen = GenerationConfig(max_new_tokens=int(g.get("max_tokens", 256)), do_sample=temp > 0,
                           temperature=max(temp, 1e-5), top_p=float(g.get("top_p", 1.0)),
                           top_k=int(g.get("top_k", 0)),
                           repetition_penalty=float(g.get("repetition_penalty", 1.0)),
                           eos_token_id=getattr(tokenizer, "eos_token_id", None))
    tmpl, eng, results = ChatTemplate(chat_format), InferenceEngine(model), []
    for item in panel["prompts"]:
        msgs = item.get("messages") or [{"role": "user", "content": item["prompt"]}]
        ids = tokenizer.encode(tmpl.apply(msgs, add_generation_prompt=True))
        out = eng.generate_tokens([ids], gen)[0]
        results.append({"id": item["id"], "response": tokenizer.decode(out)})
    return {"chat_template_applied": True, "chat_format": chat_format, "results": results}


def main(argv=None) -> Dict[str, Any]:
    ap = argparse.ArgumentParser(description="SFT behaviour + PIQA regression gate")
    ap.add_argument("panel")
    ap.add_argument("--model", help="checkpoint to generate the chat report from")
    ap.add_argument("--chat-report", help="existing report JSON instead of --model")
    ap.add_argument("--piqa", help="PIQA JSONL to score with --model")
    ap.add_argument("--piqa-report", help="existing {benchmarks: {piqa: {acc_norm}}} JSON")
    ap.add_argument("--tokenizer", default="byte")
    ap.add_argument("--chat-format", default="complexity")
    ap.add_argument("--out")
    a = ap.parse_args(argv)
    panel = json.loads(Path(a.panel).read_text())
    model = tok = None
    if a.model:
        import torch

        from ..data.tokenization import get_tokenizer
        from ..models.builder import ComplexityModel

        tok = (get_tokenizer("byte") if a.tokenizer == "byte"
               else get_tokenizer("huggingface", a.tokenizer))
        model = ComplexityModel.from_pretrained(a.model)
        if torch.cuda.is_available():
            model = model.cuda().to(torch.bfloat16)
        model.eval()
    report = (json.loads(Path(a.chat_report).read_text()) if a.chat_report
              else generate_chat_report(model, tok, panel, a.chat_format))
    if a.piqa_report:
        piqa = json.loads(Path(a.piqa_report).read_text())
    else:
        from .benchmarks import PIQABenchmark

        res = PIQABenchmark(a.piqa).run(model, tok)
        piqa = {"benchmarks": {"piqa": {"acc_norm": res.accuracy, **res.details[-1]}}}
    audit = audit_regression(panel, report, piqa)
    text = json.dumps(audit, indent=2)
    if a.out:
        Path(a.out).write_text(text)
    print(text)
    return audit


if __name__ == "__main__":
    main()
