"""User documentation stays runnable: README Python examples parse, the
modules and CLI entry points it names exist, and local links resolve."""
import ast
import importlib
import re
from pathlib import Path

ROOT = Path(__file__).resolve().parents[1]
README = (ROOT / "README.md").read_text(encoding="utf-8")


def test_python_examples_parse():
    blocks = re.findall(r"```python\n(.*?)```", README, re.S)
    assert blocks
    for b in blocks:
        ast.parse(b)


def test_documented_modules_import():
    mods = set(re.findall(r"python -m (complexity_framework_b200(?:\.\w+)+)", README))
    mods |= set(re.findall(r"^(?:from|import) (complexity_framework_b200(?:\.\w+)*)", README, re.M))
    assert mods
    for m in sorted(mods):
        importlib.import_module(m)


def test_local_links_resolve():
    missing = []
    for target in re.findall(r"\]\(([^)#\s]+)(?:#[^)]*)?\)", README):
        if re.match(r"[a-z]+://", target):
            continue
        if not (ROOT / target).exists():
            missing.append(target)
    assert not missing, missing
