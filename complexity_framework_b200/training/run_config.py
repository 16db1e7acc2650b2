"""YAML run configs merged into argparse, run fingerprints and diffs.

Counterpart of complexity/training/run_config.py:31-260: a YAML file supplies
defaults for any parser destination (command-line flags still win); the
resolved run config is written next to the checkpoints and, on resume,
compared with the stored one so silent hyper-parameter drift is reported.
"""
from __future__ import annotations

import argparse
import hashlib
import json
import subprocess
from pathlib import Path
from typing import Any, Dict, List, Optional, Sequence, Tuple

RUN_CONFIG_NAME = "run_config.json"
# keys whose change on resume is expected and not reported
_VOLATILE = {"resume", "max_steps", "save_steps", "log_steps", "checkpoint_dir", "wandb",
             "num_workers"}


def parser_destinations(parser: argparse.ArgumentParser) -> set:
    return {a.dest for a in parser._actions if a.dest != "help"}


def load_yaml_run_config(path, parser: argparse.ArgumentParser) -> Dict[str, Any]:
    import yaml

    raw = yaml.safe_load(Path(path).read_text()) or {}
    dests = parser_destinations(parser)
    out = {}
    for k, v in raw.items():
        key = k.replace("-", "_")
        if key not in dests:
            raise ValueError(f"unknown key {k!r} in run config {path}")
        out[key] = v
    return out


def parse_args_with_yaml_config(parser: argparse.ArgumentParser,
                                argv: Optional[Sequence[str]] = None) -> argparse.Namespace:
    """``--config run.yaml`` sets parser defaults; explicit flags override them."""
    pre = argparse.ArgumentParser(add_help=False)
    pre.add_argument("--config", default=None)
    known, _ = pre.parse_known_args(argv)
    if known.config:
        parser.set_defaults(**load_yaml_run_config(known.config, parser))
    if "config" not in parser_destinations(parser):
        parser.add_argument("--config", default=None, help="YAML run config")
    return parser.parse_args(argv)


def args_to_run_config(args: argparse.Namespace, extra: Optional[Dict] = None) -> Dict[str, Any]:
    d = {k: v for k, v in vars(args).items() if isinstance(v, (int, float, str, bool, type(None)))}
    d.update(extra or {})
    d["git_commit"] = current_git_commit()
    return d


def fingerprint(run_config: Dict[str, Any]) -> str:
    stable = {k: v for k, v in run_config.items() if k not in _VOLATILE and k != "git_commit"}
    return hashlib.sha256(json.dumps(stable, sort_keys=True).encode()).hexdigest()[:16]


def token_shard_fingerprint(path: Optional[str]) -> Optional[Dict[str, Any]]:
    if not path:
        return None
    from ..data.token_shards import read_token_shard_metadata

    try:
        m = read_token_shard_metadata(path)
    except (FileNotFoundError, ValueError):
        return None
    return {"num_tokens": m.get("num_tokens"), "sha256": m.get("sha256"), "dtype": m.get("dtype")}


def read_run_config(path) -> Dict[str, Any]:
    return json.loads(Path(path).read_text())


def write_run_config(path, run_config: Dict[str, Any]) -> None:
    Path(path).parent.mkdir(parents=True, exist_ok=True)
    Path(path).write_text(json.dumps(run_config, indent=2, sort_keys=True) + "\n")


def compare_run_configs(previous: Dict[str, Any], current: Dict[str, Any]) -> List[Tuple[str, Any, Any]]:
    keys = sorted((set(previous) | set(current)) - _VOLATILE - {"git_commit"})
    return [(k, previous.get(k), current.get(k)) for k in keys if previous.get(k) != current.get(k)]


def write_or_validate_run_config(checkpoint_dir, run_config: Dict[str, Any],
                                 strict: bool = False) -> List[Tuple[str, Any, Any]]:
    path = Path(checkpoint_dir) / RUN_CONFIG_NAME
    if path.exists():
        diffs = compare_run_configs(read_run_config(path), run_config)
        if diffs and strict:
            raise ValueError(f"run config changed on resume: {diffs}")
        return diffs
    write_run_config(path, run_config)
    return []


def format_run_summary(run_config: Dict[str, Any]) -> List[str]:
    return [f"{k:28s} {run_config[k]}" for k in sorted(run_config)]


def current_git_commit() -> Optional[str]:
    try:
        return subprocess.run(["git", "rev-parse", "HEAD"], capture_output=True, text=True,
                              timeout=5, cwd=Path(__file__).resolve().parent).stdout.strip() or None
    except (OSError, subprocess.SubprocessError):
        return None
