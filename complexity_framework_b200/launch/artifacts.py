"""Collect the artifacts of a finished pretraining run into one directory
with provenance.

    python -m complexity_framework_b200.launch.artifacts --run-name tr-hash-200m \
        --checkpoint ckpts/final-100000 --run-dir runs/200m --data-root data/ \
        --tokenizer tok/ --output-dir release/

Counterpart of complexity/scripts/collect_200m_run_artifacts.py:34-200.  The
output holds:

* ``model.safetensors``: the model weights only (no optimizer state); tensors
  that share storage (a tied LM head) are written as separate copies, since
  safetensors stores no aliases;
* ``model_config.json``: ``{"checkpoint_step", "model": <ModelConfig dict>}``;
* the run directory's logs and metrics (``*.csv``, ``*.jsonl``, ``*.json``,
  ``*.log``, ``*.yaml``) under their relative paths;
* the token shards' index / manifest files (``*.json`` under ``--data-root``,
  not the token payload) under ``dataset/``;
* the tokenizer files under ``tokenizer/``;
* ``artifact_manifest.json``: run name, source checkpoint with its sha256,
  and every released file with size and sha256.
"""
from __future__ import annotations

import argparse
import hashlib
import json
import shutil
from pathlib import Path
from typing import Any, Dict, Iterable, List, Optional

RUN_FILE_SUFFIXES = (".csv", ".jsonl", ".json", ".log", ".yaml", ".yml")


def sha256(path: Path, chunk: int = 1 << 24) -> str:
    h = hashlib.sha256()
    with open(path, "rb") as fh:
        for b in iter(lambda: fh.read(chunk), b""):
            h.update(b)
    return h.hexdigest()


def _copy(src: Path, dst: Path) -> Path:
    dst.parent.mkdir(parents=True, exist_ok=True)
    shutil.copy2(src, dst)
    return dst


def _model_weights(ckpt: Path):
    """(state dict, model config dict, step) of a checkpoint directory in this
    framework's layout or the reference's ``checkpoint.pt``."""
    import torch

    if (ckpt / "model.safetensors").is_file() and (ckpt / "training_state.json").is_file():
        from safetensors.torch import load_file

        step = int(json.loads((ckpt / "training_state.json").read_text())["step"])
        return (load_file(str(ckpt / "model.safetensors")),
                json.loads((ckpt / "config.json").read_text()), step, ckpt / "model.safetensors")
    st = torch.load(ckpt / "checkpoint.pt", map_location="cpu", weights_only=False)
    return st["model"], dict(st.get("config", {})), int(st.get("step", 0)), ckpt / "checkpoint.pt"


def _files(root: Path, suffixes: Iterable[str]) -> List[Path]:
    return sorted(p for p in root.rglob("*") if p.is_file() and p.suffix in tuple(suffixes))


def collect_run_artifacts(run_name: str, checkpoint: str, run_dir: str, output_dir: str,
                          data_root: Optional[str] = None,
                          tokenizer: Optional[str] = None) -> Dict[str, Any]:
    from safetensors.torch import save_file

    out, ck = Path(output_dir), Path(checkpoint)
    if out.exists() and any(out.iterdir()):
        raise FileExistsError(f"{out} is not empty")
    out.mkdir(parents=True, exist_ok=True)
    sd, cfg, step, source = _model_weights(ck)
    # separate storage for every tensor: tied weights become two equal tensors
    weights = {k: v.detach().cpu().clone().contiguous() for k, v in sd.items()}
    save_file(weights, str(out / "model.safetensors"), metadata={"format": "pt"})
    (out / "model_config.json").write_text(
        json.dumps({"checkpoint_step": step, "model": cfg}, indent=2, sort_keys=True) + "\n")
    run = Path(run_dir)
    for f in _files(run, RUN_FILE_SUFFIXES):
        if out in f.parents:
            continue
        _copy(f, out / f.relative_to(run))
    if data_root is not None:
        d = Path(data_root)
        for f in _files(d, (".json",)):
            _copy(f, out / "dataset" / f.relative_to(d))
    if tokenizer is not None:
        t = Path(tokenizer)
        for f in ([t] if t.is_file() else sorted(p for p in t.iterdir() if p.is_file())):
            _copy(f, out / "tokenizer" / f.name)
    released = []
    for f in sorted(p for p in out.rglob("*") if p.is_file()):
        released.append({"path": f.relative_to(out).as_posix(), "bytes": f.stat().st_size,
                         "sha256": sha256(f)})
    manifest = {"schema_version": 1, "run_name": run_name, "checkpoint_step": step,
                "checkpoint": {"path": str(source.resolve()), "sha256": sha256(source)},
                "files": released}
    (out / "artifact_manifest.json").write_text(json.dumps(manifest, indent=2) + "\n")
    return manifest


def main(argv=None) -> Dict[str, Any]:
    ap = argparse.ArgumentParser(description="collect a run's artifacts with provenance")
    ap.add_argument("--run-name", required=True)
    ap.add_argument("--checkpoint", required=True, help="checkpoint directory")
    ap.add_argument("--run-dir", required=True)
    ap.add_argument("--output-dir", required=True)
    ap.add_argument("--data-root")
    ap.add_argument("--tokenizer")
    a = ap.parse_args(argv)
    m = collect_run_artifacts(a.run_name, a.checkpoint, a.run_dir, a.output_dir, a.data_root,
                              a.tokenizer)
    print(json.dumps({"files": len(m["files"]), "checkpoint_step": m["checkpoint_step"]}))
    return m


if __name__ == "__main__":
    main()
