"""Pick the release checkpoint of an SFT run from its per-epoch evaluations.

    python -m complexity_framework_b200.evaluation.release --evaluation-root eval/ \
        --metrics metrics.csv --checkpoint-root ckpts/ --output selection.json

Counterpart of complexity/scripts/select_sft_v2_checkpoint.py:13-120.  Each
evaluated epoch has a directory ``epoch_<e>_step_<s>`` holding ``piqa.json``
(``checkpoint_step`` and ``benchmarks.piqa.{acc, acc_norm, correct,
correct_norm}``) and ``promotion.json`` (the regression gate's ``passed`` /
``failures``); the metrics CSV has ``step, matched_eval_loss,
matched_eval_ppl`` rows.  Only checkpoints that passed the gate are
eligible; among them the order is: highest PIQA acc_norm, then highest acc,
then lowest matched eval loss, then the earliest epoch.  With no eligible
checkpoint the run is not release-ready.

``export_release`` (and ``--export-to``) then packages the selected
checkpoint as a Hugging Face directory (counterpart of
complexity/scripts/export_sft_v2_release.py:145-275).
"""
from __future__ import annotations

import argparse
import csv
import hashlib
import json
import math
import shutil
from pathlib import Path
from typing import Any, Dict, List, Optional, Tuple

POLICY = ("promotion gate pass, then maximum PIQA acc_norm, maximum PIQA acc, "
          "minimum matched SFT eval loss, earliest epoch")


def checkpoint_for_step(root: Path, step: int) -> Optional[Path]:
    """The complete checkpoint directory of ``step``: the reference layout
    ``step_<6-digit step>/checkpoint.pt`` or this framework's ``<tag>-<step>``
    with its training state written."""
    ref = root / f"step_{step:06d}"
    if (ref / "checkpoint.pt").is_file():
        return ref
    for d in sorted(root.glob(f"*-{step}")):
        if (d / "training_state.json").is_file():
            return d
    return None


def _metrics(path: Path) -> Dict[int, Dict[str, str]]:
    with open(path, newline="", encoding="utf-8") as fh:
        return {int(r["step"]): r for r in csv.DictReader(fh) if r.get("step")}


def select_release_checkpoint(evaluation_root, metrics_path, checkpoint_root,
                              expected_epochs: Optional[int] = None) -> Dict[str, Any]:
    ev, ck = Path(evaluation_root), Path(checkpoint_root)
    rows = _metrics(Path(metrics_path))
    dirs = sorted(p for p in ev.glob("epoch_*_step_*") if p.is_dir())
    if expected_epochs is not None and len(dirs) != expected_epochs:
        raise ValueError(f"expected {expected_epochs} evaluated epochs, found {len(dirs)}")
    cands: List[Dict[str, Any]] = []
    seen = set()
    for epoch, d in enumerate(dirs, start=1):
        piqa_doc = json.loads((d / "piqa.json").read_text())
        gate = json.loads((d / "promotion.json").read_text())
        step = int(piqa_doc["checkpoint_step"])
        if step in seen:
            raise ValueError(f"step {step} evaluated twice")
        seen.add(step)
        path = checkpoint_for_step(ck, step)
        if path is None:
            raise FileNotFoundError(f"no complete checkpoint for step {step} under {ck}")
        row = rows.get(step)
        if not row or not row.get("matched_eval_loss"):
            raise ValueError(f"no matched eval metrics for step {step}")
        p = piqa_doc["benchmarks"]["piqa"]
        cands.append({"epoch": epoch, "step": step, "checkpoint": str(path.resolve()),
                      "promotion_passed": bool(gate["passed"]),
                      "promotion_failures": gate.get("failures", {}),
                      "piqa_acc": float(p["acc"]), "piqa_acc_norm": float(p["acc_norm"]),
                      "piqa_correct": int(p.get("correct", 0)),
                      "piqa_correct_norm": int(p.get("correct_norm", 0)),
                      "matched_eval_loss": float(row["matched_eval_loss"]),
                      "matched_eval_ppl": float(row.get("matched_eval_ppl") or "nan"),
                      "report_directory": str(d.resolve())})
    ok = [c for c in cands if c["promotion_passed"]]
    best = max(ok, key=lambda c: (c["piqa_acc_norm"], c["piqa_acc"], -c["matched_eval_loss"],
                                  -c["epoch"])) if ok else None
    return {"schema_version": 1, "selection_policy": POLICY, "release_ready": best is not None,
            "selected": best, "candidates": cands}


TOKENIZER_FILES = ("tokenizer.json", "tokenizer_config.json", "special_tokens_map.json",
                   "tokenizer.model", "vocab.json", "merges.txt", "tiktoken_config.json")


def _load_selected(ckpt: Path) -> Tuple[Dict[str, Any], Dict[str, Any], int, Dict[str, Any]]:
    """(state dict, model config dict, step, extras) of a checkpoint in this
    framework's layout or in the reference's (``checkpoint.pt`` holding
    ``model``, ``config``, ``step`` and optionally ``chat_template``)."""
    import torch

    if (ckpt / "model.safetensors").is_file() and (ckpt / "training_state.json").is_file():
        from safetensors.torch import load_file

        step = int(json.loads((ckpt / "training_state.json").read_text())["step"])
        cfg = json.loads((ckpt / "config.json").read_text())
        return load_file(str(ckpt / "model.safetensors")), cfg, step, {}
    st = torch.load(ckpt / "checkpoint.pt", map_location="cpu", weights_only=False)
    extras = {k: st[k] for k in ("chat_template",) if k in st}
    return st["model"], dict(st["config"]), int(st["step"]), extras


def _sha256(path: Path) -> str:
    h = hashlib.sha256()
    with open(path, "rb") as fh:
        for chunk in iter(lambda: fh.read(1 << 22), b""):
            h.update(chunk)
    return h.hexdigest()


def export_release(summary_path, output, *, tokenizer_dir=None, evaluation_root=None,
                   metrics_path=None, weights_dtype: Optional[str] = None,
                   release_name: str = "tr-hash-release") -> Dict[str, Any]:
    """Package the selected checkpoint of a release-ready selection summary as
    a Hugging Face directory: ``model.safetensors`` (one float dtype, fp32 or
    bf16, verified by reading it back), ``config.json`` for
    ``TRHashForCausalLM`` (the framework's ModelConfig fields flat, plus
    ``architectures``, ``num_experts_per_tok``, ``torch_dtype`` and the
    tokenizer's special-token ids), the tokenizer files, the evaluation
    reports, a README and ``release_manifest.json`` with the weights' sha256."""
    import torch
    from safetensors.torch import load_file, save_file

    from ..config.model_config import ModelConfig
    from ..integrations.hf import MODEL_TYPE, TRHashConfig

    summary = json.loads(Path(summary_path).read_text())
    sel = summary.get("selected")
    if not summary.get("release_ready") or not sel:
        raise ValueError("the selection summary does not authorise a release")
    out = Path(output)
    if out.exists():
        raise FileExistsError(out)
    sd, cfg, step, extras = _load_selected(Path(sel["checkpoint"]))
    if step != int(sel["step"]):
        raise ValueError(f"checkpoint is at step {step}, the selection says {sel['step']}")
    w = {k: v.detach().cpu().contiguous() for k, v in sd.items()}
    if weights_dtype is not None:
        dt = {"float32": torch.float32, "bfloat16": torch.bfloat16}[weights_dtype]
        w = {k: (v.to(dt) if v.is_floating_point() else v) for k, v in w.items()}
    fdt = {v.dtype for v in w.values() if v.is_floating_point()}
    names = {torch.float32: "float32", torch.bfloat16: "bfloat16"}
    if len(fdt) != 1 or next(iter(fdt)) not in names:
        raise ValueError(f"a release needs one float dtype (float32 or bfloat16), got {fdt}")
    dname = names[next(iter(fdt))]
    out.mkdir(parents=True)
    wpath = out / "model.safetensors"
    save_file(w, str(wpath), metadata={"format": "pt"})
    back = load_file(str(wpath))
    if back.keys() != w.keys() or any(not torch.equal(back[k], v) for k, v in w.items()):
        raise RuntimeError("safetensors read-back differs from the exported weights")
    mc = ModelConfig.from_dict(cfg)
    hf = TRHashConfig.from_model_config(mc).to_dict()
    hf.update(model_type=MODEL_TYPE, architectures=["TRHashForCausalLM"],
              num_experts_per_tok=mc.top_k, torch_dtype=dname)
    if tokenizer_dir is not None:
        tdir = Path(tokenizer_dir)
        tc = tdir / "tokenizer_config.json"
        if tc.is_file():
            t = json.loads(tc.read_text())
            ids = {v.get("content"): int(k) for k, v in t.get("added_tokens_decoder", {}).items()}
            for role in ("bos", "eos", "pad", "unk"):
                tok = t.get(f"{role}_token")
                tok = tok.get("content") if isinstance(tok, dict) else tok
                if tok in ids:
                    hf[f"{role}_token_id"] = ids[tok]
        for f in tdir.iterdir():
            if f.is_file() and f.name in TOKENIZER_FILES:
                shutil.copy2(f, out / f.name)
    (out / "config.json").write_text(json.dumps(hf, indent=2, sort_keys=True, default=str) + "\n")
    if "chat_template" in extras:
        (out / "chat_template.json").write_text(json.dumps(extras["chat_template"], indent=2) + "\n")
    rep = out / "reports"
    if evaluation_root is not None:
        shutil.copytree(evaluation_root, rep / "evaluations")
    if metrics_path is not None:
        rep.mkdir(parents=True, exist_ok=True)
        shutil.copy2(metrics_path, rep / "metrics.csv")
    rep.mkdir(parents=True, exist_ok=True)
    shutil.copy2(summary_path, rep / "selection_summary.json")
    if not math.isfinite(float(sel["matched_eval_loss"])):
        raise ValueError("the selected checkpoint has a non-finite eval loss")
    manifest = {
        "schema_version": 2, "release": release_name, "method": "full-parameter-sft",
        "selected_epoch": int(sel["epoch"]), "selected_step": step,
        "selection_policy": summary.get("selection_policy"),
        "piqa_acc": float(sel["piqa_acc"]), "piqa_acc_norm": float(sel["piqa_acc_norm"]),
        "matched_eval_loss": float(sel["matched_eval_loss"]),
        "matched_eval_ppl": float(sel.get("matched_eval_ppl", float("nan"))),
        "behavior_gate_passed": bool(sel["promotion_passed"]),
        "weights_sha256": _sha256(wpath), "weights_bytes": wpath.stat().st_size,
        "weights_dtype": dname,
        "floating_parameters": sum(v.numel() for v in w.values() if v.is_floating_point()),
        "parameters": sum(v.numel() for v in w.values()), "architecture": MODEL_TYPE,
        "num_experts": mc.num_experts, "num_experts_per_tok": mc.top_k}
    (out / "release_manifest.json").write_text(json.dumps(manifest, indent=2, sort_keys=True)
                                               + "\n")
    rows = "\n".join(f"| {c['epoch']} | {c['step']} | {c['piqa_acc_norm']:.4f} | "
                     f"{c['piqa_acc']:.4f} | {c['matched_eval_loss']:.4f} | "
                     f"{'yes' if c.get('promotion_passed') else 'no'} |"
                     for c in summary.get("candidates", []))
    (out / "README.md").write_text(
        f"---\nlicense: apache-2.0\n---\n# {release_name}\n\nLicense: Apache-2.0.\n\n"
        f"TR-Hash MoE, full-parameter SFT; selected epoch {sel['epoch']} (step {step}).\n"
        f"Selection: {summary.get('selection_policy')}.\n\n"
        "| epoch | step | PIQA acc_norm | PIQA acc | eval loss | gate |\n"
        f"|---|---|---|---|---|---|\n{rows}\n\nWeights: `model.safetensors` ({dname}, "
        f"sha256 `{manifest['weights_sha256']}`).\n")
    return manifest


def main(argv=None) -> Dict[str, Any]:
    ap = argparse.ArgumentParser(description="select the SFT release checkpoint")
    ap.add_argument("--evaluation-root", required=True)
    ap.add_argument("--metrics", required=True)
    ap.add_argument("--checkpoint-root", required=True)
    ap.add_argument("--output", required=True)
    ap.add_argument("--expected-epochs", type=int)
    ap.add_argument("--selected-checkpoint", help="write the selected path to this file")
    ap.add_argument("--export-to", help="package the selected checkpoint into this directory")
    ap.add_argument("--tokenizer-dir")
    ap.add_argument("--weights-dtype", choices=("float32", "bfloat16"))
    ap.add_argument("--release-name", default="tr-hash-release")
    a = ap.parse_args(argv)
    s = select_release_checkpoint(a.evaluation_root, a.metrics, a.checkpoint_root,
                                  a.expected_epochs)
    Path(a.output).write_text(json.dumps(s, indent=2) + "\n")
    if a.selected_checkpoint and s["selected"]:
        Path(a.selected_checkpoint).write_text(s["selected"]["checkpoint"] + "\n")
    if a.export_to and s["release_ready"]:
        export_release(a.output, a.export_to, tokenizer_dir=a.tokenizer_dir,
                       evaluation_root=a.evaluation_root, metrics_path=a.metrics,
                       weights_dtype=a.weights_dtype, release_name=a.release_name)
    print(json.dumps({"release_ready": s["release_ready"],
                      "selected_step": s["selected"]["step"] if s["selected"] else None}))
    return s


if __name__ == "__main__":
    main()
