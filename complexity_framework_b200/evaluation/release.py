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
"""
from __future__ import annotations

import argparse
import csv
import json
from pathlib import Path
from typing import Any, Dict, List, Optional

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


def main(argv=None) -> Dict[str, Any]:
    ap = argparse.ArgumentParser(description="select the SFT release checkpoint")
    ap.add_argument("--evaluation-root", required=True)
    ap.add_argument("--metrics", required=True)
    ap.add_argument("--checkpoint-root", required=True)
    ap.add_argument("--output", required=True)
    ap.add_argument("--expected-epochs", type=int)
    ap.add_argument("--selected-checkpoint", help="write the selected path to this file")
    a = ap.parse_args(argv)
    s = select_release_checkpoint(a.evaluation_root, a.metrics, a.checkpoint_root,
                                  a.expected_epochs)
    Path(a.output).write_text(json.dumps(s, indent=2) + "\n")
    if a.selected_checkpoint and s["selected"]:
        Path(a.selected_checkpoint).write_text(s["selected"]["checkpoint"] + "\n")
    print(json.dumps({"release_ready": s["release_ready"],
                      "selected_step": s["selected"]["step"] if s["selected"] else None}))
    return s


if __name__ == "__main__":
    main()
