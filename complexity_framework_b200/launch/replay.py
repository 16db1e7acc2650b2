"""Replay plans for pretokenized mixtures and token-data verification.

``build_replay_plan`` turns per-source budgets into the replay-plan format
read by ``data.corpus_mixture.PretokenizedCorpusMixtureDataset``: each phase
takes a prefix of every source's shards (rows aligned down to
``row_alignment`` so phases divide evenly over ranks x workers) and repeats it
``passes`` times; the declared unique / trained token counts are written so
the dataset can check them.  ``verify_token_data`` re-hashes every shard of a
mixture (or of a plain token shard) against its manifest.

Counterparts: scripts/build_corrective_replay_plan.py and
scripts/verify_token_shards.py of the reference.
"""
from __future__ import annotations

import hashlib
import json
from pathlib import Path
from typing import Dict, List, Mapping, Sequence, Union

from ..data.corpus_mixture import MIXTURE_FORMAT, REPLAY_PLAN_FORMAT


def _manifest(root: Path) -> dict:
    m = json.loads((root / "mixture_manifest.json").read_text())
    if m.get("format") != MIXTURE_FORMAT:
        raise ValueError("not a pretokenized mixture")
    return m


def build_replay_plan(root: Union[str, Path], phases: Sequence[Mapping],
                      row_alignment: int = 512) -> dict:
    """``phases``: ``[{"name", "passes", "fractions": {source: fraction of its rows}}]``."""
    root = Path(root)
    m = _manifest(root)
    S = int(m["seq_len"])
    shards = {e["name"]: json.loads((root / e["manifest"]).read_text())["shards"]
              for e in m["sources"]}
    out_phases: List[dict] = []
    unique: Dict[tuple, int] = {}
    trained = 0
    for i, ph in enumerate(phases):
        name = ph.get("name", f"phase_{i + 1}")
        passes = int(ph.get("passes", 1))
        sel: Dict[str, List[dict]] = {}
        rows_phase = 0
        for src, frac in ph["fractions"].items():
            if src not in shards:
                raise ValueError(f"unknown source {src}")
            total = sum(int(s["rows"]) for s in shards[src])
            want = int(total * float(frac)) // row_alignment * row_alignment
            if want < 1:
                continue
            picks, left = [], want
            for s in shards[src]:
                take = min(left, int(s["rows"]))
                if take <= 0:
                    break
                picks.append({"file": s["file"], "rows": take})
                key = (src, s["file"])
                unique[key] = max(unique.get(key, 0), take)
                left -= take
            sel[src] = picks
            rows_phase += want
        if not sel:
            raise ValueError(f"phase {name} selects no rows")
        out_phases.append({"name": name, "passes": passes, "sources": sel})
        trained += rows_phase * passes
    return {"format": REPLAY_PLAN_FORMAT, "seq_len": S, "phases": out_phases,
            "unique_tokens": sum(unique.values()) * S, "trained_tokens": trained * S}


def verify_token_data(path: Union[str, Path]) -> dict:
    """Check sizes and sha256 of a mixture's shards or of one token shard."""
    path = Path(path)
    report = {"path": str(path), "files": 0, "bad": []}
    if (path / "mixture_manifest.json").exists():
        m = _manifest(path)
        for e in m["sources"]:
            sm_path = path / e["manifest"]
            sm = json.loads(sm_path.read_text())
            for s in sm["shards"]:
                f = sm_path.parent / s["file"]
                report["files"] += 1
                data = f.read_bytes() if f.exists() else b""
                if len(data) != int(s.get("bytes", int(s["tokens"]) * 2)):
                    report["bad"].append({"file": str(f), "problem": "size"})
                elif s.get("sha256") and hashlib.sha256(data).hexdigest() != s["sha256"]:
                    report["bad"].append({"file": str(f), "problem": "sha256"})
    else:
        from ..data.token_shards import read_token_shard_metadata

        meta = read_token_shard_metadata(path)
        f = path / meta.get("data_file", "tokens.bin")
        report["files"] = 1
        if meta.get("sha256"):
            h = hashlib.sha256()
            with open(f, "rb") as fh:
                for chunk in iter(lambda: fh.read(1 << 24), b""):
                    h.update(chunk)
            if h.hexdigest() != meta["sha256"]:
                report["bad"].append({"file": str(f), "problem": "sha256"})
    report["ok"] = not report["bad"]
    return report
